"""The single-process prefix-reuse demo (reference: src/__main__.py): request B, on another
engine, takes the three shared-prefix blocks request A wrote back to the pool and prefills only
its last block; its output equals a cold run of the same prompt."""
from lake_b200 import demo
from lake_b200.engine.llm_engine import LLMEngine


def test_the_second_request_reuses_the_shared_prefix_from_the_pool():
    r = demo.run()
    assert (r["A"]["reused_blocks"], r["A"]["prefill_blocks"], r["A"]["pool_prefix_blocks"]) == (0, 4, 0)
    assert (r["B"]["reused_blocks"], r["B"]["prefill_blocks"], r["B"]["pool_prefix_blocks"]) == (3, 1, 3)
    assert r["pool_durable_blocks"] == 3
    cold = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=256, max_model_len=512, num_blocks=64)
    assert cold.generate([list(range(1, 49)) + [200, 201]], max_new_tokens=4)[0] == r["B"]["output"]
