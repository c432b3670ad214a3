"""Qwen3-shaped model (q/k RMSNorm per head, tied embeddings) on the CPU path against the dense
fp32 oracle: chunked, paged, prefix-cached greedy generation equals dense recomputation
(reference: python/lake/engine/tests/test_qwen3_dummy.py:40-230 runs its Qwen3 shell with dummy
weights; here the forward is real and checked token by token)."""
import random

from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.models.config import get_config
from lake_b200.oracle.model_ref import greedy_generate


def test_qwen3_generation_matches_the_dense_oracle():
    cfg = get_config("tiny", arch="qwen3", qk_norm=True, tie_embeddings=True)
    eng = LLMEngine(cfg, device="cpu", max_running=4, max_batched_tokens=64, max_model_len=512, num_blocks=64,
                    seed=5)
    assert eng.model.w["lm_head"].data_ptr() == eng.model.w["embed_tokens"].data_ptr()
    for i in range(cfg.n_layers):  # non-trivial norm weights: a dropped or misplaced q/k norm changes tokens
        for n in ("q_norm", "k_norm"):
            eng.model.w[f"layers.{i}.{n}"].uniform_(0.5, 1.5)
    rng = random.Random(3)
    prefix = [rng.randrange(cfg.vocab) for _ in range(64)]
    prompts = [prefix + [rng.randrange(cfg.vocab) for _ in range(9 + 5 * i)] for i in range(3)]
    outs = eng.generate(prompts, max_new_tokens=6)
    assert eng.pool.stats["hits"] >= 4  # the shared prefix was served from the page cache
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(eng.model, p, 6)
