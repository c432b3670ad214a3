"""Mixture-of-experts engine on CPU vs the dense fp32 oracle (tiny Mixtral-shaped model)."""
import random

from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.oracle.model_ref import greedy_generate


def test_moe_engine_matches_oracle_cpu():
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=64, max_model_len=512, num_blocks=64,
                    model_overrides={"n_experts": 4, "top_k": 2, "arch": "mixtral"})
    rng = random.Random(2)
    prompts = [[rng.randrange(1024) for _ in range(n)] for n in (5, 70, 23)]
    outs = eng.generate(prompts, max_new_tokens=5)
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(eng.model, p, 5)
