"""End-to-end engine on the GPU against the dense fp32 oracle."""
import random

import pytest
import torch

from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.oracle.model_ref import dense_logits

pytestmark = pytest.mark.gpu


def _check_tokens(model, prompt, out, tol_frac=0.08):
    logits = dense_logits(model, prompt + out)
    lp = len(prompt)
    for i, tok in enumerate(out):
        row = logits[lp - 1 + i]
        gap = (row.max() - row[tok]).item()
        assert gap <= tol_frac * row.std().item(), f"token {i}: {tok} is {gap} below the oracle max"


@pytest.mark.parametrize("graphs", [False, True])
def test_engine_matches_oracle(cuda_dev, graphs):
    eng = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=200, max_model_len=1024,
                    num_blocks=256, use_cuda_graphs=graphs)
    rng = random.Random(3)
    prefix = [rng.randrange(eng.cfg.vocab) for _ in range(64)]
    prompts = [prefix + [rng.randrange(eng.cfg.vocab) for _ in range(n)] for n in (1, 30, 77, 150, 5)]
    outs = eng.generate(prompts, max_new_tokens=10)
    torch.cuda.synchronize()
    assert eng.pool.stats["hits"] > 0
    for p, o in zip(prompts, outs):
        _check_tokens(eng.model, p, o)


def test_engine_llama8b_shapes_two_layers(cuda_dev):
    eng = LLMEngine("llama3-8b", device="cuda:0", max_running=4, max_batched_tokens=512, max_model_len=1024,
                    num_blocks=128, model_overrides={"n_layers": 2})
    rng = random.Random(0)
    prompts = [[rng.randrange(eng.cfg.vocab) for _ in range(n)] for n in (100, 300)]
    outs = eng.generate(prompts, max_new_tokens=3)
    for p, o in zip(prompts, outs):
        _check_tokens(eng.model, p, o, tol_frac=0.15)
