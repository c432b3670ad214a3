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


def test_engine_overlap_matches_synchronous(cuda_dev):
    """Overlapped steps on the GPU (graph replays whose PENDING inputs the token relay kernel
    resolves from the previous step's device output) give the synchronous engine's tokens."""
    rng = random.Random(4)
    prompts = [[rng.randrange(1000) for _ in range(n)] for n in (1, 30, 77, 150, 5, 64, 9)]
    outs = []
    for overlap in (False, True):
        eng = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=200, max_model_len=1024,
                        num_blocks=256, use_cuda_graphs=True, overlap=overlap)
        eng.runner.capture_graphs()
        outs.append(eng.generate(prompts, max_new_tokens=12))
        torch.cuda.synchronize()
    assert outs[0] == outs[1]


def test_engine_llama8b_shapes_two_layers(cuda_dev):
    eng = LLMEngine("llama3-8b", device="cuda:0", max_running=4, max_batched_tokens=512, max_model_len=1024,
                    num_blocks=128, model_overrides={"n_layers": 2})
    rng = random.Random(0)
    prompts = [[rng.randrange(eng.cfg.vocab) for _ in range(n)] for n in (100, 300)]
    outs = eng.generate(prompts, max_new_tokens=3)
    for p, o in zip(prompts, outs):
        _check_tokens(eng.model, p, o, tol_frac=0.15)


def test_moe_layer_grouped_gemm_matches_fp32(cuda_dev):
    """Router top-2 + gather + grouped expert GEMMs (SwiGLU, scatter) + combine vs fp32."""
    from lake_b200.models.llama import DecoderLM
    from lake_b200.models.config import get_config

    cfg = get_config("tiny-gpu", n_experts=4, top_k=2, arch="mixtral")
    m = DecoderLM(cfg, "cuda:0", torch.bfloat16, seed=1)
    t = 300
    ws = m.new_workspace(t + 8, 8)
    g = torch.Generator(device="cuda:0").manual_seed(0)
    x = torch.randn(t, cfg.hidden, device="cuda:0", generator=g).to(torch.bfloat16)
    h = torch.randn(t, cfg.hidden, device="cuda:0", generator=g).to(torch.bfloat16)
    h0 = h.float().cpu()
    m.moe.forward(0, x, h, ws, t)
    torch.cuda.synchronize()
    # fp32 reference on the same (interleaved) weights
    w = {k: v.float().cpu() for k, v in m.w.items()}
    xf = x.float().cpu()
    logits = xf @ w["layers.0.router"].t()
    topv, topi = logits.topk(2, dim=-1)
    wts = torch.softmax(topv, dim=-1)
    from lake_b200.oracle import ops_ref as ref
    out = torch.zeros_like(h0)
    for e in range(4):
        sel = (topi == e)
        rows = sel.any(-1).nonzero().flatten()
        act = ref.swiglu_from_interleaved(xf[rows] @ w["layers.0.experts.gate_up_proj"][e].t())
        y = act.to(torch.bfloat16).float() @ w["layers.0.experts.down_proj"][e].t()
        out[rows] += y * (wts * sel.float()).sum(-1)[rows][:, None]
    want = h0 + out
    err = (h.float().cpu() - want).abs().max().item()
    assert err < 0.05 * want.abs().max().item(), err
    assert int(ws.extra["moe_count"].sum()) == 2 * t


def test_engine_moe_matches_oracle(cuda_dev):
    eng = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=200, max_model_len=1024,
                    num_blocks=256, model_overrides={"n_experts": 4, "top_k": 2, "arch": "mixtral"})
    rng = random.Random(4)
    prompts = [[rng.randrange(eng.cfg.vocab) for _ in range(n)] for n in (1, 40, 130, 9)]
    outs = eng.generate(prompts, max_new_tokens=8)
    torch.cuda.synchronize()
    for p, o in zip(prompts, outs):
        _check_tokens(eng.model, p, o, tol_frac=0.1)


def test_engine_qwen3_qk_norm_matches_oracle(cuda_dev):
    """Qwen3-style per-head q/k RMSNorm fused into the QKV epilogue."""
    eng = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=200, max_model_len=1024,
                    num_blocks=256, model_overrides={"qk_norm": True, "arch": "qwen3"})
    rng = random.Random(6)
    prompts = [[rng.randrange(eng.cfg.vocab) for _ in range(n)] for n in (3, 60, 140)]
    outs = eng.generate(prompts, max_new_tokens=8)
    torch.cuda.synchronize()
    for p, o in zip(prompts, outs):
        _check_tokens(eng.model, p, o)


@pytest.mark.parametrize("w8a8", [False, True])
def test_engine_fp8_weights_match_dequantized_oracle(cuda_dev, w8a8):
    """Block-scaled e4m3 projection weights vs the oracle on the dequantised weights: W8A16 GEMMs
    (steps below the W8A8 threshold), and with the threshold at one row, W8A8 for every step
    (e4m3 activations per row and 128-column block, kind::f8f6f4 MMAs)."""
    from types import SimpleNamespace

    from lake_b200.ops._ext import native
    from lake_b200.ops.fp8 import Fp8Weight

    native().set_gemm_w8a8_min_m(1 if w8a8 else 256)
    try:
        eng = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=200, max_model_len=1024,
                        num_blocks=256, weight_dtype="fp8", use_cuda_graphs=not w8a8)
        assert isinstance(eng.model.w["layers.0.qkv_proj"], Fp8Weight)
        rng = random.Random(8)
        prompts = [[rng.randrange(eng.cfg.vocab) for _ in range(n)] for n in (5, 70, 130)]
        outs = eng.generate(prompts, max_new_tokens=6)
        torch.cuda.synchronize()
    finally:
        native().set_gemm_w8a8_min_m(256)
    oracle = SimpleNamespace(cfg=eng.model.cfg,
                             w={k: (v.dequant(torch.bfloat16, swiglu_tile=256) if isinstance(v, Fp8Weight) else v)
                                for k, v in eng.model.w.items()})
    for p, o in zip(prompts, outs):
        _check_tokens(oracle, p, o, tol_frac=0.12 if w8a8 else 0.08)


def test_kernel_write_behind_with_graph_decode(cuda_dev):
    """On the GPU the QKV epilogue (eager and graph-replayed decode steps) writes generated
    tokens' K/V into the pinned host tier through its device-mapped address; a later turn
    promoted from those pages decodes the same tokens as an engine without the tier."""
    import numpy as np

    from lake_b200.pool.agents.hostcache import HostCacheAgent
    from lake_b200.pool.pool_iface import PoolIface

    rng = np.random.default_rng(9)
    first = rng.integers(0, 2048, 40).tolist()
    eng = LLMEngine("tiny-gpu", device="cuda:0", max_running=4, max_batched_tokens=256, max_model_len=1024,
                    num_blocks=40)
    agent = HostCacheAgent(eng, l1_blocks=128)
    eng.attach_pool(PoolIface(agent))
    eng.runner.capture_graphs()
    out1 = eng.generate([first], max_new_tokens=60)[0]
    assert agent.stats["kernel_written_blocks"] == 3 and not agent.reserved
    for p in [rng.integers(0, 2048, 200).tolist() for _ in range(3)]:
        eng.generate([p], max_new_tokens=2)
    follow = first + out1 + rng.integers(0, 2048, 9).tolist()
    got = eng.generate([follow], max_new_tokens=6)[0]
    assert agent.stats["promoted_blocks"] >= 5
    ref = LLMEngine("tiny-gpu", device="cuda:0", max_running=4, max_batched_tokens=256, max_model_len=1024,
                    num_blocks=128, use_cuda_graphs=False)
    assert got == ref.generate([follow], max_new_tokens=6)[0]
