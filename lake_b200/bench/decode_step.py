"""Decode-step roofline on one GPU: a full Llama-3-8B decode iteration (CUDA-graph
replay of every layer, greedy sampling) over B running requests of context C,
against the bytes that step must move (all projection weights + lm_head once,
plus every running request's K/V pages) at the measured copy bandwidth.

Requests are adopted with pre-filled pages (the arena's contents do not change
the bytes moved), so the step is exactly what a PD-split decode instance runs.

    python -m lake_b200.bench.decode_step --batch 80 --ctx 2176
    python -m lake_b200.bench.decode_step --batch 80 --profile   # NVTX "decode_step" range, 3 steps
"""
from __future__ import annotations

import argparse
import json
import os
import random

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=80)
    ap.add_argument("--ctx", type=int, default=2176, help="tokens already in each request's KV pages")
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--weights", choices=["bf16", "fp8"], default="bf16")
    ap.add_argument("--profile", action="store_true")
    args = ap.parse_args(argv)

    from ..engine.llm_engine import LLMEngine
    from ..ops import core

    B, C = args.batch, args.ctx
    steps_total = args.warmup + (3 if args.profile else args.steps) + 2
    max_len = C + steps_total + 16
    eng = LLMEngine(args.model, device="cuda:0", max_running=B, max_batched_tokens=max(512, B),
                    max_model_len=max_len, num_blocks=B * ((max_len + 15) // 16) + 64, weight_dtype=args.weights)
    cfg = eng.cfg
    rng = random.Random(0)
    for i in range(B):
        blocks = eng.reserve_blocks(C)
        prompt = [rng.randrange(cfg.vocab) for _ in range(C)]
        eng.adopt_prefilled(f"d{i}", prompt, rng.randrange(cfg.vocab), blocks, max_new_tokens=10 ** 6)
    eng.runner.capture_graphs(max_bucket=B)
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    if args.profile:
        for _ in range(3):
            torch.cuda.nvtx.range_push("decode_step")
            eng.step()
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        core.check_status()
        print("profile steps done")
        return
    eng.runner.time_device = True
    times = []
    for _ in range(args.steps):
        out = eng.step()
        assert len(out) == B
        times.append(eng.runner.last_device_ms)
    core.check_status()
    times.sort()
    ms = times[len(times) // 2]
    # bytes a step must move: every weight except the embedding table (B rows of it), K/V of every request
    wbytes = 0
    for name, t in eng.model.w.items():
        if torch.is_tensor(t):
            n = t.numel() * t.element_size()
        else:  # block-scaled fp8: e4m3 bytes + fp32 scales
            n = t.q.numel() + t.s.numel() * 4
        wbytes += (B * cfg.hidden * 2) if name == "embed_tokens" else n
    kv_tok = cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2
    ctx_mid = C + args.warmup + args.steps // 2
    kvbytes = B * ctx_mid * kv_tok
    peaks = {}
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peaks = json.load(open(p))
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    roof_ms = (wbytes + kvbytes) / (hbm * 1e9) * 1e3
    print(json.dumps({"bench": "decode_step", "model": args.model, "weights": args.weights, "batch": B,
                      "ctx": ctx_mid, "ms_median": round(ms, 3), "ms_min": round(times[0], 3),
                      "tok_s": round(B / ms * 1e3, 1), "weight_gb": round(wbytes / 1e9, 2),
                      "kv_gb": round(kvbytes / 1e9, 2), "roofline_ms": round(roof_ms, 3),
                      "frac_of_roofline": round(roof_ms / ms, 3),
                      "hbm_source": "MEASURED_PEAKS.json" if peaks else "fallback 6650 GB/s"}))


if __name__ == "__main__":
    main()
