"""Tensor-parallel MLP block microbenchmark: fused NVLink collectives vs the
library path (cuBLAS + NCCL), one process per GPU.

One iteration is the row-parallel -> column-parallel hop of a Llama MLP with
sequence parallelism, for M tokens on a TP group of T GPUs:

  fused   : down GEMM whose epilogue pushes partial rows to their owners
            -> owner reduce + residual + RMSNorm + all-gather push
            -> gate_up GEMM (SwiGLU epilogue) that waits per row shard
  library : torch.matmul (cuBLAS) -> NCCL reduce_scatter -> residual add +
            RMSNorm (torch) -> NCCL all_gather -> torch.matmul -> SwiGLU (torch)

Timed with CUDA events on the launching stream, warm-up first, max over ranks.
Roofline: the slower of the GEMM FLOPs at the measured cuBLAS peak and the
bytes each GPU must send over NVLink at the measured 770 GB/s per direction.

    torchrun --nproc-per-node T -m lake_b200.bench.tp_layer --tokens 8192
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=14336)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    gloo = dist.new_group(backend="gloo")

    from lake_b200.ops import core
    from lake_b200.ops import tp as tpops
    from lake_b200.parallel.tp import TPGroup

    H, T = args.hidden, world
    I = args.inter // T
    M = args.tokens
    g = TPGroup(rank, world, dev, M + world, H, 8, group=gloo)
    mr = g.rows_per_rank(M)
    t = mr * T
    gen = torch.Generator(device=dev).manual_seed(rank)
    act = (torch.randn(t, I, device=dev, generator=gen) * 0.5).to(torch.bfloat16)
    w_down = (torch.randn(H, I, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    w_gu = (torch.randn(2 * I, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    w_n = torch.ones(H, dtype=torch.bfloat16, device=dev)
    h = torch.randn(mr, H, device=dev, generator=gen).to(torch.bfloat16)
    out_act = torch.empty(t, I, dtype=torch.bfloat16, device=dev)

    def fused():
        tpops.linear_rs(act, w_down, g.gemm_rs(0, mr, H, I))
        tpops.norm_push(h, w_n, 1e-5, g.norm_push(mr, 0, 0))
        tpops.linear_swiglu_ag(g.a_full[0][:t], w_gu, out_act, g.gemm_ag(0, mr))
        g.end_step()

    shard = torch.empty(mr, H, dtype=torch.bfloat16, device=dev)
    xfull = torch.empty(t, H, dtype=torch.bfloat16, device=dev)

    def library():
        part = act @ w_down.t()
        dist.reduce_scatter_tensor(shard, part)
        hh = h + shard
        x = (hh.float() * torch.rsqrt(hh.float().pow(2).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16) * w_n
        dist.all_gather_into_tensor(xfull, x)
        gu = (xfull @ w_gu.t()).view(t, -1, 2, 128)
        return torch.nn.functional.silu(gu[:, :, 0]) * gu[:, :, 1]

    # per-kernel split of the fused hop (CUDA events between the three launches, rank 0's view)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    split = [0.0, 0.0, 0.0]
    for it in range(args.warmup + args.iters):
        ev[0].record()
        tpops.linear_rs(act, w_down, g.gemm_rs(0, mr, H, I))
        ev[1].record()
        tpops.norm_push(h, w_n, 1e-5, g.norm_push(mr, 0, 0))
        ev[2].record()
        tpops.linear_swiglu_ag(g.a_full[0][:t], w_gu, out_act, g.gemm_ag(0, mr))
        g.end_step()
        ev[3].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            for j in range(3):
                split[j] += ev[j].elapsed_time(ev[j + 1]) / args.iters

    res = {}
    for name, fn in (("fused", fused), ("library", library)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / args.iters], dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=gloo)
        res[name] = ms.item()
    core.check_status(dev)
    if rank == 0:
        peaks = {}
        p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
        if os.path.exists(p):
            peaks = json.load(open(p))
        tflops = float(peaks.get("bf16_tflops", 1590.0))
        flops = 2.0 * t * I * H + 2.0 * t * H * 2 * I
        nvl_bytes = 2 * (T - 1) * mr * H * 2  # RS partials out + AG rows out, per GPU
        t_compute = flops / (tflops * 1e12) * 1e3
        t_link = nvl_bytes / 770e9 * 1e3
        roof = max(t_compute, t_link)
        print(json.dumps({"bench": "tp_mlp_hop", "tp": T, "tokens": M, "hidden": H, "inter_per_rank": I,
                          "fused_ms": round(res["fused"], 4), "library_ms": round(res["library"], 4),
                          "speedup": round(res["library"] / res["fused"], 3), "roofline_ms": round(roof, 4),
                          "fused_frac_of_roofline": round(roof / res["fused"], 3),
                          "compute_ms_at_peak": round(t_compute, 4), "nvlink_ms_at_770": round(t_link, 4),
                          "fused_split_ms": {"gemm_rs": round(split[0], 4), "norm_push": round(split[1], 4),
                                             "ag_gemm_swiglu": round(split[2], 4)},
                          "peak_source": "MEASURED_PEAKS.json" if peaks else "fallback 1590 TFLOP/s"}))
    dist.barrier(group=gloo)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
