"""Kernel microbenchmarks on the current GPU: each sm_100a kernel against its
library counterpart (cuBLAS via torch.matmul, SDPA), timed with CUDA events
after warm-up, L2 flushed between iterations.

    python -m lake_b200.bench.kernels [--only gemm,decode,prefill,norm,moe]
    python -m lake_b200.bench.kernels --profile CASE   # 3 launches of one kernel, for an ncu capture

Profile cases (inputs larger than the 126 MB L2, a few GB on the device at most):
tp2_rs / tp2_norm / tp2_swiglu_ag / tp4_* (the fused tensor-parallel kernels of one MLP hop at
4096 tokens, driven from GPU 0), gemm_gate_up (M=4096 K=4096 N=28672), gemm_w8a8_gate_up (the same shape with block-scaled fp8
weights, W8A8), decode (256 seqs x 2304 ctx, 1 layer),
prefill_tc (4 x 2048), moe_decode (8 experts, 128 tokens top-2, grouped GEMM),
gemm_decode_qkv (M=80 QKV + RoPE + KV write, stream-K; 50 MB of weights: ncu flushes
the caches between passes, so its DRAM figures still count the weight stream).
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from .. import ops
from ..oracle import ops_ref as ref

BF = torch.bfloat16


class Timer:
    def __init__(self, iters=20, warmup=5):
        self.iters, self.warmup = iters, warmup
        self.flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    def __call__(self, fn):
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(self.iters):
            self.flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        times.sort()
        return times[len(times) // 2]


def bench_gemm(t: Timer, out: list):
    shapes = [(8192, 6144, 4096, "qkv"), (8192, 4096, 4096, "o_proj"), (8192, 28672, 4096, "gate_up"),
              (8192, 4096, 14336, "down"), (256, 6144, 4096, "decode_qkv"), (256, 28672, 4096, "decode_gate_up"),
              (256, 4096, 4096, "decode_o_proj"), (256, 4096, 14336, "decode_down"),
              (256, 128256, 4096, "decode_lm_head")]
    for m, n, k, name in shapes:
        a = torch.randn(m, k, device="cuda").to(BF)
        w = (torch.randn(n, k, device="cuda") / math.sqrt(k)).to(BF)
        c = torch.empty(m, n, device="cuda", dtype=BF)
        ms = t(lambda: ops.linear(a, w, out=c))
        ms_ref = t(lambda: torch.matmul(a, w.t(), out=c))
        fl = 2 * m * n * k
        byt = (m * k + n * k + m * n) * 2
        out.append(dict(kernel="gemm_bf16", shape=name, m=m, n=n, k=k, ms=ms, tflops=fl / ms / 1e9,
                        gbs=byt / ms / 1e6, cublas_ms=ms_ref, cublas_tflops=fl / ms_ref / 1e9))


def bench_gemm_fp8(t: Timer, out: list):
    """Block-scaled fp8 weights at prefill sizes: W8A8 (e4m3 activations, kind::f8f6f4 MMAs; the
    time includes quantising the activations) and W8A16 (weights dequantised to bf16 in shared
    memory) against the bf16 GEMM of the same shape."""
    from ..ops._ext import native
    from ..ops.fp8 import quantize_blockwise

    C = native()
    for m, n, k, name in [(8192, 6144, 4096, "qkv"), (8192, 4096, 4096, "o_proj"), (8192, 28672, 4096, "gate_up"),
                          (8192, 4096, 14336, "down")]:
        a = torch.randn(m, k, device="cuda").to(BF)
        w = (torch.randn(n, k, device="cuda") / math.sqrt(k)).to(BF)
        w8 = quantize_blockwise(w)
        c = torch.empty(m, n, device="cuda", dtype=BF)
        C.gemm_w8a8_reserve(m, k)
        ms_a8 = t(lambda: ops.linear(a, w8, out=c))
        C.set_gemm_w8a8_min_m(0)
        ms_a16 = t(lambda: ops.linear(a, w8, out=c))
        C.set_gemm_w8a8_min_m(256)
        ms_bf16 = t(lambda: ops.linear(a, w, out=c))
        fl = 2 * m * n * k
        out.append(dict(kernel="gemm_fp8", shape=name, m=m, n=n, k=k, w8a8_ms=ms_a8, w8a8_tflops=fl / ms_a8 / 1e9,
                        w8a16_ms=ms_a16, w8a16_tflops=fl / ms_a16 / 1e9, bf16_ms=ms_bf16,
                        bf16_tflops=fl / ms_bf16 / 1e9))


def bench_decode(t: Timer, out: list):
    for nseq, ctx in [(256, 2304), (64, 4096), (8, 8192)]:
        hq, hkv = 32, 8
        nb = (ctx + 15) // 16
        arena = torch.randn(nseq * nb + 1, 1, 2, hkv, 16, 128, device="cuda").to(BF)
        bt = torch.randperm(nseq * nb, device="cuda").view(nseq, nb).to(torch.int32)
        sl = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(nseq, hq * 128, device="cuda").to(BF)
        o = torch.empty_like(q)
        ms = t(lambda: ops.paged_decode_attention(q, arena, 0, bt, sl, hq, hkv, 0.088, out=o))
        byt = nseq * ctx * hkv * 128 * 2 * 2
        out.append(dict(kernel="paged_decode", nseq=nseq, ctx=ctx, ms=ms, gbs=byt / ms / 1e6))


def bench_prefill(t: Timer, out: list):
    """Causal prefill attention (Llama-3-8B heads, 32q/8kv): fresh prompts and prompts behind a
    cached prefix (residual queries). The tcgen05 kernels (two heads per CTA, and one head per
    CTA) against the warp-MMA kernel and torch SDPA (causal, same FLOPs, fresh prompts only)."""
    from ..ops._ext import native

    for nseq, prefix, new in [(4, 0, 2048), (1, 0, 8192), (4, 4096, 2048)]:
        hq, hkv = 32, 8
        ctx = prefix + new
        nb = (ctx + 15) // 16
        arena = torch.randn(nseq * nb + 1, 1, 2, hkv, 16, 128, device="cuda").to(BF)
        bt = torch.randperm(nseq * nb, device="cuda").view(nseq, nb).to(torch.int32)
        sl = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
        qs = [i * new for i in range(nseq + 1)]
        tiles = ops.build_prefill_tiles(qs, [prefix] * nseq, device="cuda")
        q = torch.randn(nseq * new, hq * 128, device="cuda").to(BF)
        o = torch.empty_like(q)
        qs_t = torch.tensor(qs, dtype=torch.int32, device="cuda")
        run = lambda: ops.paged_prefill_attention(q, arena, 0, bt, sl, tiles, qs_t, None, hq, hkv, 0.088, out=o)  # noqa
        ms = t(run)
        native().set_prefill_kernel(0)
        ms_one = t(run)
        variants = {}
        for v in range(6):  # softmax variants of the two-head kernel
            native().set_prefill_kernel(10 + v)
            variants[f"v{v}_ms"] = t(run)
        native().set_prefill_kernel(1)
        tiles64 = ops.build_prefill_tiles(qs, [prefix] * nseq, tile=64, device="cuda")
        ms_mma = t(lambda: ops.paged_prefill_attention(q, arena, 0, bt, sl, tiles64, qs_t, None, hq, hkv, 0.088,
                                                       out=o, tensor_core=False))
        # visible (query, key) pairs: row i of a prompt sees prefix + i + 1 keys
        pairs = nseq * (new * prefix + new * (new + 1) // 2)
        fl = 4 * pairs * hq * 128
        row = dict(kernel="paged_prefill", nseq=nseq, prefix=prefix, new=new, ms=ms, tflops=fl / ms / 1e9,
                   one_head_ms=ms_one, one_head_tflops=fl / ms_one / 1e9, warp_mma_tflops=fl / ms_mma / 1e9,
                   **variants)
        if prefix == 0:
            qd = q.view(nseq, new, hq, 128).transpose(1, 2)
            kd = torch.randn(nseq, hq, new, 128, device="cuda").to(BF)
            ms_ref = t(lambda: torch.nn.functional.scaled_dot_product_attention(qd, kd, kd, is_causal=True))
            row.update(sdpa_ms=ms_ref, sdpa_tflops=fl / ms_ref / 1e9, vs_sdpa=ms_ref / ms)
        out.append(row)


def prefill_timeline(t: Timer, out: list):
    """Per-tile timeline of the two-head prefill kernel's heaviest CTA (4 x 2048 causal, 16 K/V
    tiles) for each softmax variant: the kernel records SM clock cycles at each hand-off (scores
    ready, scores in registers, P computed, P handed over, MMA issuer sees P / K). Reports the
    median over the steady-state tiles (2-13) of each phase."""
    from ..ops._ext import native

    nseq, new, hq, hkv = 4, 2048, 32, 8
    nb = (new + 15) // 16
    arena = torch.randn(nseq * nb + 1, 1, 2, hkv, 16, 128, device="cuda").to(BF)
    bt = torch.randperm(nseq * nb, device="cuda").view(nseq, nb).to(torch.int32)
    sl = torch.full((nseq,), new, dtype=torch.int32, device="cuda")
    qs = [i * new for i in range(nseq + 1)]
    tiles = ops.build_prefill_tiles(qs, [0] * nseq, device="cuda")
    q = torch.randn(nseq * new, hq * 128, device="cuda").to(BF)
    o = torch.empty_like(q)
    qs_t = torch.tensor(qs, dtype=torch.int32, device="cuda")
    C = native()
    for v in range(6):
        C.set_prefill_kernel(10 + v)
        C.prefill_trace_enable(True)
        for _ in range(3):
            ops.paged_prefill_attention(q, arena, 0, bt, sl, tiles, qs_t, None, hq, hkv, 0.088, out=o)
        torch.cuda.synchronize()
        C.prefill_trace_enable(False)
        tr = C.prefill_trace().tolist()
        ev = [[tr[j * 16 + e] for e in range(16)] for j in range(16)]
        rows = []
        for j in range(2, 14):
            e = ev[j]
            rows.append(dict(
                a_wait_s=e[3] - ev[j - 1][6], a_ld=e[4] - e[3], a_exp=e[5] - e[4], a_st=e[6] - e[5],
                b_wait_s=e[7] - ev[j - 1][10], b_ld=e[8] - e[7], b_exp=e[9] - e[8], b_st=e[10] - e[9],
                mma_sees_pA=e[0] - e[6], mma_sees_pB=e[1] - e[10], period=ev[j][3] - ev[j - 1][3]))
        med = {k: sorted(r[k] for r in rows)[len(rows) // 2] for k in rows[0]}
        out.append(dict(kernel="prefill_pingpong timeline (cycles, median of tiles 2-13)", variant=v,
                        ms=t(lambda: ops.paged_prefill_attention(q, arena, 0, bt, sl, tiles, qs_t, None, hq, hkv,
                                                                 0.088, out=o)), **med))
    C.set_prefill_kernel(1)


def bench_norm(t: Timer, out: list):
    x = torch.randn(8192, 4096, device="cuda").to(BF)
    w = torch.rand(4096, device="cuda").to(BF)
    o = torch.empty_like(x)
    ms = t(lambda: ops.rms_norm(x, w, 1e-5, out=o))
    out.append(dict(kernel="rmsnorm", rows=8192, dim=4096, ms=ms, gbs=2 * x.numel() * 2 / ms / 1e6))


def _moe_case(tokens=128, hidden=4096, inter=14336, experts=8, top_k=2):
    from ..ops._ext import native

    C = native()
    cap = (tokens + 127) // 128 * 128
    x = torch.randn(tokens, hidden, device="cuda").to(BF)
    logits = torch.randn(tokens, 32, device="cuda")
    wts = torch.empty(tokens * top_k, device="cuda")
    count = torch.zeros(experts, dtype=torch.int32, device="cuda")
    gathered = torch.zeros(experts * cap, hidden, device="cuda", dtype=BF)
    slot = torch.zeros(experts * cap, dtype=torch.int32, device="cuda")
    gu = (torch.randn(experts, 2 * inter, hidden, device="cuda") * 0.02).to(BF)
    dn = (torch.randn(experts, hidden, inter, device="cuda") * 0.02).to(BF)
    act = torch.empty(experts * cap, inter, device="cuda", dtype=BF)
    comb = torch.empty(tokens * top_k, hidden, device="cuda", dtype=BF)
    h = torch.zeros(tokens, hidden, device="cuda", dtype=BF)

    def run():
        count.zero_()
        C.moe_dispatch(logits, x, wts, experts, top_k, cap, 1, 0, [gathered.data_ptr()], [slot.data_ptr()], [],
                       [count.data_ptr()], [])
        C.gemm_grouped(gathered, gu, act, 2, count, cap)
        C.gemm_grouped(act, dn, None, 7, count, cap, row_slot=slot, dst_ptrs=[comb.data_ptr()])
        C.moe_combine(h, comb, wts, top_k)

    wbytes = (gu.numel() + dn.numel()) * 2
    return run, wbytes


def bench_pd_qkv(t: Timer, out: list):
    """Fused P->D: the QKV GEMM epilogue writes K/V into this GPU's arena and, over NVLink, into a
    second GPU's arena (peer-mapped). Compared with the same GEMM writing only locally."""
    if torch.cuda.device_count() < 2:
        return
    from ..ops._ext import native

    torch.cuda.set_device(0)
    native().enable_peer_access(1)
    m, hq, hkv, hidden = 8192, 32, 8, 4096
    nb = m // 16
    arena = torch.zeros(nb + 1, 1, 2, hkv, 16, 128, device="cuda:0", dtype=BF)
    peer = torch.zeros(nb + 1, 1, 2, hkv, 16, 128, device="cuda:1", dtype=BF)
    x = torch.randn(m, hidden, device="cuda").to(BF)
    w = (torch.randn((hq + 2 * hkv) * 128, hidden, device="cuda") * 0.02).to(BF)
    q = torch.empty(m, hq * 128, device="cuda", dtype=BF)
    cs = ref.rope_cache(8192, 5e5, 128, None, device="cuda")
    pos = torch.arange(m, dtype=torch.int32, device="cuda") % 2048
    slots = torch.arange(m, dtype=torch.int64, device="cuda")
    ms_local = t(lambda: ops.linear_qkv(x, w, q, cs, pos, slots, arena, 0, hq, hkv))
    ms_peer = t(lambda: ops.linear_qkv(x, w, q, cs, pos, slots, arena, 0, hq, hkv, peer, slots))
    kv_bytes = m * 2 * hkv * 128 * 2
    fl = 2 * m * w.shape[0] * hidden
    # roofline of the fused kernel: the slower of the GEMM at the measured cuBLAS peak and the
    # K/V bytes that cross NVLink at the measured 770 GB/s peer-copy rate
    roof = max(fl / (_peak_tflops() * 1e12), kv_bytes / 770e9) * 1e3
    out.append(dict(kernel="linear_qkv + P->D peer KV stores", m=m, ms_local_only=ms_local, ms_with_peer=ms_peer,
                    tflops_with_peer=fl / ms_peer / 1e9, peer_kv_gbs=kv_bytes / ms_peer / 1e6,
                    overhead_frac=ms_peer / ms_local - 1, roofline_ms=roof, frac_of_roofline=roof / ms_peer))


def _peak_tflops() -> float:
    import os

    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p)).get("bf16_tflops", 1590.0))
    return 1590.0


def bench_moe(t: Timer, out: list):
    for tokens in (128, 1024):
        run, wbytes = _moe_case(tokens)
        ms = t(run)
        out.append(dict(kernel="moe_layer (dispatch+grouped gate_up+grouped down+combine)", tokens=tokens,
                        experts=8, ms=ms, weight_gbs=wbytes / ms / 1e6))


def _tp_case(world: int, what: str, tokens: int = 8192):
    """One fused tensor-parallel kernel of the Llama-3-8B MLP hop as TP rank 0 of `world`, driven
    from one process: GPU 0 runs the kernel and its P2P stores land in buffers on GPUs 1..world-1
    (peer access, as the IPC-mapped buffers of a real group). The other ranks never run, so their
    counter slots on GPU 0 are preset: GPU 0's waits pass at once and the capture shows the
    kernel's own work and NVLink traffic.
      rs   : down_proj GEMM (K = FFN / world) whose epilogue pushes each partial row to its owner
      norm : reduce of the world partials + residual + RMSNorm + all-gather push to every rank
      swiglu_ag : gate_up GEMM (N = 2 FFN / world) over the all-gathered rows + SwiGLU"""
    from ..ops import tp as tpops
    from ..ops._ext import native

    C = native()
    if torch.cuda.device_count() < world:
        raise SystemExit(f"needs {world} GPUs")
    torch.cuda.set_device(0)
    for d in range(1, world):
        C.enable_peer_access(d)
    H, I = 4096, 14336
    mr = tokens // world
    devs = [torch.device("cuda", d) for d in range(world)]
    recv = [torch.zeros(world * mr, H, dtype=BF, device=dv) for dv in devs]
    afull = [torch.zeros(world * mr, H, dtype=BF, device=dv) for dv in devs]
    cnt = [torch.zeros(2 * world, dtype=torch.int64, device=dv) for dv in devs]  # [rs world | ag world]
    cnt[0].fill_(1 << 60)
    ptr = [c.data_ptr() for c in cnt]
    if what == "rs":
        a = torch.randn(world * mr, I // world, device="cuda").to(BF)
        w = (torch.randn(H, I // world, device="cuda") * 0.02).to(BF)
        tp = dict(world=world, rank=0, rows_per_rank=mr, m_rot=(mr // 128) % max(1, (world * mr) // 128),
                  rs_recv=[r.data_ptr() for r in recv], rs_cnt=ptr)
        return lambda: tpops.linear_rs(a, w, tp), 2 * world * mr * H * (I // world)
    if what == "norm":
        h = torch.randn(mr, H, device="cuda").to(BF)
        wn = torch.ones(H, device="cuda").to(BF)
        tp = dict(world=world, rank=0, rows_per_rank=mr, dst=[x.data_ptr() for x in afull], dst_ld=H,
                  ag_cnt=[p + 8 * world for p in ptr], store_h=1, recv=recv[0].data_ptr(), rs_cnt=ptr[0], rs_off=1)
        return lambda: tpops.norm_push(h, wn, 1e-5, tp), 0
    if what == "swiglu_ag":
        wgu = (torch.randn(2 * I // world, H, device="cuda") * 0.02).to(BF)
        act = torch.empty(world * mr, I // world, device="cuda", dtype=BF)
        tp = dict(world=world, rank=0, rows_per_rank=mr, ag_cnt=ptr[0] + 8 * world, ag_off=1, m_rot=0)
        return lambda: tpops.linear_swiglu_ag(afull[0], wgu, act, tp), 2 * world * mr * (2 * I // world) * H
    raise SystemExit(f"unknown tensor-parallel case {what}")


def bench_tp_kernels(t: Timer, out: list):
    """The fused TP kernels of one MLP hop at TP = 2 and 4 (8192 tokens), each driven from GPU 0
    (see _tp_case): CUDA-event times, GEMM rates, and the bytes each kernel pushes over NVLink."""
    for world in (2, 4):
        if torch.cuda.device_count() < world:
            continue
        for what in ("rs", "norm", "swiglu_ag"):
            fn, fl = _tp_case(world, what)
            ms = t(fn)
            mr, H = 8192 // world, 4096
            nv = {"rs": (world - 1) * mr * H * 2, "norm": (world - 1) * mr * H * 2, "swiglu_ag": 0}[what]
            row = dict(kernel=f"tp{world}_{what}", tokens=8192, ms=ms, nvlink_mb=nv / 1e6,
                       nvlink_gbs=nv / ms / 1e6 if nv else None)
            if fl:
                row["tflops"] = fl / ms / 1e9
            out.append(row)
            torch.cuda.synchronize()
            ops.core.check_status()


def profile(case: str) -> None:
    """Three launches of one kernel on a small case (for `ncu -k <kernel> -c 3`)."""
    if case.startswith("tp") and case[2:3].isdigit():  # tp2_rs, tp4_norm, tp2_swiglu_ag, ...
        fn, _ = _tp_case(int(case[2]), case.split("_", 1)[1], tokens=4096)
    elif case == "gemm_gate_up":
        a = torch.randn(4096, 4096, device="cuda").to(BF)
        w = (torch.randn(28672, 4096, device="cuda") * 0.02).to(BF)
        c = torch.empty(4096, 28672, device="cuda", dtype=BF)
        fn = lambda: ops.linear(a, w, out=c)  # noqa: E731
    elif case == "gemm_w8a8_gate_up":
        # block-scaled fp8 weights, W8A8 (activation quantisation kernel + the fp8 MMA GEMM)
        from ..ops._ext import native
        from ..ops.fp8 import quantize_blockwise

        a = torch.randn(4096, 4096, device="cuda").to(BF)
        w8 = quantize_blockwise(torch.randn(28672, 4096, device="cuda") * 0.02)
        c = torch.empty(4096, 28672, device="cuda", dtype=BF)
        native().gemm_w8a8_reserve(4096, 4096)
        fn = lambda: ops.linear(a, w8, out=c)  # noqa: E731
    elif case == "decode":
        nseq, ctx, hq, hkv = 256, 2304, 32, 8
        nb = ctx // 16
        arena = torch.randn(nseq * nb + 1, 1, 2, hkv, 16, 128, device="cuda").to(BF)
        bt = torch.randperm(nseq * nb, device="cuda").view(nseq, nb).to(torch.int32)
        sl = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(nseq, hq * 128, device="cuda").to(BF)
        o = torch.empty_like(q)
        fn = lambda: ops.paged_decode_attention(q, arena, 0, bt, sl, hq, hkv, 0.088, out=o)  # noqa: E731
    elif case == "prefill_tc":
        nseq, ctx, hq, hkv = 4, 2048, 32, 8
        nb = ctx // 16
        arena = torch.randn(nseq * nb + 1, 1, 2, hkv, 16, 128, device="cuda").to(BF)
        bt = torch.randperm(nseq * nb, device="cuda").view(nseq, nb).to(torch.int32)
        sl = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
        qs = [i * ctx for i in range(nseq + 1)]
        tiles = ops.build_prefill_tiles(qs, [0] * nseq, device="cuda")
        q = torch.randn(nseq * ctx, hq * 128, device="cuda").to(BF)
        o = torch.empty_like(q)
        qs_t = torch.tensor(qs, dtype=torch.int32, device="cuda")
        fn = lambda: ops.paged_prefill_attention(q, arena, 0, bt, sl, tiles, qs_t, None, hq, hkv, 0.088,  # noqa
                                                 out=o)
    elif case == "gemm_decode_qkv":
        # decode-size QKV projection (80 tokens, 4096 -> 6144) with RoPE + paged KV write: stream-K
        m, hq, hkv, hidden = 80, 32, 8, 4096
        x = torch.randn(m, hidden, device="cuda").to(BF)
        w = (torch.randn((hq + 2 * hkv) * 128, hidden, device="cuda") * 0.02).to(BF)
        q = torch.empty(m, hq * 128, device="cuda", dtype=BF)
        arena = torch.zeros(m // 16 + 1, 1, 2, hkv, 16, 128, device="cuda", dtype=BF)
        cs = ref.rope_cache(4096, 5e5, 128, None, device="cuda")
        pos = torch.arange(m, dtype=torch.int32, device="cuda") + 2000
        slots = torch.arange(m, dtype=torch.int64, device="cuda")
        fn = lambda: ops.linear_qkv(x, w, q, cs, pos, slots, arena, 0, hq, hkv)  # noqa: E731
    elif case == "pd_qkv":
        # fused P->D at 4096 prompt tokens: QKV GEMM + RoPE + K/V to this GPU's and GPU 1's arena
        from ..ops._ext import native

        native().enable_peer_access(1)
        m, hq, hkv, hidden = 4096, 32, 8, 4096
        nb = m // 16
        arena = torch.zeros(nb + 1, 1, 2, hkv, 16, 128, device="cuda:0", dtype=BF)
        peer = torch.zeros(nb + 1, 1, 2, hkv, 16, 128, device="cuda:1", dtype=BF)
        x = torch.randn(m, hidden, device="cuda").to(BF)
        w = (torch.randn((hq + 2 * hkv) * 128, hidden, device="cuda") * 0.02).to(BF)
        q = torch.empty(m, hq * 128, device="cuda", dtype=BF)
        cs = ref.rope_cache(8192, 5e5, 128, None, device="cuda")
        pos = torch.arange(m, dtype=torch.int32, device="cuda")
        slots = torch.arange(m, dtype=torch.int64, device="cuda")
        fn = lambda: ops.linear_qkv(x, w, q, cs, pos, slots, arena, 0, hq, hkv, peer, slots)  # noqa: E731
    elif case == "moe_decode":
        fn, _ = _moe_case(128)
    else:
        raise SystemExit(f"unknown profile case {case}")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ops.core.check_status()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,decode,prefill,norm,moe")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--profile", default=None)
    args = ap.parse_args(argv)
    if args.profile:
        profile(args.profile)
        return
    t = Timer(args.iters)
    res: list = []
    for name in args.only.split(","):
        {"gemm": bench_gemm, "gemm_fp8": bench_gemm_fp8, "decode": bench_decode, "prefill": bench_prefill, "norm": bench_norm,
         "moe": bench_moe, "pd_qkv": bench_pd_qkv, "prefill_timeline": prefill_timeline,
         "tp": bench_tp_kernels}[name](t, res)
    for r in res:
        print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()}))


if __name__ == "__main__":
    main()
