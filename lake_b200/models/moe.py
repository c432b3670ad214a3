"""Top-k routed mixture-of-experts MLP (Mixtral).

GPU path (no host synchronisation, CUDA-graph safe), four launches per layer:

    router   GEMM -> fp32 logits (router rows padded to 32)
    dispatch top-k + softmax weights, token rows gathered into per-expert
             segments (atomic slot per expert; segment capacity = tokens)
    experts  grouped tcgen05 GEMM gate_up + SwiGLU over all experts, then the
             grouped down GEMM whose scatter epilogue writes each row back to
             its (token, k) slot
    combine  h += sum_k w_k * expert_k(x)

The CPU path is the fp32 oracle (per-expert loop).
"""
from __future__ import annotations

import torch

from .. import ops
from ..oracle import ops_ref as ref


class MoE:
    def __init__(self, model, ep=None):
        self.m = model
        self.ep = ep  # lake_b200.parallel.ep.EPGroup: this rank holds experts [rank*epr, (rank+1)*epr)
        c = model.cfg
        # interleave each expert's [gate; up] rows into the SwiGLU tile layout once
        for i in range(c.n_layers):
            key = f"layers.{i}.experts.gate_up_proj"
            w = model.w[key]
            if c.intermediate % 128 == 0:
                model.w[key] = torch.stack([ref.interleave_gate_up(w[e, : c.intermediate], w[e, c.intermediate:])
                                            for e in range(c.n_experts)])

        if ep is not None:
            lo, hi = ep.rank * ep.epr, (ep.rank + 1) * ep.epr
            for i in range(c.n_layers):
                for name in ("experts.gate_up_proj", "experts.down_proj"):
                    key = f"layers.{i}.{name}"
                    model.w[key] = model.w[key][lo:hi].contiguous()
            torch.cuda.empty_cache()
        self.router_pad = {}
        if model.device.type == "cuda":
            for i in range(c.n_layers):
                r = model.w[f"layers.{i}.router"]
                pad = torch.zeros(32 * ((c.n_experts + 31) // 32), r.shape[1], dtype=r.dtype, device=r.device)
                pad[: c.n_experts] = r
                self.router_pad[i] = pad

    def workspace(self, ws, max_tokens: int) -> None:
        c, dev, dt = self.m.cfg, self.m.device, self.m.dtype
        cap = (max_tokens + 127) // 128 * 128
        rows = c.n_experts * cap
        if self.ep is not None:
            ws.extra.update(
                moe_logits=torch.zeros(max_tokens, self.router_pad[0].shape[0], dtype=torch.float32, device=dev),
                moe_w=torch.zeros(max_tokens * c.top_k, dtype=torch.float32, device=dev),
                moe_act=torch.zeros(self.ep.epr * self.ep.cap, c.intermediate, dtype=dt, device=dev),
                moe_count=self.ep.count[0])
            return
        ws.extra.update(
            moe_logits=torch.zeros(max_tokens, self.router_pad[0].shape[0], dtype=torch.float32, device=dev),
            moe_count=torch.zeros(c.n_experts, dtype=torch.int32, device=dev),
            moe_gathered=torch.zeros(rows, c.hidden, dtype=dt, device=dev),
            moe_slot=torch.full((rows,), -1, dtype=torch.int32, device=dev),
            moe_w=torch.zeros(max_tokens * c.top_k, dtype=torch.float32, device=dev),
            moe_act=torch.zeros(rows, c.intermediate, dtype=dt, device=dev),
            moe_comb=torch.zeros(max_tokens * c.top_k, c.hidden, dtype=dt, device=dev))

    def forward_gpu(self, i: int, x: torch.Tensor, h: torch.Tensor, ws, t: int) -> None:
        from ..ops._ext import native
        from ..ops.core import LAUNCHES, status_word

        c = self.m.cfg
        E, k = c.n_experts, c.top_k
        cap = (t + 127) // 128 * 128
        ex = ws.extra
        st = status_word(x.device)
        logits = ops.linear(x, self.router_pad[i], out=ex["moe_logits"][:t])
        if self.ep is not None:  # all-to-all dispatch / combine over NVLink, local experts only
            self.ep.layer(i % 2, x, logits, ex["moe_w"][: t * k], h, self.m.w[f"layers.{i}.experts.gate_up_proj"],
                          self.m.w[f"layers.{i}.experts.down_proj"], ex["moe_act"], st)
            LAUNCHES[0] += 5
            return
        count = ex["moe_count"]
        count.zero_()
        gathered = ex["moe_gathered"][: E * cap]
        slot = ex["moe_slot"][: E * cap]
        wts = ex["moe_w"][: t * k]
        C = native()
        C.moe_dispatch(logits, x, wts, E, k, cap, 1, 0, [gathered.data_ptr()], [slot.data_ptr()], [],
                       [count.data_ptr()], [], st)
        act = ex["moe_act"][: E * cap]
        C.gemm_grouped(gathered, self.m.w[f"layers.{i}.experts.gate_up_proj"], act, 2, count, cap, status=st)
        comb = ex["moe_comb"][: t * k]
        C.gemm_grouped(act, self.m.w[f"layers.{i}.experts.down_proj"], None, 7, count, cap, row_slot=slot,
                       dst_ptrs=[comb.data_ptr()], status=st)
        C.moe_combine(h, comb, wts, k, status=st)
        LAUNCHES[0] += 4  # dispatch, 2 grouped GEMMs, combine (the router GEMM counts itself)

    def route(self, i: int, x: torch.Tensor):
        c = self.m.cfg
        logits = ops.linear(x, self.m.w[f"layers.{i}.router"], out_dtype=torch.float32)
        topv, topi = logits.topk(c.top_k, dim=-1)
        return torch.softmax(topv, dim=-1), topi

    def forward(self, i: int, x: torch.Tensor, h: torch.Tensor, ws, t: int) -> None:
        c = self.m.cfg
        if x.is_cuda and c.intermediate % 128 == 0:
            if "moe_count" not in ws.extra:
                raise RuntimeError("MoE workspace missing: DecoderLM.new_workspace allocates it")
            self.forward_gpu(i, x, h, ws, t)
            return
        gate_up = self.m.w[f"layers.{i}.experts.gate_up_proj"]
        down = self.m.w[f"layers.{i}.experts.down_proj"]
        wts, idx = self.route(i, x)
        acc = torch.zeros(t, c.hidden, dtype=torch.float32, device=x.device)
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=c.n_experts).tolist()
        tok = order // c.top_k
        start = 0
        for e, n in enumerate(counts):
            if n == 0:
                continue
            sel = order[start:start + n]
            rows = tok[start:start + n]
            start += n
            xe = x.index_select(0, rows)
            if c.intermediate % 128 == 0:
                act = ops.linear_swiglu(xe, gate_up[e])
            else:
                gu = ref.linear(xe, gate_up[e])
                act = (torch.nn.functional.silu(gu[:, : c.intermediate]) * gu[:, c.intermediate:]).to(x.dtype)
            ye = ops.linear(act, down[e], out_dtype=torch.float32)
            acc.index_add_(0, rows, ye * wts.reshape(-1)[sel, None])
        h.add_(acc.to(h.dtype))
