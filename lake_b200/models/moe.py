"""Top-k routed mixture-of-experts MLP (Mixtral).

Router logits come from a GEMM on the normalised hidden state; the top-k
experts per token are weighted by a softmax over their logits. Each expert's
tokens are gathered and run through the SwiGLU expert (gate_up GEMM with the
fused SwiGLU epilogue, then down projection), and the weighted outputs are
added back into the residual stream.
"""
from __future__ import annotations

import torch

from .. import ops
from ..oracle import ops_ref as ref


class MoE:
    def __init__(self, model):
        self.m = model
        c = model.cfg
        # interleave each expert's [gate; up] rows into the SwiGLU tile layout once
        for i in range(c.n_layers):
            key = f"layers.{i}.experts.gate_up_proj"
            w = model.w[key]
            if c.intermediate % 128 == 0:
                model.w[key] = torch.stack([ref.interleave_gate_up(w[e, : c.intermediate], w[e, c.intermediate:])
                                            for e in range(c.n_experts)])

    def route(self, i: int, x: torch.Tensor):
        c = self.m.cfg
        logits = ops.linear(x, self.m.w[f"layers.{i}.router"], out_dtype=torch.float32)
        topv, topi = logits.topk(c.top_k, dim=-1)
        return torch.softmax(topv, dim=-1), topi

    def forward(self, i: int, x: torch.Tensor, h: torch.Tensor, ws, t: int) -> None:
        c = self.m.cfg
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
