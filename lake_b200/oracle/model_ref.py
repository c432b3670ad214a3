"""Dense fp32 reference forward of a DecoderLM (no paging, no caching, full
recomputation). Used as the correctness oracle for the engine: greedy tokens
and logits of the paged/chunked/prefix-cached engine must match it."""
from __future__ import annotations

import torch

from . import ops_ref as ref


def dense_logits(model, tokens: list[int]) -> torch.Tensor:
    """Logits [len(tokens), V] (fp32) of the full sequence."""
    c = model.cfg
    w = {k: v.float().cpu() for k, v in model.w.items()}
    t = len(tokens)
    ids = torch.tensor(tokens, dtype=torch.long)
    pos = torch.arange(t, dtype=torch.int32)
    cs = ref.rope_cache(c.max_position, c.rope_theta, c.head_dim, c.rope_scaling)
    h = w["embed_tokens"][ids]
    d = c.head_dim
    for i in range(c.n_layers):
        p = f"layers.{i}."
        x = ref.rms_norm(h, w[p + "input_layernorm"], c.rms_eps)
        qkv = x @ w[p + "qkv_proj"].t()
        q = qkv[:, : c.q_size].view(t, c.n_q_heads, d)
        k = qkv[:, c.q_size:c.q_size + c.kv_size].view(t, c.n_kv_heads, d)
        v = qkv[:, c.q_size + c.kv_size:].view(t, c.n_kv_heads, d)
        if c.qk_norm:
            q = ref.rms_norm(q, w[p + "q_norm"], c.rms_eps)
            k = ref.rms_norm(k, w[p + "k_norm"], c.rms_eps)
        q = ref.apply_rope(q, pos, cs)
        k = ref.apply_rope(k, pos, cs)
        o = ref.attention_one(q, k, v, pos, 1.0 / d ** 0.5).reshape(t, -1)
        h = h + o @ w[p + "o_proj"].t()
        x = ref.rms_norm(h, w[p + "post_attention_layernorm"], c.rms_eps)
        if c.n_experts:
            logits = x @ w[p + "router"].t()
            topv, topi = logits.topk(c.top_k, dim=-1)
            wts = torch.softmax(topv, dim=-1)
            out = torch.zeros_like(h)
            gu_all = w[p + "experts.gate_up_proj"]
            dn_all = w[p + "experts.down_proj"]
            for e in range(c.n_experts):
                m = topi == e
                rows = m.any(-1).nonzero().flatten()
                if rows.numel() == 0:
                    continue
                gu = x[rows] @ gu_all[e].t()
                act = ref.swiglu_from_interleaved(gu) if c.intermediate % 128 == 0 else \
                    torch.nn.functional.silu(gu[:, : c.intermediate]) * gu[:, c.intermediate:]
                y = act @ dn_all[e].t()
                wt = (wts * m.float()).sum(-1)[rows]
                out[rows] += y * wt[:, None]
            h = h + out
        else:
            gu = x @ w[p + "gate_up_proj"].t()
            act = ref.swiglu_from_interleaved(gu) if c.intermediate % 128 == 0 else \
                torch.nn.functional.silu(gu[:, : c.intermediate]) * gu[:, c.intermediate:]
            h = h + act @ w[p + "down_proj"].t()
    x = ref.rms_norm(h, w["norm"], c.rms_eps)
    return x @ w["lm_head"].t()


def greedy_generate(model, prompt: list[int], max_new_tokens: int) -> list[int]:
    toks = list(prompt)
    out = []
    for _ in range(max_new_tokens):
        nxt = int(dense_logits(model, toks)[-1].argmax())
        out.append(nxt)
        toks.append(nxt)
    return out
