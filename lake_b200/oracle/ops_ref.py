"""fp32 PyTorch reference implementations of every kernel in ``csrc/kernels``.

These are the correctness oracle for the CUDA kernels (tests compare against
them) and the CPU execution path of :mod:`lake_b200.ops`. Semantics follow the
reference model's intended forward (python/lake/engine/model_executor/models/
qwen/qwen3.py:85-259 describes the module tree; the reference never executes it)
and the pure-Python attention oracle (python/lake/kernels/attn_ref.py:13-56).
"""
from __future__ import annotations

import math

import torch

PAGE = 16
HEAD_DIM = 128


def linear(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return a.float() @ w.float().t()


def swiglu_from_interleaved(acc: torch.Tensor, tile: int = 256) -> torch.Tensor:
    """acc [M, 2I] with rows of each 256-wide tile laid out [gate 128 | up 128]."""
    m, n = acc.shape
    t = acc.view(m, n // tile, 2, tile // 2)
    g, u = t[:, :, 0, :], t[:, :, 1, :]
    return (torch.nn.functional.silu(g) * u).reshape(m, n // 2)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, tile: int = 256) -> torch.Tensor:
    """Stack gate [I, H] and up [I, H] into the tile-interleaved layout the SwiGLU epilogue reads."""
    i, h = gate.shape
    half = tile // 2
    assert i % half == 0
    g = gate.view(i // half, half, h)
    u = up.view(i // half, half, h)
    return torch.stack([g, u], dim=1).reshape(2 * i, h).contiguous()


def rope_cache(max_pos: int, theta: float, head_dim: int = HEAD_DIM, scaling: dict | None = None,
               device=None) -> torch.Tensor:
    """[max_pos, head_dim/2, 2] fp32 (cos, sin) for rotate-half RoPE.

    ``scaling`` supports the "llama3" frequency-band rule (factor, low/high
    frequency factors, original max positions).
    """
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) * 2.0 / head_dim))
    if scaling and scaling.get("rope_type", scaling.get("type")) == "llama3":
        factor = scaling["factor"]
        lo = scaling.get("low_freq_factor", 1.0)
        hi = scaling.get("high_freq_factor", 4.0)
        orig = scaling.get("original_max_position_embeddings", 8192)
        lo_wl, hi_wl = orig / lo, orig / hi
        wl = 2 * math.pi / inv
        smooth = (orig / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        scaled = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        inv = scaled
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos[:, None] * inv[None, :]
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).float()
    return cs.to(device) if device is not None else cs


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    """x [T, H, D] fp32, rotate-half convention."""
    half = x.shape[-1] // 2
    c = cs[positions.long(), :, 0][:, None, :]
    s = cs[positions.long(), :, 1][:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def write_kv(arena: torch.Tensor, layer: int, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """k, v [T, Hkv, D]; slots [T] (block*16+offset, <0 skipped)."""
    sl = slots.long()
    keep = sl >= 0
    sl = sl[keep]
    page = arena.shape[4]
    blk, off = sl // page, sl % page
    arena[blk, layer, 0, :, off, :] = k[keep].to(arena.dtype)
    arena[blk, layer, 1, :, off, :] = v[keep].to(arena.dtype)


def gather_kv(arena: torch.Tensor, layer: int, block_table: torch.Tensor, length: int):
    """Return K, V [length, Hkv, D] fp32 for one sequence."""
    page = arena.shape[4]
    nb = (length + page - 1) // page
    ids = block_table[:nb].long()
    k = arena[ids, layer, 0].float()  # [nb, Hkv, 16, D]
    v = arena[ids, layer, 1].float()
    k = k.permute(0, 2, 1, 3).reshape(nb * page, -1, k.shape[-1])[:length]
    v = v.permute(0, 2, 1, 3).reshape(nb * page, -1, v.shape[-1])[:length]
    return k, v


def attention_one(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, scale: float):
    """q [Tq, Hq, D], k/v [Tk, Hkv, D] (fp32), causal by absolute position: key j visible iff j <= q_pos."""
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * scale
    kp = torch.arange(k.shape[0], device=q.device)
    mask = kp[None, :] > q_pos.long()[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, v)


def paged_attention(q: torch.Tensor, arena: torch.Tensor, layer: int, block_tables: torch.Tensor,
                    seq_lens: torch.Tensor, query_start: torch.Tensor, positions: torch.Tensor,
                    n_q_heads: int, n_kv_heads: int, scale: float) -> torch.Tensor:
    """Generic paged attention: rows [query_start[s], query_start[s+1]) belong to sequence s."""
    d = arena.shape[-1]
    out = torch.zeros(q.shape[0], n_q_heads * d, dtype=torch.float32, device=q.device)
    qs = query_start.tolist()
    lens = seq_lens.tolist()
    for s in range(len(lens)):
        a, b = qs[s], qs[s + 1]
        if b <= a or lens[s] <= 0:
            continue
        k, v = gather_kv(arena, layer, block_tables[s], lens[s])
        qq = q[a:b].float().view(b - a, n_q_heads, d)
        o = attention_one(qq, k, v, positions[a:b], scale)
        out[a:b] = o.reshape(b - a, -1)
    return out


def greedy(logits: torch.Tensor, bitmask: torch.Tensor | None = None) -> torch.Tensor:
    lg = logits.float()
    if bitmask is not None:
        lg = apply_bitmask(lg, bitmask)
    return lg.argmax(dim=-1).to(torch.int32)


def bitmask_to_bool(bitmask: torch.Tensor, vocab: int) -> torch.Tensor:
    words = bitmask.to(torch.int64) & 0xFFFFFFFF
    bits = (words[:, :, None] >> torch.arange(32, device=bitmask.device)[None, None, :]) & 1
    return bits.reshape(bitmask.shape[0], -1)[:, :vocab].bool()


def apply_bitmask(logits: torch.Tensor, bitmask: torch.Tensor) -> torch.Tensor:
    allow = bitmask_to_bool(bitmask, logits.shape[-1])
    return logits.masked_fill(~allow, float("-inf"))


def chain_reject(draft: list[list[int]], target: list[list[int]]) -> list[list[int]]:
    """Greedy chain verification: accept matching drafts, then the target token at the first mismatch,
    or the bonus token after a fully accepted chain (target has len(draft)+1 entries per request)."""
    out = []
    for d, t in zip(draft, target):
        acc = []
        for i, tok in enumerate(d):
            acc.append(t[i])
            if t[i] != tok:
                break
        else:
            acc.append(t[len(d)])
        out.append(acc)
    return out
