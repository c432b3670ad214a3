"""Library baseline of the Llama decoder: the same engine, scheduler, paged KV arena and
prefill/decode plumbing as the native model, with every hot op taken from libraries instead of
this package's kernels. It is the same-box comparator of ``bench.py --impl torch``.

    projections   torch.nn.functional.linear (cuBLAS), unfused
    RMSNorm       torch.nn.functional.rms_norm
    RoPE, K/V     torch elementwise ops; K/V rows written into the paged arena by index_put
    prefill attn  torch SDPA per sequence over its gathered pages (lower-right causal bias)
    decode attn   torch SDPA over the batch's gathered pages with a length mask (the query heads
                  of one KV head folded into the query dimension)
    tensor par.   Megatron layout: column-parallel QKV / gate_up, row-parallel o_proj / down,
                  one NCCL all_reduce after each row-parallel GEMM; tokens replicated on ranks
    P -> D        after the step, cudaMemcpyPeerAsync of each written page (a page holds every
                  layer's K/V rows) into the decode instance's arena

Steps run eagerly (no CUDA graphs: the gathered page counts follow the batch) with overlapped
scheduling. The model reads the host copies of the step metadata the runner packs, so nothing
in the forward waits on the device.

Reference parity: the reference's model is a shell whose layers never execute
(python/lake/engine/model_executor/models/qwen/qwen3.py:100-240); this is the plain
library formulation of the same Llama block, kept beside the native kernels for comparison.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..oracle import ops_ref as ref
from .config import ModelConfig
from .llama import ForwardBatch, Workspace


class LibraryLM:
    wants_host_meta = True  # the runner attaches host copies of lens / qstart to each batch

    def __init__(self, cfg: ModelConfig, device, dtype: torch.dtype | None = None, seed: int = 0,
                 tp: tuple | None = None, weights: dict[str, torch.Tensor] | None = None):
        """`tp` = (rank, world, NCCL process group) or None. `weights`: a native model's weight
        dict (unsharded; gate_up in its tile-interleaved layout) to run the same model."""
        if cfg.n_experts or cfg.qk_norm:
            raise ValueError("the library baseline covers dense Llama-family models")
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.float32 if self.device.type == "cpu" else torch.bfloat16)
        self.rank, self.world, self.group = tp if tp is not None else (0, 1, None)
        if cfg.n_kv_heads % self.world or cfg.intermediate % self.world:
            raise ValueError(f"heads / FFN do not split over {self.world} ranks")
        self.hq, self.hk = cfg.n_q_heads // self.world, cfg.n_kv_heads // self.world
        self.inter = cfg.intermediate // self.world
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.w: dict[str, torch.Tensor] = {}
        if weights is not None:
            self._from_native(weights)
        else:
            self._random_init(seed)
        cs = ref.rope_cache(cfg.max_position, cfg.rope_theta, cfg.head_dim, cfg.rope_scaling, device=self.device)
        self.cos, self.sin = cs[..., 0].contiguous(), cs[..., 1].contiguous()
        self.layer_ready = None
        self.moe = None

    # ------------------------------------------------------------ weights
    def _random_init(self, seed: int) -> None:
        c, dev, dt = self.cfg, self.device, self.dtype
        gen = torch.Generator(device=dev).manual_seed(seed * 131 + self.rank)
        d, h = c.head_dim, c.hidden

        def rnd(*shape, std=0.02):
            return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dt)

        ones = lambda n: torch.ones(n, device=dev, dtype=dt)  # noqa: E731
        self.w["embed_tokens"] = rnd(c.vocab, h, std=1.0)
        for i in range(c.n_layers):
            p = f"layers.{i}."
            self.w[p + "input_layernorm"] = ones(h)
            self.w[p + "post_attention_layernorm"] = ones(h)
            self.w[p + "qkv_proj"] = rnd((self.hq + 2 * self.hk) * d, h)
            self.w[p + "o_proj"] = rnd(h, self.hq * d)
            self.w[p + "gate_up_proj"] = rnd(2 * self.inter, h)  # [gate; up]
            self.w[p + "down_proj"] = rnd(h, self.inter)
        self.w["norm"] = ones(h)
        self.w["lm_head"] = self.w["embed_tokens"] if c.tie_embeddings else rnd(c.vocab, h)

    def _from_native(self, full: dict[str, torch.Tensor]) -> None:
        """This rank's shard of a native weight dict, in the standard layouts."""
        c, r, d = self.cfg, self.rank, self.cfg.head_dim
        to = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        self.w["embed_tokens"] = to(full["embed_tokens"])
        for i in range(c.n_layers):
            p = f"layers.{i}."
            self.w[p + "input_layernorm"] = to(full[p + "input_layernorm"])
            self.w[p + "post_attention_layernorm"] = to(full[p + "post_attention_layernorm"])
            qkv = full[p + "qkv_proj"]
            q0, k0 = c.n_q_heads * d, c.n_q_heads * d + c.n_kv_heads * d
            self.w[p + "qkv_proj"] = to(torch.cat([qkv[r * self.hq * d:(r + 1) * self.hq * d],
                                                   qkv[q0 + r * self.hk * d:q0 + (r + 1) * self.hk * d],
                                                   qkv[k0 + r * self.hk * d:k0 + (r + 1) * self.hk * d]]))
            self.w[p + "o_proj"] = to(full[p + "o_proj"][:, r * self.hq * d:(r + 1) * self.hq * d])
            gu = full[p + "gate_up_proj"]
            if c.intermediate % 128 == 0:  # native layout: [gate 128 | up 128] per 256 rows
                g = gu.view(-1, 2, 128, gu.shape[1])
                gate, up = g[:, 0].reshape(-1, gu.shape[1]), g[:, 1].reshape(-1, gu.shape[1])
            else:
                gate, up = gu[: c.intermediate], gu[c.intermediate:]
            sl = slice(r * self.inter, (r + 1) * self.inter)
            self.w[p + "gate_up_proj"] = to(torch.cat([gate[sl], up[sl]]))
            self.w[p + "down_proj"] = to(full[p + "down_proj"][:, sl])
        self.w["norm"] = to(full["norm"])
        self.w["lm_head"] = to(full["lm_head"])

    def named_weights(self):
        return self.w.items()

    def new_workspace(self, max_tokens: int, max_samples: int, max_seqs: int = 0, max_splits: int = 1) -> Workspace:
        z = lambda *s, dt=None: torch.zeros(*s, dtype=dt or self.dtype, device=self.device)  # noqa: E731
        e = z(0)
        return Workspace(h=e, x=e, q=e, attn=e, act=e, fx=e, keys=z(max_samples, dt=torch.int64),
                         tokens=z(max_samples, dt=torch.int32))

    # ------------------------------------------------------------ engine hooks
    @staticmethod
    def resolve_tokens(ids: torch.Tensor, prev: torch.Tensor) -> None:
        """ids[i] < 0 -> prev[-1 - ids[i]] (overlapped scheduling), without a host sync."""
        j = (-1 - ids.long()).clamp(0, max(prev.numel() - 1, 0))
        ids.copy_(torch.where(ids < 0, prev[j].to(ids.dtype), ids))

    def copy_pages(self, arena: torch.Tensor, peer: torch.Tensor, src: list[int], dst: list[int]) -> None:
        """Whole pages into the peer arena (cudaMemcpyPeerAsync per contiguous run)."""
        i = 0
        while i < len(src):
            j = i + 1
            while j < len(src) and src[j] == src[j - 1] + 1 and dst[j] == dst[j - 1] + 1:
                j += 1
            peer[dst[i]:dst[i] + (j - i)].copy_(arena[src[i]:src[i] + (j - i)], non_blocking=True)
            i = j

    # ------------------------------------------------------------ forward
    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        half = x.shape[-1] // 2
        c = self.cos[pos][:, None, :].to(x.dtype)
        s = self.sin[pos][:, None, :].to(x.dtype)
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)

    def _attention(self, i: int, q: torch.Tensor, b: ForwardBatch, arena: torch.Tensor, host: dict) -> torch.Tensor:
        c, bs = self.cfg, arena.shape[4]
        g = self.hq // self.hk
        out = torch.empty_like(q)
        nd, lens, qs = b.n_decode, host["lens"], host["qstart"]
        if nd:
            nblk = -(-max(lens[:nd]) // bs)
            bt = b.block_tables[:nd, :nblk].long()
            k = arena[bt, i, 0].permute(0, 2, 1, 3, 4).reshape(nd, self.hk, nblk * bs, c.head_dim)
            v = arena[bt, i, 1].permute(0, 2, 1, 3, 4).reshape(nd, self.hk, nblk * bs, c.head_dim)
            mask = torch.arange(nblk * bs, device=q.device)[None, :] < b.seq_lens[:nd, None]
            qd = q[:nd].view(nd, self.hk, g, c.head_dim)  # the group's query heads as query rows
            o = F.scaled_dot_product_attention(qd, k, v, attn_mask=mask[:, None, None, :], scale=self.scale)
            out[:nd] = o.reshape(nd, self.hq, c.head_dim)
        from torch.nn.attention.bias import causal_lower_right

        for s in range(nd, len(lens)):
            r0, r1 = qs[s], qs[s + 1]
            n, ctx = r1 - r0, lens[s]
            if n <= 0:
                continue
            nblk = -(-ctx // bs)
            bt = b.block_tables[s, :nblk].long()
            k = arena[bt, i, 0].permute(1, 0, 2, 3).reshape(self.hk, nblk * bs, c.head_dim)[:, :ctx]
            v = arena[bt, i, 1].permute(1, 0, 2, 3).reshape(self.hk, nblk * bs, c.head_dim)[:, :ctx]
            k = k.repeat_interleave(g, dim=0)[None]
            v = v.repeat_interleave(g, dim=0)[None]
            qp = q[r0:r1].transpose(0, 1)[None]  # [1, hq, n, d]
            o = F.scaled_dot_product_attention(qp, k, v, attn_mask=causal_lower_right(n, ctx), scale=self.scale)
            out[r0:r1] = o[0].transpose(0, 1)
        return out

    def _reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(x, group=self.group)
        return x

    def forward(self, b: ForwardBatch, arena: torch.Tensor, ws: Workspace):
        c, w = self.cfg, self.w
        host = getattr(b, "host", None)
        if host is None:  # direct callers: take the metadata from the device tensors
            host = {"rows": int((b.slots >= 0).sum()), "lens": b.seq_lens.tolist(),
                    "qstart": b.query_start.tolist()}
        t = host["rows"]  # real rows; padding rows (tensor-parallel multiples) follow them
        r = b.sample_rows.shape[0]
        if t == 0:
            return ws.tokens[:0]
        d, bs = c.head_dim, arena.shape[4]
        pos = b.positions[:t].long()
        slots = b.slots[:t]
        blk, off = slots // bs, slots % bs
        h = F.embedding(b.input_ids[:t].long(), w["embed_tokens"])
        for i in range(c.n_layers):
            p = f"layers.{i}."
            x = F.rms_norm(h, (c.hidden,), w[p + "input_layernorm"], c.rms_eps)
            qkv = F.linear(x, w[p + "qkv_proj"])
            q = qkv[:, : self.hq * d].view(t, self.hq, d)
            k = qkv[:, self.hq * d:(self.hq + self.hk) * d].view(t, self.hk, d)
            v = qkv[:, (self.hq + self.hk) * d:].view(t, self.hk, d)
            q, k = self._rope(q, pos), self._rope(k, pos)
            arena[blk, i, 0, :, off] = k.to(arena.dtype)
            arena[blk, i, 1, :, off] = v.to(arena.dtype)
            attn = self._attention(i, q.contiguous(), b, arena, host)
            h = h + self._reduce(F.linear(attn.view(t, self.hq * d), w[p + "o_proj"]))
            x = F.rms_norm(h, (c.hidden,), w[p + "post_attention_layernorm"], c.rms_eps)
            gu = F.linear(x, w[p + "gate_up_proj"])
            act = F.silu(gu[:, : self.inter]) * gu[:, self.inter:]
            h = h + self._reduce(F.linear(act, w[p + "down_proj"]))
        if b.peer_arena is not None and b.peer_slots is not None and b.peer_arena is not arena:
            self._send_written_pages(slots, b.peer_slots[:t], arena, b.peer_arena)
        if r == 0:
            return ws.tokens[:0]
        fx = F.rms_norm(h.index_select(0, b.sample_rows), (c.hidden,), w["norm"], c.rms_eps)
        logits = F.linear(fx, w["lm_head"]).float()
        if b.want_logits:
            return logits
        if b.bitmask is not None:
            logits = ref.apply_bitmask(logits, b.bitmask)
        toks = ws.tokens[:r]
        toks.copy_(logits.argmax(-1).to(torch.int32))
        return toks

    def _send_written_pages(self, slots: torch.Tensor, peer_slots: torch.Tensor, arena: torch.Tensor,
                            peer: torch.Tensor) -> None:
        """Pages this step wrote for a remote (decode) instance -> the peer arena, page by page."""
        bs = arena.shape[4]
        sel = peer_slots >= 0
        pairs = torch.unique(torch.stack([slots[sel] // bs, peer_slots[sel] // bs], 1), dim=0).tolist()
        if pairs:
            self.copy_pages(arena, peer, [a for a, _ in pairs], [b for _, b in pairs])
