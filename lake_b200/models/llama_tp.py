"""Tensor-parallel decoder (Llama family) with the collectives fused into the
kernels around them over NVLink peer memory.

Rank r of a group of T holds q heads [r*Hq/T, (r+1)*Hq/T), kv heads
[r*Hkv/T, ...), the matching o_proj columns, an intermediate slice of
gate_up / down, and a vocab slice of lm_head. The residual stream is split by
rows (sequence parallel): rank r owns rows [r*Mr, (r+1)*Mr) with
Mr = ceil(tokens/T). Per layer:

    qkv  : column-parallel GEMM over all rows; waits per row shard for the
           all-gather pushes, RoPE + paged-KV write for the local kv heads
    attn : paged attention over the local heads (unchanged kernels)
    o    : row-parallel GEMM, epilogue pushes partial rows to their owners
    norm : owner sums the partials + residual, RMSNorm, pushes the normalised
           row to every rank's next GEMM input
    gate_up (SwiGLU) / down / norm : same pattern

and lm_head is vocab-parallel: each rank's argmax epilogue leaves (score,
index) keys, one kernel takes the max over ranks. All ranks compute the same
tokens, so each runs an identical scheduler.

Reference parity: the reference's parallelism layer is a stub
(python/lake/engine/distributed/parallel_state.py:1-60, communication_op.py:1-40);
this is the working B200 form of TP=2/4/8.
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import tp as tpops
from ..parallel.tp import SLOT_E, SLOT_FX, TPGroup
from .config import ModelConfig
from .llama import DecoderLM, ForwardBatch, Workspace


def shard_weights(full: dict[str, torch.Tensor], cfg: ModelConfig, rank: int, world: int) -> dict[str, torch.Tensor]:
    """Slice a full (unsharded) weight dict into rank's tensor-parallel shard."""
    d = cfg.head_dim
    hq, hk = cfg.n_q_heads // world, cfg.n_kv_heads // world
    inter = cfg.intermediate // world
    vocab = cfg.vocab // world
    out = {}
    for name, t in full.items():
        if name.endswith("qkv_proj"):
            q = t[: cfg.n_q_heads * d].view(cfg.n_q_heads, d, -1)[rank * hq:(rank + 1) * hq]
            k = t[cfg.n_q_heads * d:(cfg.n_q_heads + cfg.n_kv_heads) * d].view(cfg.n_kv_heads, d, -1)
            v = t[(cfg.n_q_heads + cfg.n_kv_heads) * d:].view(cfg.n_kv_heads, d, -1)
            k = k[rank * hk:(rank + 1) * hk]
            v = v[rank * hk:(rank + 1) * hk]
            out[name] = torch.cat([q.reshape(-1, t.shape[1]), k.reshape(-1, t.shape[1]),
                                   v.reshape(-1, t.shape[1])]).contiguous()
        elif name.endswith("o_proj"):
            out[name] = t[:, rank * hq * d:(rank + 1) * hq * d].contiguous()
        elif name.endswith("gate_up_proj"):
            # tile-interleaved [gate 128 | up 128] blocks: a contiguous run of blocks per rank
            out[name] = t[rank * 2 * inter:(rank + 1) * 2 * inter].contiguous()
        elif name.endswith("down_proj"):
            out[name] = t[:, rank * inter:(rank + 1) * inter].contiguous()
        elif name == "lm_head":
            out[name] = t[rank * vocab:(rank + 1) * vocab].contiguous()
        else:
            out[name] = t
    return out


class TPDecoderLM:
    def __init__(self, cfg: ModelConfig, group: TPGroup, device, seed: int = 0,
                 full_weights: dict[str, torch.Tensor] | None = None, weight_dtype: str = "bf16"):
        T = group.world
        for n, what in ((cfg.n_q_heads, "q heads"), (cfg.n_kv_heads, "kv heads"), (cfg.vocab, "vocab")):
            if n % T:
                raise ValueError(f"{what} ({n}) not divisible by tp={T}")
        if (cfg.intermediate // T) % 128 or cfg.intermediate % T:
            raise ValueError("intermediate/tp must be a multiple of 128")
        if cfg.n_experts or cfg.qk_norm:
            raise ValueError("tensor-parallel path covers dense Llama-family layers")
        self.cfg = cfg
        self.g = group
        self.rank, self.world = group.rank, T
        self.device = torch.device(device)
        self.dtype = torch.bfloat16
        self.hq, self.hk = cfg.n_q_heads // T, cfg.n_kv_heads // T
        self.vocab_local = cfg.vocab // T
        # local "view" of the config for the runner (kv heads of this rank's arena)
        if full_weights is None:
            # generate layer by layer and keep this rank's slice of each weight (a 70B model's
            # full bf16 weights would not fit next to the shards)
            def keep(n, t):
                s = shard_weights({n: t}, cfg, group.rank, T)[n]
                return s.clone() if s.numel() < t.numel() else s  # a slice view would pin the whole tensor

            full = DecoderLM(cfg, self.device, self.dtype, seed=seed, shard=keep)
            self.w = full.w
            self.rope_cs = full.rope_cs
            self.scale = full.scale
            del full
        else:
            from ..oracle import ops_ref as ref
            import math

            self.rope_cs = ref.rope_cache(cfg.max_position, cfg.rope_theta, cfg.head_dim, cfg.rope_scaling,
                                          device=self.device)
            self.scale = 1.0 / math.sqrt(cfg.head_dim)
        if full_weights is not None:
            self.w = {k: v.to(self.device) for k, v in shard_weights(full_weights, cfg, self.rank, T).items()}
            del full_weights
        if weight_dtype == "fp8":  # block-scaled e4m3 projections (W8A16 GEMMs); norms/embeddings stay bf16
            from ..ops.fp8 import quantize_blockwise, quantize_gate_up

            for k in list(self.w):
                if k.endswith("gate_up_proj"):
                    self.w[k] = quantize_gate_up(self.w[k])
                elif k.endswith(("qkv_proj", "o_proj", "down_proj")) or k == "lm_head":
                    self.w[k] = quantize_blockwise(self.w[k])
        torch.cuda.empty_cache()
        self.tp_world = T
        self.fp8 = weight_dtype == "fp8"

    # ------------------------------------------------------------------ workspace
    def new_workspace(self, max_tokens: int, max_samples: int, max_seqs: int = 0, max_splits: int = 1) -> Workspace:
        c, dev, dt = self.cfg, self.device, self.dtype
        mr = self.g.mr_max
        rows = mr * self.world
        ws = Workspace(
            h=torch.zeros(mr, c.hidden, dtype=dt, device=dev),  # owned residual rows
            x=torch.zeros(0, c.hidden, dtype=dt, device=dev),
            q=torch.zeros(rows, self.hq * c.head_dim, dtype=dt, device=dev),
            attn=torch.zeros(rows, self.hq * c.head_dim, dtype=dt, device=dev),
            act=torch.zeros(rows, c.intermediate // self.world, dtype=dt, device=dev),
            fx=torch.zeros(0, c.hidden, dtype=dt, device=dev),
            keys=torch.zeros(max_samples, dtype=torch.int64, device=dev),
            tokens=torch.zeros(max_samples, dtype=torch.int32, device=dev),
        )
        ws.extra["row_map"] = torch.full((rows,), -1, dtype=torch.int32, device=dev)
        ws.extra["ids"] = torch.zeros(mr, dtype=torch.int32, device=dev)
        if max_splits > 1 and max_seqs:
            ws.ws_o = torch.zeros(max_seqs * self.hk * max_splits * c.group * c.head_dim, dtype=torch.float32,
                                  device=dev)
            ws.ws_ml = torch.zeros(max_seqs * self.hk * max_splits * c.group * 2, dtype=torch.float32, device=dev)
        return ws

    # ------------------------------------------------------------------ forward
    def forward(self, b: ForwardBatch, arena: torch.Tensor, ws: Workspace):
        c, g, w = self.cfg, self.g, self.w
        t = b.num_tokens  # padded to a multiple of world by the runner
        mr = t // self.world
        assert mr * self.world == t and mr <= g.mr_max
        r0 = self.rank * mr
        h = ws.h[:mr]
        ops.embedding(b.input_ids[r0:r0 + mr], w["embed_tokens"], out=h)
        tpops.norm_push(h, w["layers.0.input_layernorm"], c.rms_eps, g.norm_push(mr, None, SLOT_E))
        ag_slot, rs_slot, k = SLOT_E, 0, 0
        nr = b.sample_rows.shape[0]
        for i in range(c.n_layers):
            p = f"layers.{i}."
            tpops.linear_qkv_ag(g.a_full[ag_slot][:t], w[p + "qkv_proj"], ws.q[:t], self.rope_cs, b.positions,
                                b.slots, arena, i, self.hq, self.hk, g.gemm_ag(ag_slot, mr), b.peer_arena,
                                b.peer_slots)
            attn = self._attention(i, b, arena, ws, t)
            tpops.linear_rs(attn, w[p + "o_proj"], g.gemm_rs(rs_slot, mr, c.hidden, self.hq * c.head_dim, self.fp8))
            k += 1
            ag_slot = k % 2
            tpops.norm_push(h, w[p + "post_attention_layernorm"], c.rms_eps, g.norm_push(mr, rs_slot, ag_slot))
            act = ws.act[:t]
            tpops.linear_swiglu_ag(g.a_full[ag_slot][:t], w[p + "gate_up_proj"], act, g.gemm_ag(ag_slot, mr))
            rs_slot ^= 1
            tpops.linear_rs(act, w[p + "down_proj"],
                            g.gemm_rs(rs_slot, mr, c.hidden, c.intermediate // self.world, self.fp8))
            k += 1
            if i + 1 < c.n_layers:
                ag_slot = k % 2
                tpops.norm_push(h, w[f"layers.{i + 1}.input_layernorm"], c.rms_eps,
                                g.norm_push(mr, rs_slot, ag_slot))
            else:
                rm = ws.extra["row_map"][:t]
                rm.fill_(-1)
                if nr:
                    rm.index_copy_(0, b.sample_rows, torch.arange(nr, dtype=torch.int32, device=self.device))
                tpops.norm_push(h, w["norm"], c.rms_eps, g.norm_push(mr, rs_slot, SLOT_FX, row_map=rm,
                                                                    store_h=False))
            rs_slot ^= 1
        if nr == 0:
            g.end_step()
            return ws.tokens[:0]
        tpops.linear_argmax_tp(g.fx[:nr], w["lm_head"], g.amax[:nr],
                               g.lm_argmax(mr, nr, self.vocab_local, self.fp8))
        toks = g.argmax_combine(ws.tokens, nr)
        g.end_step()
        return toks

    def _attention(self, i, b, arena, ws, t):
        c = self.cfg
        q, out = ws.q[:t], ws.attn[:t]
        nd = b.n_decode
        if nd:
            ops.paged_decode_attention(q[:nd], arena, i, b.block_tables[:nd], b.seq_lens[:nd], self.hq, self.hk,
                                       self.scale, out=out[:nd], splits=b.decode_splits, ws_o=ws.ws_o,
                                       ws_ml=ws.ws_ml)
        if b.prefill_tiles.shape[0]:
            ops.paged_prefill_attention(q, arena, i, b.block_tables, b.seq_lens, b.prefill_tiles, b.query_start,
                                        b.positions, self.hq, self.hk, self.scale, out=out)
        return out
