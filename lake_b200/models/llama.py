"""Decoder-only transformer (Llama-3 / Mixtral / Qwen3 families) built on the
lake_b200 kernels.

Per layer on the GPU path (every step is one sm_100a kernel launch):

    x    = rmsnorm(h)                                   rmsnorm
    q    = QKV(x) -> RoPE(q); RoPE(k), v -> paged arena linear_qkv (fused epilogue)
    o    = paged attention (decode rows | prefill tiles) paged_decode / paged_prefill
    h    = h + O(o)                                      linear_residual (in place)
    x    = rmsnorm(h)                                   rmsnorm
    a    = silu(G(x)) * U(x)                             linear_swiglu (fused epilogue)
    h    = h + D(a)                                      linear_residual (in place)

and at the end ``argmax(lm_head(rmsnorm(h[sample_rows])))`` in one GEMM with an
argmax epilogue (bitmask applied in the epilogue when grammar-constrained).
Mixtral layers replace the MLP with top-k routed experts (lake_b200.models.moe).
Qwen3 adds per-head q/k RMSNorm before RoPE.

Weight names follow the vLLM packed layout the reference uses
(python/lake/engine/model_executor/models/qwen/qwen3.py:85-259):
``qkv_proj``, ``o_proj``, ``gate_up_proj``, ``down_proj``, ``embed_tokens``,
``lm_head``; the reference's modules are identity shells, this one runs.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field

import torch

from .. import ops
from ..oracle import ops_ref as ref
from ..utils.trace import nvtx
from .config import ModelConfig

# Mixed steps run the decode rows' attention on a side stream beside the prefill rows' attention
# (LAKEB_ATTN_OVERLAP=1).
ATTN_OVERLAP = [os.environ.get("LAKEB_ATTN_OVERLAP", "0") == "1"]


@dataclass
class ForwardBatch:
    """Device tensors describing one engine step.

    Rows are ordered [decode rows (one per decode sequence)] + [prefill rows].
    Sequences are ordered the same way: sequence s < n_decode is decode row s.
    """

    input_ids: torch.Tensor  # [T] int32
    positions: torch.Tensor  # [T] int32
    slots: torch.Tensor  # [T] int64 KV write slot per row
    block_tables: torch.Tensor  # [S, max_blocks] int32
    seq_lens: torch.Tensor  # [S] int32 context length after this step
    n_decode: int
    prefill_tiles: torch.Tensor  # [n_tiles, 4] int32 (seq, row, n, pos)
    query_start: torch.Tensor  # [S+1] int32 (oracle path)
    sample_rows: torch.Tensor  # [R] int64 rows whose next token is sampled
    bitmask: torch.Tensor | None = None  # [R, ceil(V/32)] int32
    peer_arena: torch.Tensor | None = None  # decode instance's arena (P2P) for fused P->D
    peer_slots: torch.Tensor | None = None  # [T] int64 slots in the peer arena
    decode_splits: int = 1
    want_logits: bool = False
    # host copies of the step metadata, for models that need sequence boundaries on the host
    # (set by the runner when the model asks for them: {"rows", "lens", "qstart"})
    host: dict | None = None

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])


@dataclass
class Workspace:
    """Preallocated activation buffers sized for the largest step (reused, graph-safe)."""

    h: torch.Tensor
    x: torch.Tensor
    q: torch.Tensor
    attn: torch.Tensor
    act: torch.Tensor
    fx: torch.Tensor
    keys: torch.Tensor
    tokens: torch.Tensor
    ws_o: torch.Tensor | None = None
    ws_ml: torch.Tensor | None = None
    extra: dict = field(default_factory=dict)


class DecoderLM:
    def __init__(self, cfg: ModelConfig, device: torch.device | str = "cpu", dtype: torch.dtype | None = None,
                 seed: int = 0, init: str = "random", ep=None, weights: str | None = None, shard=None):
        """`shard(name, tensor) -> tensor`: applied to each weight as soon as it is generated, so
        a tensor-parallel rank keeps only its slice and never holds the whole model (the values
        are those of the unsharded model with the same seed)."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.float32 if self.device.type == "cpu" else torch.bfloat16)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.w: dict[str, torch.Tensor] = {}
        self._shard = shard
        if init in ("random", "zeros"):  # zeros: allocate only (a checkpoint overwrites every tensor)
            self._random_init(seed, zeros=init == "zeros")
        if weights:
            from .checkpoint import load_checkpoint

            load_checkpoint(self, weights)  # before the MoE set-up re-lays out the expert weights
        self.rope_cs = ref.rope_cache(cfg.max_position, cfg.rope_theta, cfg.head_dim, cfg.rope_scaling,
                                      device=self.device)
        self.layer_ready = None  # per-layer CUDA events while weights stream in (runtime.coldstart)
        self.moe = None
        if cfg.n_experts:
            from .moe import MoE

            self.moe = MoE(self, ep)

    # ------------------------------------------------------------ weights
    def _param(self, name, shape, gen, std=0.02, ones=False):
        if ones:
            t = torch.ones(shape, dtype=self.dtype, device=self.device)
        elif getattr(self, "_zeros", False):
            t = torch.zeros(shape, dtype=self.dtype, device=self.device)
        else:
            t = torch.empty(shape, dtype=torch.float32, device=self.device)
            t.normal_(0.0, std, generator=gen)
            t = t.to(self.dtype)
        if self._shard is not None:
            t = self._shard(name, t)
        self.w[name] = t
        return t

    def _random_init(self, seed: int, zeros: bool = False) -> None:
        self._zeros = zeros
        c = self.cfg
        gen = torch.Generator(device=self.device).manual_seed(seed)
        h, d = c.hidden, c.head_dim
        self._param("embed_tokens", (c.vocab, h), gen, std=1.0)
        for i in range(c.n_layers):
            p = f"layers.{i}."
            self._param(p + "input_layernorm", (h,), gen, ones=True)
            self._param(p + "post_attention_layernorm", (h,), gen, ones=True)
            self._param(p + "qkv_proj", ((c.n_q_heads + 2 * c.n_kv_heads) * d, h), gen)
            self._param(p + "o_proj", (h, c.n_q_heads * d), gen)
            if c.qk_norm:
                self._param(p + "q_norm", (d,), gen, ones=True)
                self._param(p + "k_norm", (d,), gen, ones=True)
            if c.n_experts:
                self._param(p + "router", (c.n_experts, h), gen)
                self._param(p + "experts.gate_up_proj", (c.n_experts, 2 * c.intermediate, h), gen)
                self._param(p + "experts.down_proj", (c.n_experts, h, c.intermediate), gen)
            else:
                # gate_up stored tile-interleaved ([gate 128 | up 128] per 256 rows) for the SwiGLU epilogue
                self._param(p + "gate_up_proj", (2 * c.intermediate, h), gen)
                self._param(p + "down_proj", (h, c.intermediate), gen)
        self._param("norm", (h,), gen, ones=True)
        if c.tie_embeddings:
            self.w["lm_head"] = self.w["embed_tokens"]
        else:
            self._param("lm_head", (c.vocab, h), gen)

    def load_weights(self, named: dict[str, torch.Tensor], strict: bool = False) -> list[str]:
        """Load HF-named or packed weights. ``gate_proj``/``up_proj`` pairs are interleaved,
        ``q/k/v_proj`` packed. Returns names that were set."""
        c = self.cfg
        done = []
        staged: dict[str, dict[str, torch.Tensor]] = {}
        for name, t in named.items():
            n = name.replace("model.", "").replace(".self_attn.", ".").replace(".mlp.", ".")
            n = n.replace(".weight", "")
            if c.n_experts and self._load_expert(n, t):  # Mixtral block_sparse_moe naming
                done.append(n)
                continue
            for part in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj"):
                if n.endswith(part):
                    staged.setdefault(n[: -len(part)], {})[part] = t
                    break
            else:
                if n in self.w:
                    self.w[n].copy_(t.to(self.dtype))
                    done.append(n)
                elif strict:
                    raise KeyError(n)
        for prefix, parts in staged.items():
            if {"q_proj", "k_proj", "v_proj"} <= parts.keys():
                self.w[prefix + "qkv_proj"].copy_(
                    torch.cat([parts["q_proj"], parts["k_proj"], parts["v_proj"]]).to(self.dtype))
                done.append(prefix + "qkv_proj")
            if {"gate_proj", "up_proj"} <= parts.keys():
                w = ref.interleave_gate_up(parts["gate_proj"], parts["up_proj"]) if c.intermediate % 128 == 0 \
                    else torch.cat([parts["gate_proj"], parts["up_proj"]])
                self.w[prefix + "gate_up_proj"].copy_(w.to(self.dtype))
                done.append(prefix + "gate_up_proj")
        return done

    def _load_expert(self, n: str, t: torch.Tensor) -> bool:
        """layers.L.block_sparse_moe.gate -> router; experts.E.w1 / w3 / w2 -> rows of the packed
        [gate; up] and down tensors of expert E (the MoE set-up interleaves them afterwards)."""
        import re

        m = re.fullmatch(r"layers\.(\d+)\.block_sparse_moe\.gate", n)
        if m:
            self.w[f"layers.{m.group(1)}.router"].copy_(t.to(self.dtype))
            return True
        m = re.fullmatch(r"layers\.(\d+)\.block_sparse_moe\.experts\.(\d+)\.(w1|w2|w3)", n)
        if not m:
            return False
        i, e, which = m.group(1), int(m.group(2)), m.group(3)
        I = self.cfg.intermediate
        if which == "w2":
            self.w[f"layers.{i}.experts.down_proj"][e].copy_(t.to(self.dtype))
        else:
            rows = slice(0, I) if which == "w1" else slice(I, 2 * I)
            self.w[f"layers.{i}.experts.gate_up_proj"][e, rows].copy_(t.to(self.dtype))
        return True

    def quantize_fp8(self) -> None:
        """Replace the dense projection weights by block-scaled e4m3 (W8A16 GEMMs); norms,
        embeddings and MoE experts stay bf16."""
        from ..ops.fp8 import quantize_blockwise, quantize_gate_up

        for k in list(self.w):
            if k.endswith(("qkv_proj", "o_proj", "gate_up_proj", "down_proj")) and "experts" not in k:
                gu = k.endswith("gate_up_proj") and self.cfg.intermediate % 128 == 0
                self.w[k] = quantize_gate_up(self.w[k]) if gu else quantize_blockwise(self.w[k])
        if not self.cfg.tie_embeddings:
            self.w["lm_head"] = quantize_blockwise(self.w["lm_head"])
        torch.cuda.empty_cache()

    def named_weights(self):
        return dict(self.w)

    # ------------------------------------------------------------ forward
    def new_workspace(self, max_tokens: int, max_samples: int, max_seqs: int = 0, max_splits: int = 1) -> Workspace:
        c = self.cfg
        dev, dt = self.device, self.dtype
        ws = Workspace(
            h=torch.zeros(max_tokens, c.hidden, dtype=dt, device=dev),
            x=torch.zeros(max_tokens, c.hidden, dtype=dt, device=dev),
            q=torch.zeros(max_tokens, c.q_size, dtype=dt, device=dev),
            attn=torch.zeros(max_tokens, c.q_size, dtype=dt, device=dev),
            act=torch.zeros(max_tokens, c.intermediate, dtype=dt, device=dev),
            fx=torch.zeros(max_samples, c.hidden, dtype=dt, device=dev),
            keys=torch.zeros(max_samples, dtype=torch.int64, device=dev),
            tokens=torch.zeros(max_samples, dtype=torch.int32, device=dev),
        )
        if max_splits > 1 and max_seqs:
            ws.ws_o = torch.zeros(max_seqs * c.n_kv_heads * max_splits * c.group * c.head_dim, dtype=torch.float32,
                                  device=dev)
            ws.ws_ml = torch.zeros(max_seqs * c.n_kv_heads * max_splits * c.group * 2, dtype=torch.float32,
                                   device=dev)
        if c.qk_norm:
            ws.extra["qkv"] = torch.zeros(max_tokens, c.q_size + 2 * c.kv_size, dtype=dt, device=dev)
        if self.moe is not None and dev.type == "cuda":
            self.moe.workspace(ws, max_tokens)
        return ws

    def _attention(self, i: int, b: ForwardBatch, arena: torch.Tensor, ws: Workspace, t: int) -> torch.Tensor:
        c = self.cfg
        q, out = ws.q[:t], ws.attn[:t]
        nd = b.n_decode
        side = self._attn_side_stream() if (nd and t > nd) else None
        if side is not None:
            # mixed step: the decode rows' attention (K/V-bandwidth-bound) runs on a side stream
            # beside the prefill rows' attention (tensor-core-bound); both only read q and the
            # arena and write disjoint rows of `out`
            main = torch.cuda.current_stream(self.device)
            ev_in, ev_out = torch.cuda.Event(), torch.cuda.Event()
            ev_in.record(main)
            side.wait_event(ev_in)
            with torch.cuda.stream(side):
                ops.paged_decode_attention(q[:nd], arena, i, b.block_tables[:nd], b.seq_lens[:nd], c.n_q_heads,
                                           c.n_kv_heads, self.scale, out=out[:nd], splits=b.decode_splits,
                                           ws_o=ws.ws_o, ws_ml=ws.ws_ml)
                ev_out.record(side)
            ops.paged_prefill_attention(q, arena, i, b.block_tables, b.seq_lens, b.prefill_tiles, b.query_start,
                                        b.positions, c.n_q_heads, c.n_kv_heads, self.scale, out=out)
            main.wait_event(ev_out)
            return out
        if nd:
            ops.paged_decode_attention(q[:nd], arena, i, b.block_tables[:nd], b.seq_lens[:nd], c.n_q_heads,
                                       c.n_kv_heads, self.scale, out=out[:nd], splits=b.decode_splits,
                                       ws_o=ws.ws_o, ws_ml=ws.ws_ml)
        if t > nd:
            ops.paged_prefill_attention(q, arena, i, b.block_tables, b.seq_lens, b.prefill_tiles, b.query_start,
                                        b.positions, c.n_q_heads, c.n_kv_heads, self.scale, out=out)
        return out

    def _attn_side_stream(self):
        """Side stream of the mixed-step attention overlap (LAKEB_ATTN_OVERLAP=1; off outside CUDA
        and while a graph is being captured)."""
        if self.device.type != "cuda" or not ATTN_OVERLAP[0] or torch.cuda.is_current_stream_capturing():
            return None
        st = getattr(self, "_side", None)
        if st is None:
            st = self._side = torch.cuda.Stream(self.device)
        return st

    def _qkv(self, i: int, x: torch.Tensor, b: ForwardBatch, arena: torch.Tensor, ws: Workspace, t: int):
        c = self.cfg
        p = f"layers.{i}."
        if not c.qk_norm:
            ops.linear_qkv(x, self.w[p + "qkv_proj"], ws.q[:t], self.rope_cs, b.positions, b.slots, arena, i,
                           c.n_q_heads, c.n_kv_heads, b.peer_arena, b.peer_slots)
            return
        if x.is_cuda and c.head_dim == 128:  # per-head q/k RMSNorm fused into the QKV epilogue
            ops.linear_qkv(x, self.w[p + "qkv_proj"], ws.q[:t], self.rope_cs, b.positions, b.slots, arena, i,
                           c.n_q_heads, c.n_kv_heads, b.peer_arena, b.peer_slots, self.w[p + "q_norm"],
                           self.w[p + "k_norm"], c.rms_eps)
            return
        # Qwen3: per-head RMSNorm on q and k before RoPE.
        qkv = ops.linear(x, self.w[p + "qkv_proj"], out=ws.extra["qkv"][:t])
        d = c.head_dim
        qh = qkv[:, : c.q_size].reshape(t * c.n_q_heads, d)
        kh = qkv[:, c.q_size:c.q_size + c.kv_size].reshape(t * c.n_kv_heads, d)
        qn = ops.rms_norm(qh.contiguous(), self.w[p + "q_norm"], c.rms_eps).view(t, c.n_q_heads, d).float()
        kn = ops.rms_norm(kh.contiguous(), self.w[p + "k_norm"], c.rms_eps).view(t, c.n_kv_heads, d).float()
        v = qkv[:, c.q_size + c.kv_size:].reshape(t, c.n_kv_heads, d).float()
        qr = ref.apply_rope(qn, b.positions, self.rope_cs)
        kr = ref.apply_rope(kn, b.positions, self.rope_cs)
        ws.q[:t].copy_(qr.reshape(t, -1))
        ref.write_kv(arena, i, b.slots, kr, v)
        if b.peer_arena is not None and b.peer_slots is not None:
            ref.write_kv(b.peer_arena, i, b.peer_slots, kr, v)

    def _mlp(self, i: int, x: torch.Tensor, h: torch.Tensor, ws: Workspace, t: int) -> None:
        p = f"layers.{i}."
        if self.moe is not None:
            self.moe.forward(i, x, h, ws, t)
            return
        c = self.cfg
        if c.intermediate % 128 == 0:
            act = ops.linear_swiglu(x, self.w[p + "gate_up_proj"], out=ws.act[:t])
        else:  # plain [gate; up] layout (oracle path for odd sizes)
            gu = ref.linear(x, self.w[p + "gate_up_proj"])
            act = (torch.nn.functional.silu(gu[:, : c.intermediate]) * gu[:, c.intermediate:]).to(x.dtype)
        ops.linear_residual(act, self.w[p + "down_proj"], h, out=h)

    def forward(self, b: ForwardBatch, arena: torch.Tensor, ws: Workspace):
        """Run one step. Returns sampled token ids (int32 [R]) or fp32 logits [R, V] if b.want_logits."""
        c = self.cfg
        t = b.num_tokens
        h, x = ws.h[:t], ws.x[:t]
        ready = self.layer_ready
        if ready is not None:
            torch.cuda.current_stream(self.device).wait_event(ready["embed"])
        ops.embedding(b.input_ids, self.w["embed_tokens"], out=h)
        for i in range(c.n_layers):
            p = f"layers.{i}."
            if ready is not None:  # layer-async cold start: this layer's weights may still be in flight
                torch.cuda.current_stream(self.device).wait_event(ready[i])
            with nvtx(p):
                ops.rms_norm(h, self.w[p + "input_layernorm"], c.rms_eps, out=x)
                self._qkv(i, x, b, arena, ws, t)
                attn = self._attention(i, b, arena, ws, t)
                ops.linear_residual(attn, self.w[p + "o_proj"], h, out=h)
                ops.rms_norm(h, self.w[p + "post_attention_layernorm"], c.rms_eps, out=x)
                self._mlp(i, x, h, ws, t)
        if self.moe is not None and self.moe.ep is not None:
            self.moe.ep.end_step()  # expert-parallel wait targets: the bases advance by this step's totals
        r = b.sample_rows.shape[0]
        if r == 0:
            return ws.tokens[:0]
        fx = ws.fx[:r]
        if ready is not None:
            torch.cuda.current_stream(self.device).wait_event(ready["head"])
        torch.index_select(h, 0, b.sample_rows, out=fx)
        ops.rms_norm(fx, self.w["norm"], c.rms_eps, out=fx)
        if b.want_logits:
            return ops.linear(fx, self.w["lm_head"], out_dtype=torch.float32)
        return ops.linear_argmax(fx, self.w["lm_head"], bitmask=b.bitmask, keys=ws.keys[:r], out=ws.tokens[:r])
