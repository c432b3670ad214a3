"""Dispatch layer: every op takes torch tensors and runs the sm_100a kernel for
CUDA inputs (raising if the native module is missing) or the fp32 oracle for
CPU inputs."""
from __future__ import annotations

import torch

from ..oracle import ops_ref as ref
from ._ext import native
from .fp8 import Fp8Weight, unpack


def _dense(w):
    return w.dequant() if isinstance(w, Fp8Weight) else w

_STATUS: dict[int, torch.Tensor] = {}
# Number of lake_b200 kernel launches issued from Python (graph replays add their captured count).
LAUNCHES = [0]


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels write error codes into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS[idx] = t
    return t


_ERRORS = {1: "mbarrier wait timed out", 2: "peer flag wait timed out", 3: "index out of bounds", 4: "bad argument"}


class KernelError(RuntimeError):
    """A kernel recorded an error code in its device's status word. `timeout`: a bounded wait
    (an mbarrier phase or a peer's flag) ran out of time, the code a lost peer produces."""

    def __init__(self, device_index: int, code: int):
        self.device_index, self.code = device_index, code
        super().__init__(f"lake_b200 kernel error on cuda:{device_index}: {_ERRORS.get(code, code)}")

    @property
    def timeout(self) -> bool:
        return self.code in (1, 2)


def check_status(device: torch.device | None = None) -> None:
    """Raise KernelError if any kernel on `device` recorded an error (synchronises on the word)."""
    for idx, t in list(_STATUS.items()):
        if device is not None and device.index is not None and idx != device.index:
            continue
        code = int(t.item())
        if code:
            t.zero_()
            raise KernelError(idx, code)


# ------------------------------------------------------------------ GEMMs
def linear(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """out = a @ w.T with a [M, K], w [N, K] (bf16); out bf16 or fp32."""
    dt = out_dtype or (out.dtype if out is not None else a.dtype)
    if a.is_cuda:
        if out is None:
            out = torch.empty(a.shape[0], w.shape[0], dtype=dt, device=a.device)
        wq, ws = unpack(w)
        native().linear(a, wq, out, status_word(a.device), 0, ws)
        LAUNCHES[0] += 1
        return out
    r = ref.linear(a, _dense(w)).to(dt)
    if out is not None:
        out.copy_(r)
        return out
    return r


def linear_residual(a: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """out = residual + a @ w.T (out may be residual itself)."""
    if a.is_cuda:
        if out is None:
            out = torch.empty_like(residual)
        wq, ws = unpack(w)
        native().linear_residual(a, wq, residual, out, status_word(a.device), ws)
        LAUNCHES[0] += 1
        return out
    r = (residual.float() + ref.linear(a, _dense(w))).to(residual.dtype)
    if out is not None:
        out.copy_(r)
        return out
    return r


def linear_swiglu(a: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up with w_gate_up in the tile-interleaved layout (see interleave_gate_up)."""
    if out is None:
        out = torch.empty(a.shape[0], w_gate_up.shape[0] // 2, dtype=a.dtype, device=a.device)
    if a.is_cuda:
        if isinstance(w_gate_up, Fp8Weight) and w_gate_up.swiglu_tile != 128:
            raise ValueError("fp8 SwiGLU weights use the 128-row gate/up interleave (ops.fp8.quantize_gate_up)")
        wq, ws = unpack(w_gate_up)
        native().linear_swiglu(a, wq, out, status_word(a.device), None, ws)
        LAUNCHES[0] += 1
        return out
    tile = w_gate_up.swiglu_tile if isinstance(w_gate_up, Fp8Weight) else 256
    out.copy_(ref.swiglu_from_interleaved(ref.linear(a, _dense(w_gate_up)), tile).to(out.dtype))
    return out


def linear_qkv(a: torch.Tensor, w_qkv: torch.Tensor, q_out: torch.Tensor, rope_cs: torch.Tensor,
               positions: torch.Tensor, slots: torch.Tensor, arena: torch.Tensor, layer: int,
               n_q_heads: int, n_kv_heads: int, peer_arena: torch.Tensor | None = None,
               peer_slots: torch.Tensor | None = None, q_norm: torch.Tensor | None = None,
               k_norm: torch.Tensor | None = None, qk_eps: float = 1e-6) -> torch.Tensor:
    """QKV projection with RoPE (and, with q_norm/k_norm, per-head RMSNorm before RoPE as in
    Qwen3). q -> q_out; K, V -> arena at `slots` (and peer_arena at peer_slots)."""
    if a.is_cuda:
        wq, ws = unpack(w_qkv)
        native().linear_qkv(a, wq, q_out, rope_cs, positions, slots, arena, layer, n_q_heads, n_kv_heads,
                            peer_arena, peer_slots, status_word(a.device), None, q_norm, k_norm, qk_eps, ws)
        LAUNCHES[0] += 1
        return q_out
    acc = ref.linear(a, _dense(w_qkv))
    t = a.shape[0]
    d = arena.shape[-1]
    q = acc[:, : n_q_heads * d].view(t, n_q_heads, d)
    k = acc[:, n_q_heads * d:(n_q_heads + n_kv_heads) * d].view(t, n_kv_heads, d)
    v = acc[:, (n_q_heads + n_kv_heads) * d:].view(t, n_kv_heads, d)
    if q_norm is not None and k_norm is not None:
        q = ref.rms_norm(q, q_norm, qk_eps)
        k = ref.rms_norm(k, k_norm, qk_eps)
    q = ref.apply_rope(q, positions, rope_cs)
    k = ref.apply_rope(k, positions, rope_cs)
    q_out.copy_(q.reshape(t, -1).to(q_out.dtype))
    ref.write_kv(arena, layer, slots, k, v)
    if peer_arena is not None and peer_slots is not None:
        ref.write_kv(peer_arena, layer, peer_slots, k, v)
    return q_out


def linear_argmax(a: torch.Tensor, w: torch.Tensor, bitmask: torch.Tensor | None = None,
                  keys: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy token ids (int32 [M]) of a @ w.T without materialising the logits."""
    m = a.shape[0]
    if a.is_cuda:
        if keys is None:
            keys = torch.empty(m, dtype=torch.int64, device=a.device)
        if out is None:
            out = torch.empty(m, dtype=torch.int32, device=a.device)
        wq, ws = unpack(w)
        native().linear_argmax(a, wq, keys, bitmask, status_word(a.device), None, ws)
        native().unpack_argmax(keys, out, m)
        LAUNCHES[0] += 2
        return out
    r = ref.greedy(ref.linear(a, _dense(w)), bitmask)
    if out is not None:
        out.copy_(r)
        return out
    return r


def greedy_from_keys(keys: torch.Tensor) -> torch.Tensor:
    return (0xFFFFFFFF - (keys & 0xFFFFFFFF)).to(torch.int32)


# ------------------------------------------------------------------ attention
def decode_splits(num_seqs: int, n_kv_heads: int, max_blocks: int) -> int:
    return int(native().decode_splits(num_seqs, n_kv_heads, max_blocks))


def paged_decode_attention(q: torch.Tensor, arena: torch.Tensor, layer: int, block_tables: torch.Tensor,
                           seq_lens: torch.Tensor, n_q_heads: int, n_kv_heads: int, scale: float,
                           out: torch.Tensor | None = None, splits: int | None = None,
                           ws_o: torch.Tensor | None = None, ws_ml: torch.Tensor | None = None) -> torch.Tensor:
    """One query row per sequence; row s attends to keys [0, seq_lens[s])."""
    n = seq_lens.shape[0]
    if out is None:
        out = torch.empty(q.shape[0], n_q_heads * arena.shape[-1], dtype=q.dtype, device=q.device)
    if q.is_cuda:
        if splits is None:
            splits = decode_splits(n, n_kv_heads, block_tables.shape[1])
        if splits > 1 and (ws_o is None or ws_ml is None):
            g = n_q_heads // n_kv_heads
            ws_o = torch.empty(n * n_kv_heads * splits * g * ref.HEAD_DIM, dtype=torch.float32, device=q.device)
            ws_ml = torch.empty(n * n_kv_heads * splits * g * 2, dtype=torch.float32, device=q.device)
        native().paged_decode(q, out, arena, layer, block_tables, seq_lens, n_q_heads, n_kv_heads, scale, splits,
                              ws_o, ws_ml, status_word(q.device))
        LAUNCHES[0] += 2 if splits > 1 else 1
        return out
    qs = torch.arange(n + 1, dtype=torch.int32)
    pos = (seq_lens - 1).to(torch.int32)
    r = ref.paged_attention(q[:n], arena, layer, block_tables, seq_lens, qs, pos, n_q_heads, n_kv_heads, scale)
    out[:n].copy_(r.to(out.dtype))
    return out


PREFILL_TILE = 128  # query rows per tile of the tensor-core prefill kernel


def build_prefill_tiles(query_start: list[int], pos_start: list[int], tile: int = PREFILL_TILE,
                        device: torch.device | str = "cpu") -> torch.Tensor:
    """int32 [n_tiles, 4] of (seq, first query row, n queries, first query position)."""
    rows = []
    for s in range(len(query_start) - 1):
        a, b = query_start[s], query_start[s + 1]
        t = a
        while t < b:
            n = min(tile, b - t)
            rows.append((s, t, n, pos_start[s] + (t - a)))
            t += n
    if not rows:
        return torch.zeros(0, 4, dtype=torch.int32, device=device)
    return torch.tensor(rows, dtype=torch.int32, device=device)


def paged_prefill_attention(q: torch.Tensor, arena: torch.Tensor, layer: int, block_tables: torch.Tensor,
                            seq_lens: torch.Tensor, tiles: torch.Tensor, query_start: torch.Tensor,
                            positions: torch.Tensor, n_q_heads: int, n_kv_heads: int, scale: float,
                            out: torch.Tensor | None = None, tensor_core: bool = True) -> torch.Tensor:
    """Causal attention of packed query rows against each sequence's paged context.

    tensor_core=True runs the tcgen05 kernel (tiles of up to PREFILL_TILE rows);
    False runs the warp-MMA kernel (tiles of up to 64 rows)."""
    if out is None:
        out = torch.empty(q.shape[0], n_q_heads * arena.shape[-1], dtype=q.dtype, device=q.device)
    if q.is_cuda:
        native().paged_prefill(q, out, arena, layer, block_tables, seq_lens, tiles, n_q_heads, n_kv_heads, scale,
                               status_word(q.device), tensor_core)
        LAUNCHES[0] += 1
        return out
    r = ref.paged_attention(q, arena, layer, block_tables, seq_lens, query_start, positions, n_q_heads,
                            n_kv_heads, scale)
    out.copy_(r.to(out.dtype))
    return out


# ------------------------------------------------------------------ elementwise
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        native().rmsnorm(x, w, out, eps)
        LAUNCHES[0] += 1
        return out
    out.copy_(ref.rms_norm(x, w, eps).to(out.dtype))
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
    if table.is_cuda:
        native().embedding(ids, table, out, status_word(table.device))
        LAUNCHES[0] += 1
        return out
    out.copy_(table[ids.long()])
    return out


def greedy_sample(logits: torch.Tensor, bitmask: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    if logits.is_cuda:
        if out is None:
            out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
        native().argmax(logits, bitmask, out)
        LAUNCHES[0] += 1
        return out
    r = ref.greedy(logits, bitmask)
    if out is not None:
        out.copy_(r)
        return out
    return r


def apply_token_bitmask(logits: torch.Tensor, bitmask: torch.Tensor) -> torch.Tensor:
    """In place: disallowed tokens (bit 0) -> -inf."""
    if logits.is_cuda:
        native().apply_bitmask(logits, bitmask)
        LAUNCHES[0] += 1
        return logits
    logits.copy_(ref.apply_bitmask(logits, bitmask))
    return logits


def chain_reject_sample(draft: torch.Tensor, draft_off: torch.Tensor, target: torch.Tensor,
                        target_off: torch.Tensor, max_out: int):
    """Verify draft chains against target argmax tokens. Returns (tokens [n, max_out], lengths [n])."""
    n = draft_off.shape[0] - 1
    out = torch.full((n, max_out), -1, dtype=torch.int32, device=draft.device)
    out_len = torch.zeros(n, dtype=torch.int32, device=draft.device)
    if draft.is_cuda:
        native().chain_reject(draft, draft_off, target, target_off, out, out_len)
        LAUNCHES[0] += 1
        return out, out_len
    d_off, t_off = draft_off.tolist(), target_off.tolist()
    dl = [draft[d_off[i]:d_off[i + 1]].tolist() for i in range(n)]
    tl = [target[t_off[i]:t_off[i] + (d_off[i + 1] - d_off[i]) + 1].tolist() for i in range(n)]
    for i, acc in enumerate(ref.chain_reject(dl, tl)):
        out[i, : len(acc)] = torch.tensor(acc, dtype=torch.int32)
        out_len[i] = len(acc)
    return out, out_len


def resolve_tokens(ids: torch.Tensor, prev: torch.Tensor) -> None:
    """In place: ids[i] < 0 -> prev[-1 - ids[i]] (tokens the previous, still in-flight step sampled)."""
    if ids.is_cuda:
        native().resolve_tokens(ids, prev)
        LAUNCHES[0] += 1
        return
    neg = ids < 0
    if bool(neg.any()):
        j = (-1 - ids[neg]).long()
        ids[neg] = torch.where(j < prev.numel(), prev[j.clamp(max=max(prev.numel() - 1, 0))], torch.zeros_like(j)).to(
            ids.dtype)


def page_copy(src: torch.Tensor, dst: torch.Tensor, src_ids: torch.Tensor, dst_ids: torch.Tensor,
              page_bytes: int, sub_off: int = 0, sub_bytes: int | None = None) -> None:
    """dst page dst_ids[i] <- src page src_ids[i] (page-major byte buffers)."""
    if sub_bytes is None:
        sub_bytes = page_bytes
    if src.is_cuda or dst.is_cuda:
        native().page_copy(src, dst, src_ids, dst_ids, page_bytes, sub_off, sub_bytes,
                           status_word(src.device if src.is_cuda else dst.device))
        LAUNCHES[0] += 1
        return
    s = src.view(torch.uint8).view(-1, page_bytes)
    d = dst.view(torch.uint8).view(-1, page_bytes)
    d[dst_ids.long(), sub_off:sub_off + sub_bytes] = s[src_ids.long(), sub_off:sub_off + sub_bytes]
