"""Turns a SchedulerOutput into device tensors, runs the model, returns tokens.

Step metadata (token ids, positions, KV slots, block tables, sequence lengths,
prefill tiles, sample rows) is packed on the host into pinned staging buffers
and copied to fixed device buffers with two ``cudaMemcpyAsync`` calls; the
sampled token ids come back through a pinned buffer. Pure-decode steps replay
a CUDA graph captured per batch-size bucket (all buffers have fixed
addresses; tensor-parallel steps included, their collective targets are
device-resident), mixed prefill/decode steps launch eagerly.

Reference parity: ModelRunner.prepare_inputs / prepare_attn / execute_model
(python/lake/engine/model_runner.py:182-323) and InputBuffers.materialize
(python/lake/engine/input_batch.py:81-133), which build the same geometry as
host lists; AttentionMetadata (python/lake/engine/attention_metadata.py:15-89).
"""
from __future__ import annotations

import bisect
import time

import numpy as np
import torch

from .. import ops
from ..models.llama import DecoderLM, ForwardBatch
from .request import PENDING
from .scheduler import SchedulerOutput

GRAPH_BUCKETS = [1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512]


class ModelRunner:
    def __init__(self, model: DecoderLM, arena: torch.Tensor, max_tokens: int, max_seqs: int,
                 max_blocks_per_seq: int, use_cuda_graphs: bool = True, block_size: int = 16, row_multiple: int = 1,
                 max_samples: int | None = None):
        self.model = model
        self.arena = arena
        self.device = model.device
        self.cuda = self.device.type == "cuda"
        self.max_tokens = max_tokens
        self.max_seqs = max_seqs
        # sampled rows per step: one per sequence, or one per position of a verify chunk
        self.max_samples = max_samples = max(max_samples or max_seqs, max_seqs)
        self.maxb = max_blocks_per_seq
        self.bs = block_size
        self.row_multiple = row_multiple  # tensor parallel: rows padded to a multiple of the group size
        self.vocab_words = (model.cfg.vocab + 31) // 32
        cfg = model.cfg
        self.max_splits = 1
        if self.cuda:
            self.max_splits = max(ops.decode_splits(n, cfg.n_kv_heads // row_multiple, max_blocks_per_seq)
                                  for n in range(1, max_seqs + 1))
        self.ws = model.new_workspace(max_tokens, max_samples, max_seqs, self.max_splits)
        self.host_meta = getattr(model, "wants_host_meta", False)
        # int32 staging: ids | pos | seq_lens | qstart | tiles | block_tables
        self.max_tiles = max_tokens // 64 + max_seqs
        self._lay = {}
        off = 0
        for name, n in (("ids", max_tokens), ("pos", max_tokens), ("lens", max_seqs), ("qstart", max_seqs + 1),
                        ("tiles", self.max_tiles * 4), ("bt", max_seqs * max_blocks_per_seq)):
            self._lay[name] = (off, n)
            off += (n + 3) // 4 * 4  # keep every region 16-byte aligned (tiles are read as int4)
        self.n_i32 = off
        pin = self.cuda
        self.h_i32 = torch.zeros(off, dtype=torch.int32, pin_memory=pin)
        # int64 staging: slots [max_tokens] | sample rows [max_samples] | peer slots [max_tokens]
        self.h_i64 = torch.zeros(2 * max_tokens + max_samples, dtype=torch.int64, pin_memory=pin)
        self.peer_off = max_tokens + max_samples
        self.peer_arena: torch.Tensor | None = None  # decode instance's arena (IPC-mapped) for fused P->D
        # host tier slab (pinned, device-mapped) the QKV epilogue also writes decode K/V into, page by
        # page as `req.mirror_blocks` names them: the D -> pool write-behind done by the kernel
        self.mirror_arena: torch.Tensor | None = None
        # sampled ids come back through two pinned buffers (one step may be in flight while the
        # previous one is read); d_prev keeps the last step's ids on the device for the next
        # step's PENDING inputs (overlapped scheduling)
        self.h_toks = [torch.zeros(max_samples, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self.h_tok = self.h_toks[0]
        self._tok_flip = 0
        self.d_prev = torch.zeros(max(1, max_seqs), dtype=torch.int32, device=self.device)
        # the device status word comes back with each step's tokens (one pinned int per in-flight step)
        self.h_status = [torch.zeros(1, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self.has_pending = False
        self.relay = False  # keep sampled ids in d_prev (set by an engine that overlaps steps)
        self._staged = None  # event after the last metadata copy: the pinned staging is reusable
        self.d_i32 = torch.zeros(off, dtype=torch.int32, device=self.device)
        self.d_i64 = torch.zeros(2 * max_tokens + max_samples, dtype=torch.int64, device=self.device)
        self.np_i32 = self.h_i32.numpy()
        self.np_i64 = self.h_i64.numpy()
        self.use_graphs = use_cuda_graphs and self.cuda
        # capture a bucket's graph on first use; off for expert parallelism, whose capture warm-up
        # runs the group's exchange and so must happen on every rank at once (capture_graphs)
        self.lazy_capture = True
        self.graphs: dict[int, tuple] = {}
        self.graph_launches: dict[int, int] = {}
        self.has_peer = False
        self.stream = torch.cuda.current_stream(self.device) if self.cuda else None
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.last_device_ms = 0.0
        self.time_device = False
        self.gap_ms = 0.0  # with time_device: summed device time between consecutive timed steps
        self._prev_ev1 = None

    # ------------------------------------------------------------ views
    def _v(self, buf, name, n=None, shape=None):
        off, cap = self._lay[name]
        t = buf[off: off + (n if n is not None else cap)]
        return t.reshape(*shape) if shape else t

    def _batch_views(self, t: int, s: int, ntiles: int, nrows: int, nd: int, splits: int,
                     bitmask=None, peer=None) -> ForwardBatch:
        d, d64 = self.d_i32, self.d_i64
        return ForwardBatch(
            input_ids=self._v(d, "ids", t), positions=self._v(d, "pos", t), slots=d64[:t],
            block_tables=self._v(d, "bt", s * self.maxb, (s, self.maxb)), seq_lens=self._v(d, "lens", s),
            n_decode=nd, prefill_tiles=self._v(d, "tiles", ntiles * 4, (ntiles, 4)),
            query_start=self._v(d, "qstart", s + 1),
            sample_rows=d64[self.max_tokens: self.max_tokens + nrows], bitmask=bitmask,
            peer_arena=(self.peer_arena if self.peer_arena is not None else self.mirror_arena) if peer else None,
            peer_slots=d64[self.peer_off:self.peer_off + t] if peer else None, decode_splits=splits)

    # ------------------------------------------------------------ host packing
    def _pack(self, out: SchedulerOutput, pad_decode_to: int = 0):
        """Fill the pinned staging buffers. Returns (t, s, ntiles, nrows, nd)."""
        if self._staged is not None:  # the previous step's copies may still be queued on the stream
            self._staged.synchronize()
            self._staged = None
        bs, maxb = self.bs, self.maxb
        ids = self._v(self.np_i32, "ids")
        pos = self._v(self.np_i32, "pos")
        lens = self._v(self.np_i32, "lens")
        qst = self._v(self.np_i32, "qstart")
        tiles = self._v(self.np_i32, "tiles", shape=(self.max_tiles, 4))
        bt = self._v(self.np_i32, "bt", shape=(self.max_seqs, maxb))
        slots = self.np_i64[: self.max_tokens]
        rows = self.np_i64[self.max_tokens: self.max_tokens + self.max_samples]
        pslots = self.np_i64[self.peer_off:]
        mirror = self.mirror_arena is not None and self.peer_arena is None
        self.has_peer = False
        self.has_pending = False
        row = 0
        nrows = 0
        ntiles = 0
        chunks = out.chunks
        nd = len(out.decode)
        s = 0
        for ch in chunks:
            req = ch.req
            n = ch.n
            p0 = ch.start
            if n == 1:
                tok = req.tokens_slice(p0, p0 + 1)[0]
                if tok == PENDING:  # sampled by the in-flight step: resolved on the device
                    tok = -1 - req.meta["pslot"]
                    self.has_pending = True
                ids[row] = tok
                pos[row] = p0
                slots[row] = req.block_ids[p0 // bs] * bs + p0 % bs
            else:
                # a verify chunk is the last token followed by its draft
                ids[row:row + n] = (req.tokens_slice(p0, p0 + n) if not ch.draft
                                    else req.tokens_slice(p0, p0 + 1) + ch.draft)
                pr = np.arange(p0, p0 + n, dtype=np.int64)
                pos[row:row + n] = pr
                blk = np.asarray(req.block_ids, dtype=np.int64)
                slots[row:row + n] = blk[pr // bs] * bs + pr % bs
            rb = req.remote_blocks
            mb = req.mirror_blocks if mirror else None
            if rb is not None:
                self.has_peer = True
                pr = np.arange(p0, p0 + n, dtype=np.int64)
                rbk = np.asarray(rb, dtype=np.int64)
                pslots[row:row + n] = rbk[pr // bs] * bs + pr % bs
            elif mb:
                self.has_peer = True
                for j in range(n):  # rows of pages the agent gave a host slot
                    pg = (p0 + j) // bs
                    sl = mb.get(pg)
                    pslots[row + j] = sl * bs + (p0 + j) % bs if sl is not None else -1
            else:
                pslots[row:row + n] = -1
            nb = len(req.block_ids)
            bt[s, :nb] = _block_ids_np(req)
            lens[s] = p0 + n
            qst[s] = row
            if s >= nd:
                t0 = row
                while t0 < row + n:
                    k = min(ops.core.PREFILL_TILE, row + n - t0)
                    tiles[ntiles] = (s, t0, k, p0 + (t0 - row))
                    ntiles += 1
                    t0 += k
            ns = ch.n_samples  # the last row, or every row of a verify chunk
            if ns == 1:
                rows[nrows] = row + n - 1
                nrows += 1
            elif ns:
                rows[nrows:nrows + ns] = np.arange(row + n - ns, row + n)
                nrows += ns
            row += n
            s += 1
            if s == nd and pad_decode_to > nd:
                # padding decode rows for a graph bucket: zero-length sequences, no KV write
                for j in range(nd, pad_decode_to):
                    ids[row] = 0
                    pos[row] = 0
                    slots[row] = -1
                    pslots[row] = -1
                    lens[s] = 0
                    qst[s] = row
                    rows[nrows] = row
                    nrows += 1
                    row += 1
                    s += 1
        qst[s] = row
        if mirror and pad_decode_to:
            self.has_peer = True  # the captured graph always reads the slot list (-1: no host copy)
        pad = -row % self.row_multiple
        if pad:  # rows outside every sequence: no KV write, never sampled
            ids[row:row + pad] = 0
            pos[row:row + pad] = 0
            slots[row:row + pad] = -1
            pslots[row:row + pad] = -1
            row += pad
        return row, s, ntiles, nrows, nd if not pad_decode_to else max(nd, pad_decode_to)

    def _h2d(self, t: int, s: int, nrows: int):
        # block tables are the largest piece: copy only the used rows
        off_bt, _ = self._lay["bt"]
        n32 = off_bt + s * self.maxb
        self.d_i32[:n32].copy_(self.h_i32[:n32], non_blocking=True)
        self.d_i64[:t].copy_(self.h_i64[:t], non_blocking=True)
        self.d_i64[self.max_tokens:self.max_tokens + nrows].copy_(
            self.h_i64[self.max_tokens:self.max_tokens + nrows], non_blocking=True)
        self.h2d_bytes += n32 * 4 + (t + nrows) * 8
        if self.has_peer:
            o = self.peer_off
            self.d_i64[o:o + t].copy_(self.h_i64[o:o + t], non_blocking=True)
            self.h2d_bytes += t * 8
        self._staged = torch.cuda.Event()
        self._staged.record()

    # ------------------------------------------------------------ graphs
    def _bucket(self, nd: int) -> int | None:
        i = bisect.bisect_left(GRAPH_BUCKETS, nd)
        if i == len(GRAPH_BUCKETS) or GRAPH_BUCKETS[i] > self.max_seqs:
            return None
        return GRAPH_BUCKETS[i]

    def _splits(self, nd: int) -> int:
        if not self.cuda or nd == 0:
            return 1
        return ops.decode_splits(nd, self.model.cfg.n_kv_heads // self.row_multiple, self.maxb)

    def _get_graph(self, bucket: int):
        g = self.graphs.get(bucket)
        if g is not None:
            return g
        splits = self._splits(bucket)
        t = bucket + (-bucket) % self.row_multiple  # rows as _pack pads them (tensor parallel)
        mirror = self.mirror_arena is not None and self.peer_arena is None
        batch = self._batch_views(t, bucket, 0, bucket, bucket, splits, peer=mirror)
        # the captured replay must see valid metadata: zero-length padding sequences
        self.d_i32.zero_()
        self.d_i64[:t].fill_(-1)
        if mirror:
            self.d_i64[self.peer_off:self.peer_off + t].fill_(-1)
        self.d_i64[self.max_tokens:self.max_tokens + bucket].copy_(torch.arange(bucket, device=self.device))
        # the warm-up forwards overwrite d_prev, which may hold the in-flight step's sampled ids
        # (overlapped scheduling, graph captured on first use): keep them
        prev = self.d_prev.clone() if self.relay else None
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._forward(batch, self.relay)
        torch.cuda.current_stream(self.device).wait_stream(s)
        if prev is not None:
            self.d_prev.copy_(prev)
        graph = torch.cuda.CUDAGraph()
        c0 = ops.core.LAUNCHES[0]
        with torch.cuda.graph(graph):
            toks = self._forward(batch, self.relay)
        self.graph_launches[bucket] = ops.core.LAUNCHES[0] - c0
        ops.core.LAUNCHES[0] = c0
        self.graphs[bucket] = (graph, toks)
        return self.graphs[bucket]

    def capture_graphs(self, max_bucket: int | None = None) -> None:
        if not self.use_graphs:
            return
        for b in GRAPH_BUCKETS:
            if b > self.max_seqs or (max_bucket and b > max_bucket):
                break
            self._get_graph(b)

    def _forward(self, batch: ForwardBatch, resolve: bool):
        """Model forward with the overlapped-scheduling token relay around it: PENDING inputs
        are read from d_prev first, and this step's sampled ids are kept in d_prev after."""
        if resolve:
            (getattr(self.model, "resolve_tokens", None) or ops.resolve_tokens)(batch.input_ids, self.d_prev)
        toks = self.model.forward(batch, self.arena, self.ws)
        n = toks.shape[0]
        if n and self.relay:
            self.d_prev[:n].copy_(toks[:n])
        return toks

    # ------------------------------------------------------------ execute
    def execute(self, out: SchedulerOutput, bitmask: torch.Tensor | None = None) -> list[int]:
        """Run one step; returns one sampled token per sampling chunk (chunk order).

        Requests with ``remote_blocks`` (prefill for a decode instance) get their
        K/V rows written into ``self.peer_arena`` too, by the QKV epilogue."""
        return self.collect(self.launch(out, bitmask))

    def launch(self, out: SchedulerOutput, bitmask: torch.Tensor | None = None):
        """Enqueue one step (metadata copies, graph replay or eager forward, the async copy of
        the sampled ids to a pinned buffer) without waiting for it; collect() returns its ids."""
        if out.is_empty:
            return None
        nd = len(out.decode)
        has_remote = any(c.req.remote_blocks is not None for c in out.prefill)
        pure_decode = not out.prefill and bitmask is None
        streaming = getattr(self.model, "layer_ready", None) is not None  # weights still loading: run eagerly
        bucket = self._bucket(nd) if (pure_decode and self.use_graphs and not streaming) else None
        if bucket is not None and bucket not in self.graphs and not self.lazy_capture:
            bucket = None  # expert-parallel ranks capture only together (capture_graphs): run this step eagerly
        t, s, ntiles, nrows, nd_eff = self._pack(out, pad_decode_to=bucket or 0)
        if not self.cuda:
            self._copy_cpu(t, s, nrows)
            batch = self._batch_views(t, s, ntiles, nrows, nd_eff, 1, bitmask, has_remote or self.has_peer)
            toks = self._forward(batch, self.has_pending)
            return ("cpu", toks[: sum(c.n_samples for c in out.chunks)].tolist())
        graph = None
        if bucket is not None:
            graph, toks = self._get_graph(bucket)  # capture (if new) before this step's metadata lands
        self._h2d(t, s, nrows)
        ev0 = ev1 = None
        if self.time_device:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        if graph is not None:
            graph.replay()
            ops.core.LAUNCHES[0] += self.graph_launches[bucket]
        else:
            batch = self._batch_views(t, s, ntiles, nrows, nd_eff, self._splits(nd_eff), bitmask,
                                      has_remote or self.has_peer)
            if self.host_meta:
                batch.host = {"rows": out.num_tokens, "lens": self._v(self.np_i32, "lens", s).tolist(),
                              "qstart": self._v(self.np_i32, "qstart", s + 1).tolist()}
            toks = self._forward(batch, self.has_pending)
        if ev1 is not None:
            ev1.record()
        nsamp = sum(c.n_samples for c in out.chunks)
        h = self.h_toks[self._tok_flip]
        hs = self.h_status[self._tok_flip]
        self._tok_flip ^= 1
        h[:nsamp].copy_(toks[:nsamp], non_blocking=True)
        hs.copy_(ops.core.status_word(self.device), non_blocking=True)
        self.d2h_bytes += nsamp * 4 + 4
        done = torch.cuda.Event()
        done.record()
        return ("cuda", h, nsamp, done, ev0, ev1, hs)

    def collect(self, handle) -> list[int]:
        """Wait for a launched step and return its sampled ids (chunk order)."""
        if handle is None:
            return []
        if handle[0] == "cpu":
            return handle[1]
        _, h, nsamp, done, ev0, ev1, hs = handle
        done.synchronize()
        if ev1 is not None:
            self.last_device_ms = ev0.elapsed_time(ev1)
            if self._prev_ev1 is not None:  # device time between the previous step's end and this one's start
                self.gap_ms += max(0.0, self._prev_ev1.elapsed_time(ev0))
            self._prev_ev1 = ev1
        code = int(hs[0])
        if code:  # a kernel of this step recorded an error: clear the word, fail the step
            ops.core.status_word(self.device).zero_()
            raise ops.core.KernelError(self.device.index or 0, code)
        return h[:nsamp].tolist()

    def execute_null(self) -> None:
        """A zero-token forward: every collective the model issues still runs (expert parallel)."""
        batch = self._batch_views(0, 0, 0, 0, 0, 1)
        self.model.forward(batch, self.arena, self.ws)
        torch.cuda.current_stream(self.device).synchronize()

    def _copy_cpu(self, t, s, nrows):
        self.d_i32.copy_(self.h_i32)
        self.d_i64.copy_(self.h_i64)


def _block_ids_np(req) -> np.ndarray:
    """The request's page ids as an int32 array, kept in step with `req.block_ids`: pages are
    only appended to the same list (a new list means a new allocation), so the cached array
    grows by its tail instead of converting the whole Python list every step."""
    ids = req.block_ids
    c = req.meta.get("bt_np")
    if c is None or req.meta.get("bt_src") is not ids or c[1] > len(ids):
        arr = np.asarray(ids, dtype=np.int32)
        req.meta["bt_np"] = (np.resize(arr, max(16, 2 * len(ids))), len(ids))
        req.meta["bt_src"] = ids
        return arr
    buf, n = c
    if n < len(ids):
        if len(ids) > buf.shape[0]:
            buf = np.resize(buf, 2 * len(ids))
        buf[n:len(ids)] = ids[n:]
        req.meta["bt_np"] = (buf, len(ids))
    return buf[:len(ids)]


def now() -> float:
    return time.perf_counter()
