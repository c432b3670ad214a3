"""Tensor-parallel group over NVLink peer memory (one process per GPU).

Each rank allocates ONE symmetric buffer (its own cudaMalloc, exported with
CUDA IPC and mapped by every peer) holding:

    a_full[3]  [world*Mr_max, hidden] bf16   inputs of the column-parallel GEMMs
                                              (all-gather targets: slot E for the
                                              embedding norm, then slots 0/1 alternate)
    recv[2]    [world, Mr_max, hidden] bf16   reduce-scatter receive buffers (alternate)
    fx         [max_samples, hidden]    bf16   lm_head input (sampled rows, gathered)
    amax       [max_samples]            u64    vocab-shard argmax keys
    counters   ag[4][world] rs[2][world] done[world]   u64, monotonically increasing

Kernels push data into peers' buffers with P2P stores and then add 1 per CTA
to the counter slot [my rank] of every destination; a waiting kernel compares
each source's counter with the running total this host tracks (every rank
issues the same calls with the same grids, so the totals agree). Buffer reuse
is safe by construction: a slot is written again only after a chain of
data-dependent waits that includes every reader's finish (two-deep rotation
for all-gather and reduce-scatter, a dedicated slot for the first norm of a
step, a dedicated lm_head buffer).

Expected totals are split in two: a device-resident base per counter family
(the totals at the start of the current step, in local memory) and a
within-step offset that is a kernel argument. A waiting kernel compares with
base + offset; end_step() launches a one-block kernel that adds the step's
totals to the bases. A step's offsets and totals depend only on its shape, so
a captured step replays with correct targets (CUDA graphs for decode) and
eager and replayed steps mix freely.
"""
from __future__ import annotations

import math

import torch

from ..ops._ext import native

SLOT_E, SLOT_FX = 2, 3  # all-gather counter families 0, 1 alternate; 2 = first norm of a step; 3 = lm_head rows


class TPGroup:
    def __init__(self, rank: int, world: int, device, max_tokens: int, hidden: int, max_samples: int,
                 group=None, status: torch.Tensor | None = None):
        import torch.distributed as dist

        assert 1 <= world <= 8
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.hidden = hidden
        self.mr_max = math.ceil(max_tokens / world)
        self.max_samples = max_samples
        self.status = status
        e = 2  # bf16 bytes
        rows = world * self.mr_max
        lay = {}
        off = 0

        def add(name, nbytes):
            nonlocal off
            lay[name] = off
            off += (nbytes + 255) // 256 * 256

        for s in range(3):
            add(f"a{s}", rows * hidden * e)
        for s in range(2):
            add(f"r{s}", world * self.mr_max * hidden * e)
        add("fx", max_samples * hidden * e)
        add("amax", max_samples * 8)
        self.n_cnt = 7 * world
        add("cnt", self.n_cnt * 8)
        self.lay, self.nbytes = lay, off
        C = native()
        with torch.cuda.device(self.device):
            self.buf = C.alloc_ipc_tensor([off], torch.uint8)
            handle = C.ipc_export(self.buf)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.peer_bufs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                self.peer_bufs.append(self.buf if r == rank else C.ipc_import(h, [off], torch.uint8))
        self.base = [b.data_ptr() for b in self.peer_bufs]
        # local typed views
        self.a_full = [self._view(self.buf, f"a{s}", torch.bfloat16, (rows, hidden)) for s in range(3)]
        self.recv = [self._view(self.buf, f"r{s}", torch.bfloat16, (world, self.mr_max, hidden)) for s in range(2)]
        self.fx = self._view(self.buf, "fx", torch.bfloat16, (max_samples, hidden))
        self.amax = self._view(self.buf, "amax", torch.int64, (max_samples,))
        self.cnt = self._view(self.buf, "cnt", torch.int64, (self.n_cnt,))
        self.expect = {("ag", s): 0 for s in range(4)}
        self.expect.update({("rs", s): 0 for s in range(2)})
        self.expect[("done", 0)] = 0
        self._fam = list(self.expect)  # family -> index into bases
        self.bases = torch.zeros(len(self._fam), dtype=torch.int64, device=self.device)
        self._c = C
        with torch.cuda.device(self.device):
            C.gemm_workspace_init()  # GEMM grids (and so the counter totals) are planned with it present
        dist.barrier(group=group)

    def _view(self, buf, name, dtype, shape):
        n = math.prod(shape) * torch.tensor([], dtype=dtype).element_size()
        o = self.lay[name]
        return buf[o:o + n].view(dtype).view(*shape)

    # ---------------------------------------------------------------- addresses
    def _cnt_ptr(self, rank: int, family: str, slot: int) -> int:
        idx = {"ag": 0, "rs": 4 * self.world, "done": 6 * self.world}[family] + slot * self.world
        return self.base[rank] + self.lay["cnt"] + idx * 8

    def _ptr(self, rank: int, name: str) -> int:
        return self.base[rank] + self.lay[name]

    def _base_ptr(self, family: str, slot: int) -> int:
        return self.bases.data_ptr() + self._fam.index((family, slot)) * 8

    def end_step(self) -> None:
        """Close a step: advance the device bases by the step's totals (stream-ordered after
        every kernel of the step; captured along with a graph) and restart the offsets."""
        deltas = [self.expect[f] for f in self._fam]
        if any(deltas):
            self._c.tp_advance(self.bases.data_ptr(), deltas)
        for f in self._fam:
            self.expect[f] = 0

    # ---------------------------------------------------------------- call builders
    def rows_per_rank(self, t: int) -> int:
        return math.ceil(t / self.world)

    def gemm_ag(self, slot: int, mr: int, wait_all: bool = False) -> dict:
        """Column-parallel GEMM over a_full[slot] (or fx): wait per row shard (or for all shards)."""
        d = dict(world=self.world, rank=self.rank, rows_per_rank=mr, ag_cnt=self._cnt_ptr(self.rank, "ag", slot),
                 ag_off=self.expect[("ag", slot)], ag_base=self._base_ptr("ag", slot),
                 m_rot=0 if wait_all else (self.rank * mr) // 128)
        if wait_all:
            d["rows_per_rank"] = 1 << 30
            d["ag_all"] = 1
        return d

    def gemm_rs(self, slot: int, mr: int, n: int, k: int, fp8: bool = False) -> dict:
        """Row-parallel GEMM ([world*mr, k] x [n, k]^T) whose epilogue pushes partial rows to their
        owners' recv[slot] (`fp8`: block-scaled fp8 weights, whose kernel has its own grid)."""
        d = dict(world=self.world, rank=self.rank, rows_per_rank=mr,
                 m_rot=(((self.rank + 1) % self.world) * mr) // 128,
                 rs_recv=[self._ptr(r, f"r{slot}") for r in range(self.world)],
                 rs_cnt=[self._cnt_ptr(r, "rs", slot) for r in range(self.world)])
        self.expect[("rs", slot)] += self._c.gemm_grid(self.world * mr, n, k, 6, fp8)
        return d

    def norm_push(self, mr: int, rs_slot: int | None, ag_slot: int, row_map: torch.Tensor | None = None,
                  store_h: bool = True) -> dict:
        """Reduce-scatter completion (+residual) + RMSNorm + all-gather push into a_full[ag_slot] (or fx)."""
        if ag_slot == SLOT_FX:
            dst = [self._ptr(r, "fx") for r in range(self.world)]
        else:
            dst = [self._ptr(r, f"a{ag_slot}") for r in range(self.world)]
        d = dict(world=self.world, rank=self.rank, rows_per_rank=mr, dst=dst, dst_ld=self.hidden,
                 ag_cnt=[self._cnt_ptr(r, "ag", ag_slot) for r in range(self.world)], store_h=int(store_h),
                 row_map=None if row_map is None else row_map.data_ptr())
        if rs_slot is not None:
            d.update(recv=self._ptr(self.rank, f"r{rs_slot}"), rs_cnt=self._cnt_ptr(self.rank, "rs", rs_slot),
                     rs_off=self.expect[("rs", rs_slot)], rs_base=self._base_ptr("rs", rs_slot))
        self.expect[("ag", ag_slot)] += self._c.tp_norm_grid(mr)
        return d

    def lm_argmax(self, mr_unused: int, n_rows: int, vocab_local: int, fp8: bool = False) -> dict:
        """lm_head GEMM over the gathered sampled rows (fx, [n_rows, hidden]) with the argmax epilogue."""
        d = self.gemm_ag(SLOT_FX, 0, wait_all=True)
        d.update(done_cnt=[self._cnt_ptr(r, "done", 0) for r in range(self.world)],
                 col_offset=self.rank * vocab_local)
        self.expect[("done", 0)] += self._c.gemm_grid(n_rows, vocab_local, self.hidden, 4, fp8)
        return d

    def argmax_combine(self, out: torch.Tensor, n: int) -> torch.Tensor:
        self._c.tp_argmax_combine([self._ptr(r, "amax") for r in range(self.world)],
                                  self._cnt_ptr(self.rank, "done", 0), self.expect[("done", 0)], out, n,
                                  self.status, self._base_ptr("done", 0))
        return out[:n]
