"""Expert-parallel group over NVLink peer memory (one process per GPU).

Experts are split across the group (rank r owns experts [r*E/W, (r+1)*E/W));
attention and the router are replicated and each rank serves its own
requests. Per MoE layer, with parity p = layer % 2:

    dispatch (one kernel): top-k routing, each token row stored straight into
        the owner rank's gathered[p] segment of the chosen expert (slot from a
        system-scope atomic on the owner's count[p]), with the slot it must
        come back to; +1 per CTA on every owner's dispatch counter
    wait     the owner waits for every rank's dispatch (counts are final)
    experts  grouped tcgen05 GEMMs over the gathered rows; the down GEMM's
        scatter epilogue stores each result row into the source rank's
        comb[p] slot (P2P stores), +1 per CTA on every source's combine counter
    combine  the source waits for every owner, h += sum_k w_k * comb[p][t, k]

Every rank takes every step (ranks with no tokens still dispatch nothing,
serve their experts and signal), so counter totals agree across ranks. A
buffer of parity p is rewritten two layers later only after a chain of waits
that includes every reader's finish.

Wait targets are a device-resident base per counter family plus an offset
within the step (a kernel argument); end_step() adds the step's totals to the
bases with one small kernel. A step captured in a CUDA graph therefore replays
with fresh targets, which lets expert-parallel decode steps run from graphs.

Symmetric buffer (one cudaMalloc per rank, IPC-mapped by every peer):
    gathered[2] [epr*cap, hidden] bf16 | slot[2], src[2] [epr*cap] int32 |
    count[2] [epr] int32 | comb[2] [max_tokens*top_k, hidden] bf16 |
    counters dispatch[2][world], combine[2][world] u64
"""
from __future__ import annotations

import math

import torch

from ..ops._ext import native


class EPGroup:
    def __init__(self, rank: int, world: int, device, max_tokens: int, hidden: int, n_experts: int, top_k: int,
                 group=None):
        import torch.distributed as dist

        if n_experts % world:
            raise ValueError(f"{n_experts} experts do not split over {world} ranks")
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.hidden, self.top_k = hidden, top_k
        self.n_experts, self.epr = n_experts, n_experts // world
        self.max_tokens = max_tokens
        # every token of every rank may pick the same expert
        self.cap = (world * max_tokens + 127) // 128 * 128
        rows = self.epr * self.cap
        lay, off = {}, 0

        def add(name, nbytes):
            nonlocal off
            lay[name] = off
            off += (nbytes + 255) // 256 * 256

        for p in range(2):
            add(f"g{p}", rows * hidden * 2)
            add(f"s{p}", rows * 4)
            add(f"r{p}", rows * 4)
            add(f"n{p}", self.epr * 4)
            add(f"c{p}", max_tokens * top_k * hidden * 2)
        add("cnt", 4 * world * 8)
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
        self.gathered = [self._view(f"g{p}", torch.bfloat16, (rows, hidden)) for p in range(2)]
        self.slot = [self._view(f"s{p}", torch.int32, (rows,)) for p in range(2)]
        self.src = [self._view(f"r{p}", torch.int32, (rows,)) for p in range(2)]
        self.count = [self._view(f"n{p}", torch.int32, (self.epr,)) for p in range(2)]
        self.comb = [self._view(f"c{p}", torch.bfloat16, (max_tokens * top_k, hidden)) for p in range(2)]
        # within-step offsets of the wait targets; the device bases hold every earlier step's totals
        self.expect = {("d", p): 0 for p in range(2)}
        self.expect.update({("c", p): 0 for p in range(2)})
        self._fam = list(self.expect)
        self.bases = torch.zeros(len(self._fam), dtype=torch.int64, device=self.device)
        self._c = C
        self.down_grid = C.gemm_grid(rows, hidden, hidden, 7)  # grouped: data-parallel, K does not change the grid
        dist.barrier(group=group)

    def _view(self, name, dtype, shape):
        n = math.prod(shape) * torch.tensor([], dtype=dtype).element_size()
        o = self.lay[name]
        return self.buf[o:o + n].view(dtype).view(*shape)

    def _ptr(self, rank: int, name: str) -> int:
        return self.base[rank] + self.lay[name]

    def _base(self, fam: str, p: int) -> int:
        return self.bases.data_ptr() + self._fam.index((fam, p)) * 8

    def end_step(self) -> None:
        """Close a step: the bases advance by the step's totals (stream-ordered after every
        kernel of the step, and captured with it) and the offsets restart."""
        deltas = [self.expect[f] for f in self._fam]
        if any(deltas):
            self._c.tp_advance(self.bases.data_ptr(), deltas)
        for f in self._fam:
            self.expect[f] = 0

    def _cnt(self, rank: int, fam: str, p: int) -> int:
        idx = (0 if fam == "d" else 2 * self.world) + p * self.world
        return self.base[rank] + self.lay["cnt"] + idx * 8

    # ---------------------------------------------------------------- one MoE layer
    def layer(self, p: int, x: torch.Tensor, logits: torch.Tensor, wts: torch.Tensor, h: torch.Tensor,
              w_gate_up: torch.Tensor, w_down: torch.Tensor, act: torch.Tensor, status) -> None:
        C, W = self._c, self.world
        t = x.shape[0]
        C.moe_dispatch(logits, x, wts, self.n_experts, self.top_k, self.cap, W, self.rank,
                       [self._ptr(r, f"g{p}") for r in range(W)], [self._ptr(r, f"s{p}") for r in range(W)],
                       [self._ptr(r, f"r{p}") for r in range(W)], [self._ptr(r, f"n{p}") for r in range(W)],
                       [self._cnt(r, "d", p) for r in range(W)], status)
        self.expect[("d", p)] += C.moe_dispatch_grid()
        C.wait_counters(self._cnt(self.rank, "d", p), W, self.expect[("d", p)], status, base=self._base("d", p))
        C.gemm_grouped(self.gathered[p], w_gate_up, act, 2, self.count[p], self.cap, status=status)
        tp = dict(world=W, rank=self.rank, rows_per_rank=1, rs_cnt=[self._cnt(r, "c", p) for r in range(W)])
        C.gemm_grouped(act, w_down, None, 7, self.count[p], self.cap, row_slot=self.slot[p], row_rank=self.src[p],
                       dst_ptrs=[self._ptr(r, f"c{p}") for r in range(W)], tp=tp, status=status)
        self.expect[("c", p)] += self.down_grid
        self.count[p].zero_()  # consumed; peers refill it two layers on, after waits that follow this point
        C.moe_combine(h, self.comb[p][: t * self.top_k], wts, self.top_k, self._cnt(self.rank, "c", p), W,
                      self.expect[("c", p)], status, wait_base=self._base("c", p))
