"""Prefill/decode disaggregation inside one box.

A decode instance (D) owns its requests. To start one it reserves pages in its
own KV arena and grants them to its prefill partner (P) together with the
prompt. P runs the prompt through its engine; the QKV projection's epilogue
stores every K/V row both into P's own arena (P's attention reads it) and into
D's granted pages through the IPC-mapped peer arena, so the P->D KV transfer
happens inside the GEMM, tile by tile, over NVLink. P then reports the first
sampled token and D adopts the request straight into its decode batch.

Control messages travel through shared-memory rings (parallel.channel); bulk
KV never leaves the kernels.

Reference parity: the PD-split mode of the Router (go/router/modeselect.go:58-69)
and the TransferService Publish/Pull protocol (rust/transfer/src/service.rs:
184-318), which the reference implements as host-side byte copies.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from ..engine.llm_engine import LLMEngine
from .channel import ShmRing
from .peer import export_tensor, import_tensor

GRANT, DONE, MARK, EXIT = 1, 2, 3, 4


class DecodeSide:
    def __init__(self, eng: LLMEngine, to_p: ShmRing, from_p: ShmRing):
        self.eng = eng
        self.to_p, self.from_p = to_p, from_p
        self.pending: dict[int, tuple] = {}
        self.next_idx = 0
        self.kv_bytes = 0  # prompt KV bytes P wrote into this arena
        self.page_bytes = eng.arena[0].numel() * eng.arena.element_size()

    def submit(self, prompt: list[int], max_new_tokens: int) -> bool:
        blocks = self.eng.reserve_blocks(len(prompt))
        if blocks is None:
            return False
        idx = self.next_idx
        self.next_idx += 1
        self.pending[idx] = (list(prompt), blocks, max_new_tokens, time.perf_counter())
        msg = np.empty(5 + len(blocks) + len(prompt), dtype=np.int64)
        msg[:4] = (GRANT, idx, max_new_tokens, len(blocks))
        msg[4:4 + len(blocks)] = blocks
        msg[4 + len(blocks)] = len(prompt)
        msg[5 + len(blocks):] = prompt
        self.to_p.put_wait(msg)
        return True

    def poll(self) -> int:
        n = 0
        while True:
            m = self.from_p.get()
            if m is None:
                return n
            if m[0] == DONE:
                idx, tok = int(m[1]), int(m[2])
                prompt, blocks, max_new, arrival = self.pending.pop(idx)
                self.eng.adopt_prefilled(f"pd-{idx}", prompt, tok, blocks, max_new, arrival=arrival)
                self.kv_bytes += len(blocks) * self.page_bytes
                n += 1

    def mark(self, code: int) -> None:
        self.to_p.put_wait([MARK, code])

    def shutdown(self) -> None:
        self.to_p.put_wait([EXIT])

    @property
    def inflight(self) -> int:
        return len(self.pending) + len(self.eng.scheduler.running) + len(self.eng.scheduler.waiting)


class PrefillSide:
    def __init__(self, eng: LLMEngine, from_d: ShmRing, to_d: ShmRing):
        self.eng = eng
        self.from_d, self.to_d = from_d, to_d
        self.marks: list[int] = []
        self.exit = False
        self.first_tokens = 0

    def poll(self) -> None:
        while True:
            m = self.from_d.get()
            if m is None:
                return
            kind = int(m[0])
            if kind == GRANT:
                idx, nb = int(m[1]), int(m[3])
                blocks = m[4:4 + nb].tolist()
                plen = int(m[4 + nb])
                prompt = m[5 + nb:5 + nb + plen].tolist()
                self.eng.add_remote_prefill(prompt, blocks, rid=f"pd-{idx}")
            elif kind == MARK:
                self.marks.append(int(m[1]))
            elif kind == EXIT:
                self.exit = True

    def step(self) -> int:
        self.poll()
        outs = self.eng.step()
        for o in outs:
            idx = int(o.rid.split("-", 1)[1])
            self.to_d.put_wait([DONE, idx, o.new_tokens[0]])
        self.first_tokens += len(outs)
        return len(outs)

    def idle(self) -> bool:
        return not self.eng.has_unfinished()


def ring_names(job: str, d_rank: int) -> tuple[str, str]:
    return f"lakeb_{job}_d{d_rank}_to_p", f"lakeb_{job}_d{d_rank}_from_p"


def connect_pair(eng: LLMEngine, role: str, rank: int, partner: int, group, job: str,
                 shm_path: str | None = None):
    """Wire a prefill/decode pair of processes: D exports its arena and creates the rings,
    P maps the arena and opens the rings. Collective over `group` (every rank calls it)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    handle = export_tensor(eng.arena, shm_path) if role == "decode" else None
    d_rank = rank if role == "decode" else partner
    to_p_name, from_p_name = ring_names(job, d_rank)
    if role == "decode":
        to_p = ShmRing(to_p_name, create=True)
        from_p = ShmRing(from_p_name, create=True)
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, role, handle), group=group)
    if role == "decode":
        return DecodeSide(eng, to_p, from_p)
    h = [g for g in gathered if g[0] == partner][0][2]
    if eng.arena.is_cuda:
        torch.cuda.set_device(eng.arena.device)
    peer = import_tensor(h)
    if peer.shape[1:] != eng.arena.shape[1:]:
        raise ValueError(f"peer arena layout {tuple(peer.shape)} does not match {tuple(eng.arena.shape)}")
    eng.runner.peer_arena = peer
    return PrefillSide(eng, ShmRing(to_p_name), ShmRing(from_p_name))


def serve_prefill(side: PrefillSide, until_mark: int | None = None, idle_sleep_s: float = 0.0002) -> None:
    """Prefill loop: step while there is work; return on EXIT or once `until_mark` arrives."""
    while not side.exit:
        if until_mark is not None and until_mark in side.marks:
            side.marks.remove(until_mark)
            return
        if side.idle():
            side.poll()
            if side.idle() and not side.exit and (until_mark is None or until_mark not in side.marks):
                time.sleep(idle_sleep_s)
            continue
        side.step()
        if side.eng.device.type == "cuda":
            torch.cuda.synchronize(side.eng.device)
