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
    """Decode instance's side of PD-split. It may be fed by several prefill instances
    (many-to-one): each grant goes to the partner with the fewest requests outstanding."""

    def __init__(self, eng: LLMEngine, links: list[tuple[ShmRing, ShmRing]]):
        self.eng = eng
        self.links = links  # (to_p, from_p) per prefill partner
        self.to_p, self.from_p = links[0]
        self.pending: dict[int, tuple] = {}
        self.outstanding = [0] * len(links)
        self.next_idx = 0
        self.kv_bytes = 0  # prompt KV bytes P wrote into this arena
        self.page_bytes = eng.arena[0].numel() * eng.arena.element_size()

    def submit(self, prompt: list[int], max_new_tokens: int) -> bool:
        blocks = self.eng.reserve_blocks(len(prompt))
        if blocks is None:
            return False
        idx = self.next_idx
        self.next_idx += 1
        li = min(range(len(self.links)), key=lambda i: self.outstanding[i])
        self.outstanding[li] += 1
        self.pending[idx] = (list(prompt), blocks, max_new_tokens, time.perf_counter(), li)
        msg = np.empty(5 + len(blocks) + len(prompt), dtype=np.int64)
        msg[:4] = (GRANT, idx, max_new_tokens, len(blocks))
        msg[4:4 + len(blocks)] = blocks
        msg[4 + len(blocks)] = len(prompt)
        msg[5 + len(blocks):] = prompt
        self.links[li][0].put_wait(msg)
        return True

    def poll(self) -> int:
        n = 0
        for _, from_p in self.links:
            while True:
                m = from_p.get()
                if m is None:
                    break
                if m[0] == DONE:
                    idx, tok = int(m[1]), int(m[2])
                    prompt, blocks, max_new, arrival, li = self.pending.pop(idx)
                    self.outstanding[li] -= 1
                    self.eng.adopt_prefilled(f"pd-{idx}", prompt, tok, blocks, max_new, arrival=arrival)
                    self.kv_bytes += len(blocks) * self.page_bytes
                    n += 1
        return n

    def mark(self, code: int) -> None:
        for to_p, _ in self.links:
            to_p.put_wait([MARK, code])

    def shutdown(self) -> None:
        for to_p, _ in self.links:
            to_p.put_wait([EXIT])

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


def ring_names(job: str, d_rank: int, p_rank: int) -> tuple[str, str]:
    return f"lakeb_{job}_d{d_rank}p{p_rank}_to_p", f"lakeb_{job}_d{d_rank}p{p_rank}_from_p"


def connect_pair(eng: LLMEngine, role: str, rank: int, partner, group, job: str,
                 shm_path: str | None = None):
    """Wire prefill and decode processes: each decode instance D exports its arena and
    creates one ring pair per prefill partner; a prefill instance P maps its D's arena and
    opens their rings. `partner` is D's list of prefill ranks (or one rank) on the decode
    side and P's decode rank on the prefill side. Collective over `group` (every rank calls it)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    handle = export_tensor(eng.arena, shm_path) if role == "decode" else None
    if role == "decode":
        partners = list(partner) if isinstance(partner, (list, tuple)) else [partner]
        links = []
        for p in partners:
            a, b = ring_names(job, rank, p)
            links.append((ShmRing(a, create=True), ShmRing(b, create=True)))
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, role, handle), group=group)
    if role == "decode":
        return DecodeSide(eng, links)
    h = [g for g in gathered if g[0] == partner][0][2]
    if eng.arena.is_cuda:
        torch.cuda.set_device(eng.arena.device)
    peer = import_tensor(h)
    if peer.shape[1:] != eng.arena.shape[1:]:
        raise ValueError(f"peer arena layout {tuple(peer.shape)} does not match {tuple(eng.arena.shape)}")
    eng.runner.peer_arena = peer
    to_p_name, from_p_name = ring_names(job, partner, rank)
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
