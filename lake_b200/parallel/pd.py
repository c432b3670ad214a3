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

Tensor-parallel instances: a P or D instance may be a TP group of T ranks. The
group's first rank (leader) holds the links to the partner instances and makes
every scheduling decision; it sends its decisions (granted pages, adopted
requests, step boundaries) to the other ranks through a GroupCtl, which replay
them in the same order, so every rank of the group schedules the same batch and
allocates the same pages. P's TP rank i holds the same KV heads as D's TP rank i
and stores them into that rank's arena, so the fused P->D store stays one peer
write per rank. P's followers acknowledge each step; the leader reports a
prefill done only after every rank's stores completed.

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
# leader -> follower commands inside a TP instance
G_STEP, G_PHASE, G_EXIT, G_EVENTS = 11, 12, 13, 14
EV_SUBMIT, EV_ADOPT, EV_GRANT, EV_DIRECT = 21, 22, 23, 24


class GroupCtl:
    """Leader -> followers command rings of one tensor-parallel instance, plus one
    acknowledgement ring per follower. Collective construction: the leader creates the
    rings before the group's rendezvous, followers open them after it."""

    def __init__(self, job: str, members: list[int], rank: int, create: bool):
        self.members = list(members)
        self.rank = rank
        self.is_leader = rank == members[0]
        lead = members[0]
        names = {f: (f"lakeb_{job}_g{lead}f{f}_cmd", f"lakeb_{job}_g{lead}f{f}_ack") for f in members[1:]}
        if self.is_leader:
            self.rings = {f: (ShmRing(c, create=create), ShmRing(a, capacity_words=1024, create=create))
                          for f, (c, a) in names.items()} if create else None
        else:
            self.rings = None
        self._names = names

    def open(self) -> None:
        """Followers attach to the leader's rings (after the rendezvous)."""
        if not self.is_leader and self.rings is None:
            c, a = self._names[self.rank]
            self.cmd, self.ackr = ShmRing(c), ShmRing(a, capacity_words=1024)
            self.rings = {}

    @property
    def size(self) -> int:
        return len(self.members)

    def send(self, msg) -> None:
        for cmd, _ in self.rings.values():
            cmd.put_wait(msg)

    def recv(self, timeout_s: float = 600.0) -> np.ndarray:
        t0 = time.perf_counter()
        spins = 0
        while True:
            m = self.cmd.get()
            if m is not None:
                return m
            spins += 1
            if spins > 1000:
                time.sleep(0.0001)
            if time.perf_counter() - t0 > timeout_s:
                raise TimeoutError(f"TP follower {self.rank}: no command from the leader in {timeout_s} s")

    def ack(self, step: int) -> None:
        self.ackr.put_wait([step])

    def wait_acks(self, step: int, timeout_s: float = 600.0) -> None:
        t0 = time.perf_counter()
        for f, (_, ack) in self.rings.items():
            while True:
                m = ack.get()
                if m is not None:
                    if int(m[0]) != step:
                        raise RuntimeError(f"TP follower {f} acknowledged step {int(m[0])}, expected {step}")
                    break
                if time.perf_counter() - t0 > timeout_s:
                    raise TimeoutError(f"TP follower {f} did not finish step {step} in {timeout_s} s")


def _pack_events(events: list[tuple], cmd: int = G_STEP) -> np.ndarray:
    """[cmd, n, (kind, idx, a, b, len(list1), *list1, len(list2), *list2)...]"""
    parts = [np.array([cmd, len(events)], dtype=np.int64)]
    for kind, idx, a, b, l1, l2 in events:
        parts.append(np.array([kind, idx, a, b, len(l1)], dtype=np.int64))
        parts.append(np.asarray(l1, dtype=np.int64))
        parts.append(np.array([len(l2)], dtype=np.int64))
        parts.append(np.asarray(l2, dtype=np.int64))
    return np.concatenate(parts)


def _unpack_events(m: np.ndarray) -> list[tuple]:
    n = int(m[1])
    pos = 2
    out = []
    for _ in range(n):
        kind, idx, a, b, n1 = (int(x) for x in m[pos:pos + 5])
        pos += 5
        l1 = m[pos:pos + n1].tolist()
        pos += n1
        n2 = int(m[pos])
        pos += 1
        l2 = m[pos:pos + n2].tolist()
        pos += n2
        out.append((kind, idx, a, b, l1, l2))
    return out


class DecodeSide:
    """Decode instance's side of PD-split. It may be fed by several prefill instances
    (many-to-one): each grant goes to the partner with the fewest requests outstanding."""

    def __init__(self, eng: LLMEngine, links: list[tuple[ShmRing, ShmRing]], ctl: GroupCtl | None = None,
                 direct_min_hit: float = 0.5):
        self.eng = eng
        # D-direct: a prompt whose prefix this instance already holds (a session's next turn) is
        # prefilled here instead of on a prefill instance, when its cached share is at least this
        self.direct_min_hit = direct_min_hit
        self.direct = 0
        self.local = 0  # requests prefilled here because the prefill partners were saturated
        self.links = links  # (to_p, from_p) per prefill partner (the leader's; empty on followers)
        self.ctl = ctl
        self.pending: dict[int, tuple] = {}
        self.outstanding = [0] * len(links)
        self.next_idx = 0
        self.kv_bytes = 0  # prompt KV bytes P wrote into this arena (all ranks of the instance)
        self.page_bytes = eng.arena[0].numel() * eng.arena.element_size()
        self.group_size = ctl.size if ctl is not None else 1
        self.events: list[tuple] = []  # leader: decisions since the last step, replayed by followers
        self.exit = False

    @property
    def is_follower(self) -> bool:
        return self.ctl is not None and not self.ctl.is_leader

    def local_hit(self, prompt: list[int]) -> int:
        """Prompt tokens this instance's prefix cache holds (whole blocks, last token excluded)."""
        from ..engine.block_pool import chain_block_hashes

        bs = self.eng.ec.block_size
        hashes = chain_block_hashes(prompt, bs, full_only=True)[:(len(prompt) - 1) // bs]
        return self.eng.pool.peek(hashes) * bs

    def submit(self, prompt: list[int], max_new_tokens: int, local: bool = False) -> str | None:
        """Start a request: returns the engine request id it will run under ("pd-N" once its
        prefill instance reports back, "dd-N" when prefilled here), or None if no pages are free.
        `local`: prefill it here in any case (COLOCATED on this instance: its prefill partners
        are saturated and this instance's chunked mixed steps take the overflow)."""
        if local:
            self.local += 1
        if local or (self.direct_min_hit > 0 and len(prompt) > 1
                     and self.local_hit(prompt) >= self.direct_min_hit * len(prompt)):
            # D-direct (reference mode selection: local hit -> D_DIRECT): extend the cached prefix here
            rid = f"dd-{self.next_idx}"
            if self.ctl is not None:
                self.events.append((EV_DIRECT, self.next_idx, max_new_tokens, 0, list(prompt), []))
            self.next_idx += 1
            self.eng.add_request(list(prompt), max_new_tokens, rid=rid)
            self.direct += 0 if local else 1
            return rid
        blocks = self.eng.reserve_blocks(len(prompt))
        if self.ctl is not None:
            self.events.append((EV_SUBMIT, self.next_idx if blocks is not None else -1, max_new_tokens, 0,
                                list(prompt), blocks or []))
        if blocks is None:
            return None
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
        return f"pd-{idx}"

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
                    self.kv_bytes += len(blocks) * self.page_bytes * self.group_size
                    if self.ctl is not None:
                        self.events.append((EV_ADOPT, idx, tok, 0, [], []))
                    n += 1
        return n

    def step(self):
        """One decode iteration; a TP leader first sends its decisions and the step to the followers."""
        if self.ctl is not None:
            self.ctl.send(_pack_events(self.events))
            self.events = []
        return self.eng.step()

    def phase(self, code: int) -> None:
        """TP leader: tell the followers a phase of the caller's loop ended (they return from
        follow()); decisions made since the last step go first."""
        if self.ctl is not None:
            if self.events:
                self.ctl.send(_pack_events(self.events, G_EVENTS))
                self.events = []
            self.ctl.send([G_PHASE, code])

    def follow(self, on_step=None) -> int:
        """TP follower: replay the leader's decisions and steps until a phase marker (returns
        its code) or the exit command (returns -1)."""
        while True:
            m = self.ctl.recv()
            kind = int(m[0])
            if kind == G_PHASE:
                return int(m[1])
            if kind == G_EXIT:
                self.exit = True
                return -1
            for ev, idx, a, _, l1, l2 in _unpack_events(m):
                if ev == EV_SUBMIT:
                    got = self.eng.reserve_blocks(len(l1))
                    if (got or []) != l2 or (got is None) != (idx < 0):
                        raise RuntimeError(f"TP decode follower page allocation diverged: {got} vs {l2}")
                    if idx >= 0:
                        self.pending[idx] = (l1, got, a, time.perf_counter(), 0)
                elif ev == EV_ADOPT:
                    prompt, blocks, max_new, arrival, _ = self.pending.pop(idx)
                    self.eng.adopt_prefilled(f"pd-{idx}", prompt, a, blocks, max_new, arrival=arrival)
                elif ev == EV_DIRECT:
                    self.next_idx = idx + 1
                    self.eng.add_request(l1, a, rid=f"dd-{idx}")
            if kind == G_EVENTS:
                continue
            outs = self.eng.step()
            if on_step is not None:
                on_step(outs)

    def mark(self, code: int) -> None:
        for to_p, _ in self.links:
            to_p.put_wait([MARK, code])

    def close(self) -> None:
        """Release this side's rings (the creator's close also unlinks them)."""
        _close_rings([r for link in self.links for r in link], self.ctl)

    def shutdown(self) -> None:
        for to_p, _ in self.links:
            to_p.put_wait([EXIT])
        if self.ctl is not None and self.ctl.is_leader:
            self.ctl.send([G_EXIT])

    @property
    def inflight(self) -> int:
        return len(self.pending) + len(self.eng.scheduler.running) + len(self.eng.scheduler.waiting)

    @property
    def saturated(self) -> bool:
        """Every prefill partner has at least `queue` grants outstanding (see `queue_depth`)."""
        return bool(self.links) and min(self.outstanding) >= self.queue_depth

    queue_depth = 8


class PrefillSide:
    """Prefill instance's side of PD-split. It may serve several decode instances
    (one-to-many, single-GPU instances): `links` holds one (from_d, to_d) ring pair per decode
    instance, a grant's destination is the link it came on, and it exits once every decode
    instance has sent EXIT."""

    def __init__(self, eng: LLMEngine, from_d: ShmRing | None, to_d: ShmRing | None, ctl: GroupCtl | None = None,
                 links: list[tuple[ShmRing, ShmRing]] | None = None):
        self.eng = eng
        self.links = links if links is not None else ([(from_d, to_d)] if from_d is not None else [])
        if len(self.links) > 1 and ctl is not None:
            raise ValueError("a tensor-parallel prefill instance feeds one decode instance")
        self.from_d, self.to_d = (self.links[0] if self.links else (from_d, to_d))  # the leader's first link
        self.ctl = ctl
        self.marks: list[int] = []
        self.exit = False
        self.exits = 0
        self.origin: dict[str, tuple[int, int]] = {}  # engine request id -> (link, the decode side's index)
        self.first_tokens = 0
        self.events: list[tuple] = []
        self.steps = 0
        self.step_t0 = 0.0  # host clock (time.perf_counter) when the last step began

    @property
    def is_follower(self) -> bool:
        return self.ctl is not None and not self.ctl.is_leader

    def poll(self) -> None:
        for li, (from_d, _) in enumerate(self.links):
            while True:
                m = from_d.get()
                if m is None:
                    break
                kind = int(m[0])
                if kind == GRANT:
                    idx, nb = int(m[1]), int(m[3])
                    blocks = m[4:4 + nb].tolist()
                    plen = int(m[4 + nb])
                    prompt = m[5 + nb:5 + nb + plen].tolist()
                    rid = f"pd-{idx}" if len(self.links) == 1 else f"pd{li}-{idx}"
                    self.origin[rid] = (li, idx)
                    self.eng.add_remote_prefill(prompt, blocks, rid=rid, dest=li if len(self.links) > 1 else 0)
                    if self.ctl is not None:
                        self.events.append((EV_GRANT, idx, 0, 0, prompt, blocks))
                elif kind == MARK:
                    self.marks.append(int(m[1]))
                elif kind == EXIT:
                    self.exits += 1
                    self.exit = self.exits >= len(self.links)

    def mark_complete(self, code: int) -> bool:
        """Every decode instance this side serves has sent MARK `code` (consumed here)."""
        if self.marks.count(code) < max(1, len(self.links)):
            return False
        self.marks = [c for c in self.marks if c != code]
        return True

    def step(self) -> int:
        self.step_t0 = time.perf_counter()
        self.poll()
        if self.ctl is not None:
            self.ctl.send(_pack_events(self.events))
            self.events = []
        outs = self.eng.step()
        self.steps += 1
        if self.ctl is not None:
            if self.eng.device.type == "cuda":
                torch.cuda.synchronize(self.eng.device)
            self.ctl.wait_acks(self.steps)  # every rank's K/V stores into D's arenas completed
        for o in outs:
            li, idx = self.origin.pop(o.rid, (0, None))
            if idx is None:
                idx = int(o.rid.split("-", 1)[1])
            self.links[li][1].put_wait([DONE, idx, o.new_tokens[0]])
        self.first_tokens += len(outs)
        return len(outs)

    def phase(self, code: int) -> None:
        if self.ctl is not None:
            if self.events:
                self.ctl.send(_pack_events(self.events, G_EVENTS))
                self.events = []
            self.ctl.send([G_PHASE, code])

    def follow(self, on_step=None) -> int:
        """TP follower: replay the leader's grants and steps until a phase marker (returns its
        code) or the exit command (returns -1)."""
        while True:
            m = self.ctl.recv()
            kind = int(m[0])
            if kind == G_PHASE:
                return int(m[1])
            if kind == G_EXIT:
                self.exit = True
                return -1
            for _, idx, _, _, prompt, blocks in _unpack_events(m):
                self.eng.add_remote_prefill(prompt, blocks, rid=f"pd-{idx}")
            if kind == G_EVENTS:
                continue
            self.step_t0 = time.perf_counter()
            self.eng.step()
            self.steps += 1
            if self.eng.device.type == "cuda":
                torch.cuda.synchronize(self.eng.device)
            self.ctl.ack(self.steps)
            if on_step is not None:
                on_step()

    def idle(self) -> bool:
        return not self.eng.has_unfinished()

    def close(self) -> None:
        _close_rings([r for link in self.links for r in link if r is not None] or
                     [r for r in (self.from_d, self.to_d) if r is not None], self.ctl)


def _close_rings(rings, ctl) -> None:
    for r in rings:
        r.close()
    if ctl is not None:
        if ctl.rings:
            for cmd, ack in ctl.rings.values():
                cmd.close()
                ack.close()
        for r in (getattr(ctl, "cmd", None), getattr(ctl, "ackr", None)):
            if r is not None:
                r.close()


def ring_names(job: str, d_rank: int, p_rank: int) -> tuple[str, str]:
    return f"lakeb_{job}_d{d_rank}p{p_rank}_to_p", f"lakeb_{job}_d{d_rank}p{p_rank}_from_p"


def connect_pair(eng: LLMEngine, role: str, rank: int, partner, group, job: str,
                 shm_path: str | None = None, members: list[int] | None = None,
                 decode_instances: list[int] | None = None):
    """Wire prefill and decode instances. Each decode instance D exports its arena and its
    leader creates one ring pair per prefill partner; a prefill instance P maps its D's
    arena and its leader opens their rings. Collective over `group` (every rank calls it).

    `members`: the global ranks of this rank's instance in TP order (None or one rank for a
    single-GPU instance); an instance is named by its leader `members[0]`. `partner` is, on
    the decode side, the list of prefill leaders feeding this instance; on the prefill side,
    the decode instance's member list (or its single rank). P's TP rank i maps the arena of
    D's TP rank i (the same KV heads).

    `decode_instances` (prefill side, single-GPU instances): the ranks of several single-GPU
    decode instances this prefill instance serves (one-to-many); it maps every one of their
    arenas and opens a ring pair to each. Each of those decode instances lists this rank among
    its `partner` prefill leaders."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    members = list(members) if members else [rank]
    leader = members[0]
    ctl = GroupCtl(job, members, rank, create=rank == leader) if len(members) > 1 else None
    handle = export_tensor(eng.arena, shm_path) if role == "decode" else None
    links = []
    if role == "decode" and rank == leader:
        partners = list(partner) if isinstance(partner, (list, tuple)) else [partner]
        for p in partners:
            a, b = ring_names(job, rank, p)
            links.append((ShmRing(a, create=True), ShmRing(b, create=True)))
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, role, handle), group=group)
    if ctl is not None:
        ctl.open()
    if role == "decode":
        return DecodeSide(eng, links, ctl)
    if decode_instances:
        if len(members) > 1:
            raise ValueError("a tensor-parallel prefill instance feeds one decode instance")
        if eng.arena.is_cuda:
            torch.cuda.set_device(eng.arena.device)
        arenas = []
        for d in decode_instances:
            peer = import_tensor([g for g in gathered if g[0] == d][0][2])
            if peer.shape[1:] != eng.arena.shape[1:]:
                raise ValueError(f"peer arena layout {tuple(peer.shape)} does not match {tuple(eng.arena.shape)}")
            arenas.append(peer)
        eng.set_peer_arenas(arenas)
        plinks = []
        for d in decode_instances:
            a, b = ring_names(job, d, rank)
            plinks.append((ShmRing(a), ShmRing(b)))
        return PrefillSide(eng, None, None, None, links=plinks)
    d_members = list(partner) if isinstance(partner, (list, tuple)) else [partner]
    if len(d_members) != len(members):
        raise ValueError(f"prefill instance of {len(members)} ranks cannot feed a decode instance of "
                         f"{len(d_members)} (TP sizes must match: rank i stores KV heads of rank i)")
    mine = d_members[members.index(rank)]
    h = [g for g in gathered if g[0] == mine][0][2]
    if eng.arena.is_cuda:
        torch.cuda.set_device(eng.arena.device)
    peer = import_tensor(h)
    if peer.shape[1:] != eng.arena.shape[1:]:
        raise ValueError(f"peer arena layout {tuple(peer.shape)} does not match {tuple(eng.arena.shape)}")
    eng.runner.peer_arena = peer
    if rank != leader:
        return PrefillSide(eng, None, None, ctl)
    to_p_name, from_p_name = ring_names(job, d_members[0], rank)
    return PrefillSide(eng, ShmRing(to_p_name), ShmRing(from_p_name), ctl)


def serve_prefill(side: PrefillSide, until_mark: int | None = None, idle_sleep_s: float = 0.0002,
                  on_step=None) -> None:
    """Prefill loop: step while there is work; return on EXIT or once `until_mark` arrives.
    A TP follower replays its leader instead; the leader tells it where the loop ended."""
    if side.is_follower:
        while not side.exit:
            code = side.follow(on_step)
            if until_mark is not None and code == until_mark:
                return
        return
    while not side.exit:
        if until_mark is not None and side.mark_complete(until_mark):
            side.phase(until_mark)
            return
        if side.idle():
            side.poll()
            if side.idle() and not side.exit and (until_mark is None or side.marks.count(until_mark)
                                                  < max(1, len(side.links))):
                time.sleep(idle_sleep_s)
            continue
        side.step()
        if side.eng.device.type == "cuda":
            torch.cuda.synchronize(side.eng.device)
        if on_step is not None:
            on_step()
    if side.ctl is not None:
        side.ctl.send([G_EXIT])  # grants received after the last step are never computed
