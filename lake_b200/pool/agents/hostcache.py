"""L1 (pinned host DRAM) tier under the engine's HBM prefix cache.

D -> pool: when a request finishes, every full page of its KV (prompt and
decode-extended tokens) that the pool does not hold yet is copied device ->
pinned host on a side stream (one cudaMemcpyAsync per page: pages are
contiguous in the page-first arena), ordered after the step that produced it
by an event. Pages stay resident in HBM as prefix cache.

pool -> P: when a request arrives, prompt pages missing from HBM but present
in L1 are copied host -> device into fresh pages on the same side stream and
registered in the engine's prefix cache; the compute stream waits for that
stream before the next step, so admission reuses them instead of recomputing.

HBM eviction: before the block pool hands out a cached page again, the
compute stream waits for that page's write-behind copy (if still in flight).
L1 itself is an LRU over pinned slots; its evictions are counted.

Kernel write-behind (mirror=True, the default for non-prefill instances): the
L1 slab is also the QKV epilogue's second KV target. Before each step the agent
gives every page of generated tokens that the step writes a reserved L1 slot
(`req.mirror_blocks`); the epilogue stores those rows' K/V into host memory as
it produces them (through the slab's device-mapped address), so when the
request finishes its decode-extended pages are already in L1 and are only
registered, not copied. Prompt pages (and the page shared by the prompt's end
and the first generated tokens) still take the copy at finish.

Reference parity: the L0<->L1 promote/demote path of
rust/tiered-store/src/engine.rs:495-606 and the SGLang-style host cache the
reference's engine targets (python/lake/engine/agent.py:15-41 contract).
"""
from __future__ import annotations

import time
from collections import OrderedDict

import torch

from ...engine.block_pool import chain_block_hashes
from ..types import FinishRequest, PreparePlan, ReadyHandle, StepStats


class HostCacheAgent:
    def __init__(self, engine, l1_blocks: int, node_id: str = "node-0", mirror: bool = True, durable=None):
        self.eng = engine
        self.node_id = node_id
        self.bs = engine.ec.block_size
        arena = engine.arena
        self.page_elems = arena[0].numel()
        cuda = arena.is_cuda
        self.l1 = torch.empty(l1_blocks, self.page_elems, dtype=arena.dtype, pin_memory=cuda)
        # the slab as a KV arena: the QKV epilogue's host-side write-behind target
        self.mirror_arena = self.l1.view(l1_blocks, *arena.shape[1:]) if mirror else None
        if self.mirror_arena is not None and cuda:
            from ...ops._ext import native

            native().register_host_arena(self.l1)  # checked pinned once, outside any graph capture
        self.reserved: set[int] = set()  # slots a running request's epilogue is writing into
        # optional durable tier (durable.DurableTier): finished pages are committed to L2 with
        # PutEnd in the background; their slots stay pinned until their bytes are taken
        self.durable = durable
        self.pinned: dict[int, int] = {}
        self._pin_lock = __import__("threading").Lock()
        self.slot_of: OrderedDict[bytes, int] = OrderedDict()  # LRU: oldest first
        self.free_slots = list(range(l1_blocks - 1, -1, -1))
        self.pending: dict[int, torch.cuda.Event] = {}  # device page -> write-behind copy event
        self.stream = torch.cuda.Stream(arena.device) if cuda else None
        self.stats = {"writeback_blocks": 0, "promoted_blocks": 0, "l1_evictions": 0, "evict_waits": 0,
                      "writeback_ms": 0.0, "promote_ms": 0.0, "kernel_written_blocks": 0, "copied_blocks": 0,
                      "mirror_slots_short": 0, "l2_promoted_blocks": 0, "pinned_skips": 0}
        engine.pool.on_evict = self._on_evict
        self._ready: int | None = None

    # ------------------------------------------------------------ L1 slots
    def _evict_lru(self) -> int | None:
        """Take the oldest L1 entry whose slot is not pinned by a durable commit in flight."""
        with self._pin_lock:
            pinned = set(self.pinned)
        for h, s in self.slot_of.items():
            if s in pinned:
                self.stats["pinned_skips"] += 1
                continue
            del self.slot_of[h]
            self.stats["l1_evictions"] += 1
            return s
        return None

    def _take_slot(self) -> int | None:
        """A slot outside the LRU (free, else the LRU's oldest unpinned); None when none is left."""
        if self.free_slots:
            return self.free_slots.pop()
        return self._evict_lru()

    def _pin(self, slot: int) -> None:
        with self._pin_lock:
            self.pinned[slot] = self.pinned.get(slot, 0) + 1

    def _unpin(self, slot: int) -> None:
        with self._pin_lock:
            n = self.pinned.get(slot, 0) - 1
            if n > 0:
                self.pinned[slot] = n
            else:
                self.pinned.pop(slot, None)

    def _release(self, slot: int) -> None:
        self.reserved.discard(slot)
        self.free_slots.append(slot)

    def _slot_for(self, h: bytes) -> int:
        s = self.slot_of.get(h)
        if s is not None:
            self.slot_of.move_to_end(h)
            return s
        s = self._take_slot()
        if s is None:
            raise RuntimeError("host tier: every L1 slot is reserved or pinned")
        self.slot_of[h] = s
        return s

    def _page(self, page: int) -> torch.Tensor:
        return self.eng.arena[page].view(-1)

    def _on_evict(self, page: int, h: bytes) -> None:
        ev = self.pending.pop(page, None)
        if ev is not None and not ev.query():
            torch.cuda.current_stream(self.eng.arena.device).wait_event(ev)
            self.stats["evict_waits"] += 1

    # ------------------------------------------------------------ D -> pool
    def on_request_finished(self, finish: FinishRequest) -> None:
        req = self.eng.requests.get(finish.req_id)
        if req is None:
            return
        t0 = time.perf_counter()
        toks = req.all_tokens
        n_full = min(req.num_computed, len(toks)) // self.bs
        hashes = chain_block_hashes(toks[: n_full * self.bs], self.bs, full_only=True)
        pages = req.meta.get("final_block_ids") or req.block_ids
        mirrored = req.mirror_blocks or {}
        req.mirror_blocks = None
        todo = []
        kernel_written = 0
        for i, (h, p) in enumerate(zip(hashes, pages)):
            slot = mirrored.pop(i, None)
            if h in self.slot_of:  # another request's copy is already in L1
                if slot is not None:
                    self._release(slot)
                self.slot_of.move_to_end(h)
                continue
            if slot is not None:  # written by the QKV epilogue as it was produced: register only
                self.reserved.discard(slot)
                self.slot_of[h] = slot
                kernel_written += 1
            else:
                todo.append((h, p))
        for slot in mirrored.values():  # pages that never filled up
            self._release(slot)
        self.stats["kernel_written_blocks"] += kernel_written
        self.stats["writeback_blocks"] += kernel_written
        ev = None
        if todo:
            ev = self._copy_behind(todo)
        self._commit_durable(req.rid, hashes, ev)
        self.stats["writeback_ms"] += (time.perf_counter() - t0) * 1000

    def _commit_durable(self, rid: str, hashes: list[bytes], ready) -> None:
        """Hand the request's full pages (now all in L1) to the durable tier, slots pinned."""
        if self.durable is None or not hashes:
            return
        chain = []
        for h in hashes:
            slot = self.slot_of.get(h)
            if slot is None:  # evicted already (L1 smaller than one request): the chain ends here
                break
            self._pin(slot)
            chain.append((h, slot, self.l1[slot].data_ptr(), self.durable.is_durable(h)))
        if chain and not all(c[3] for c in chain):
            self.durable.commit(rid, chain, ready, self._unpin)
        else:
            for _, slot, _, _ in chain:
                self._unpin(slot)

    def _copy_behind(self, todo):
        """Copy the pages device -> L1 (side stream on the GPU); returns the copies' event."""
        self.stats["copied_blocks"] += len(todo)
        if self.stream is None:
            for h, p in todo:
                self.l1[self._slot_for(h)].copy_(self._page(p))
        else:
            dev = self.eng.arena.device
            produced = torch.cuda.current_stream(dev).record_event()
            self.stream.wait_event(produced)
            with torch.cuda.stream(self.stream):
                for h, p in todo:
                    self.l1[self._slot_for(h)].copy_(self._page(p), non_blocking=True)
                ev = self.stream.record_event()
            for _, p in todo:
                self.pending[p] = ev
        self.stats["writeback_blocks"] += len(todo)
        return ev if self.stream is not None else None

    # ------------------------------------------------------------ pool -> P
    def prefetch(self, req) -> int:
        t0 = time.perf_counter()
        pool = self.eng.pool
        usable = max(0, (len(req.prompt) - 1) // self.bs)  # the last prompt token is always computed
        hashes = chain_block_hashes(req.prompt[: usable * self.bs], self.bs, full_only=True)
        n_local = pool.peek(hashes)
        todo = []
        for h in hashes[n_local:]:
            s = self.slot_of.get(h)
            if s is None and self.durable is not None and self.durable.is_durable(h):
                s = self._take_slot()  # back from L2 (a validated record) into an L1 slot
                if s is not None and self.durable.read_into(h, self.l1[s].data_ptr()):
                    self.slot_of[h] = s
                    self.stats["l2_promoted_blocks"] += 1
                elif s is not None:
                    self.free_slots.append(s)
                    s = None
            if s is None or not pool.can_alloc(1):
                break
            page = pool.alloc(1)[0]
            self.slot_of.move_to_end(h)
            todo.append((h, s, page))
        if not todo:
            return 0
        if self.stream is None:
            for h, s, page in todo:
                self._page(page).copy_(self.l1[s])
        else:
            dev = self.eng.arena.device
            self.stream.wait_event(torch.cuda.current_stream(dev).record_event())
            with torch.cuda.stream(self.stream):
                for h, s, page in todo:
                    self._page(page).copy_(self.l1[s], non_blocking=True)
            torch.cuda.current_stream(dev).wait_stream(self.stream)
        for h, s, page in todo:
            pool.register(page, h)
            pool.release([page])  # resident and cached; admission takes its own reference
        self.stats["promoted_blocks"] += len(todo)
        self.stats["promote_ms"] += (time.perf_counter() - t0) * 1000
        return len(todo)

    # ------------------------------------------------------------ fences (pages are the engine's)
    def _reserve_mirror_pages(self, plan: PreparePlan) -> None:
        """Give each page of generated tokens this step writes a reserved L1 slot, so the QKV
        epilogue stores its K/V into host memory as well."""
        reqs = self.eng.requests
        for io in plan.write_set:
            req = reqs.get(io.req_id)
            if req is None or io.token_end <= io.token_start:
                continue
            first = -(-len(req.prompt) // self.bs)  # the first page that holds generated tokens only
            for pg in range(max(first, io.token_start // self.bs), (io.token_end - 1) // self.bs + 1):
                mb = req.mirror_blocks
                if mb is None:
                    mb = req.mirror_blocks = {}
                if pg in mb:
                    continue
                slot = self._take_slot()
                if slot is None:
                    self.stats["mirror_slots_short"] += 1  # the page is copied at finish instead
                    break
                mb[pg] = slot
                self.reserved.add(slot)

    def prepare_step(self, plan: PreparePlan) -> ReadyHandle:
        if self.mirror_arena is not None and self.eng.runner.mirror_arena is self.mirror_arena:
            self._reserve_mirror_pages(plan)
        self._ready = plan.step_id
        stats = {io.req_id: StepStats() for io in plan.write_set}
        return ReadyHandle(plan.step_id, stats, list(plan.read_set), list(plan.write_set), {}, {})

    def done(self, step_id: int) -> None:
        self._ready = None

    def commit_write_extent(self, req_id: str, token_end: int) -> None:
        return None

    @property
    def l1_len(self) -> int:
        return len(self.slot_of)
