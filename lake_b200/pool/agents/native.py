"""Production in-process storage agent of one compute node.

It ties three layers together:
  * L0 = the engine's HBM page pool (engine.block_pool.BlockPool) and arena,
  * L1 / L2 / L3 = the C++ tier engine (pinned host slots, NVMe segment files,
    object directory), and
  * the pool's location authority (C++, in process or behind gRPC via a port).

Data paths
  * D -> pool (writeback): when a request finishes, its full pages that the
    pool does not hold yet are copied device -> pinned host (one
    cudaMemcpyAsync per page on a side stream), committed durably to L2 with
    the PutEnd protocol (admit, flush, register, refs, barrier) and published
    in the authority. Pages stay resident in L0 as prefix cache.
  * pool -> prefill (D->P reuse): when a request arrives, prompt pages that are
    missing from L0 but present in L1/L2/L3 are promoted: L2/L3 bytes are read
    into an L1 slot by the tier engine, then copied host -> device into a fresh
    L0 page that is registered in the engine's prefix cache, so the scheduler's
    admission reuses them instead of recomputing.

Reference parity: the agent contract of python/lake/engine/agent.py:15-41, the
PutEnd protocol of rust/storage-agent/src/putend.rs:193-382 and the tier
promotion path of rust/tiered-store/src/engine.rs:495-606 (which move bytes
between in-memory maps); here bytes move between HBM, pinned DRAM and files.
"""
from __future__ import annotations

import os
import tempfile
import time

import torch

from ... import _host as H
from ...engine.block_pool import chain_block_hashes
from ..types import FinishRequest, PoolError, PoolErrorCode, PreparePlan, PrefixHint, ReadyHandle, StepStats
from .fences import StepFences

L0, L1, L2 = 1, 2, 3


def make_pool_node(model_id: str, page_bytes: int, l0_blocks: int, l1_blocks: int = 64, l2_blocks: int = 256,
                   storage_dir: str | None = None, pinned: bool = False):
    """A KV pool node (tier engine + its L1 slab) for NativeAgent(shared_tiers=...)."""
    root = storage_dir or tempfile.mkdtemp(prefix="lakeb_pool_")
    l1 = torch.zeros(l1_blocks * page_bytes, dtype=torch.uint8, pin_memory=pinned)
    tiers = H.TierEngine(H.TierCaps(l0_blocks, l1_blocks, l2_blocks), page_bytes, l1.data_ptr(),
                         os.path.join(root, "l2"), os.path.join(root, "l3"), model_id)
    return tiers, l1


class NativeAgent(StepFences):
    def __init__(self, engine, node_id: str = "node-0", model_id: str | None = None, revision: str = "",
                 authority: "H.Authority | None" = None, port=None, l1_blocks: int = 64, l2_blocks: int = 256,
                 storage_dir: str | None = None, writeback: str = "all", shared_tiers=None,
                 storage_node_id: str | None = None):
        super().__init__()
        self.eng = engine
        self.node_id = node_id
        # the node whose tiers hold the written-back blocks (their L2 locations): this engine's
        # node, or the pool node whose tiers several engines share (shared_tiers)
        self.storage_node_id = storage_node_id or node_id
        self.model_id = model_id or engine.cfg.name
        self.revision = revision
        self.bs = engine.ec.block_size
        self.page_bytes = engine.arena[0].numel() * engine.arena.element_size()
        self.authority = authority or H.Authority()
        self.port = port or H.AuthorityPort(self.authority)
        if authority is None or not self.authority.has_namespace(self.model_id, revision):
            self.authority.register_model(H.ModelDescriptor(self.model_id, revision, engine.cfg.n_layers, self.bs,
                                                            self.page_bytes))
        pin = engine.arena.is_cuda
        if shared_tiers is not None:
            # a pool node several engines use (its L1 slab and tier engine): what one engine wrote
            # back, another promotes
            self.tiers, self.l1 = shared_tiers
        else:
            root = storage_dir or tempfile.mkdtemp(prefix="lakeb_tiers_")
            self.l1 = torch.zeros(l1_blocks * self.page_bytes, dtype=torch.uint8, pin_memory=pin)
            self.tiers = H.TierEngine(H.TierCaps(engine.pool.num_blocks, l1_blocks, l2_blocks), self.page_bytes,
                                      self.l1.data_ptr(), os.path.join(root, "l2"), os.path.join(root, "l3"),
                                      self.model_id)
        self.stream = torch.cuda.Stream(engine.arena.device) if engine.arena.is_cuda else None
        self.writeback = writeback
        self.written: set[bytes] = set()
        self.stats = {"writeback_blocks": 0, "promoted_blocks": 0, "writeback_ms": 0.0, "promote_ms": 0.0}
        self._staging = torch.zeros(self.page_bytes, dtype=torch.uint8, pin_memory=pin)

    # ------------------------------------------------------------ helpers
    def _page_view(self, page: int) -> torch.Tensor:
        return self.eng.arena[page].view(-1).view(torch.uint8)

    def _ids(self, hashes):
        return [H.KVBlockID(self.model_id, h, 1, self.revision) for h in hashes]

    # ------------------------------------------------------------ probe / prefetch
    def probe_prefix(self, req) -> PrefixHint:
        hashes = chain_block_hashes(req.prompt, self.bs, full_only=True)
        r = self.authority.lookup_prefix(self.model_id, self.revision, 1, hashes, self.node_id)
        local = self.eng.pool.peek(hashes)
        hit = max(r.hit_length, local)
        return PrefixHint(computed_tokens=min(hit * self.bs, len(req.prompt)), reused_blocks=hit,
                          local_hit=local > 0, prebuilt=local * self.bs >= len(req.prompt))

    def prefetch(self, req) -> int:
        """Promote the request's prompt pages that live in L1/L2/L3 but not in L0."""
        t0 = time.perf_counter()
        hashes = chain_block_hashes(req.prompt, self.bs, full_only=True)[: max(0, (len(req.prompt) - 1) // self.bs)]
        pool = self.eng.pool
        n_local = pool.peek(hashes)
        promoted = 0
        for h in hashes[n_local:]:
            if self.tiers.local_tier(h) in (H.TierId.NONE, H.TierId.L0):
                break
            if not pool.can_alloc(1):
                break
            page = pool.alloc(1)[0]
            was_l2 = self.tiers.is_l2_durable(h)
            try:
                cp, evict, fx = self.tiers.promote_to_l0(h, lambda: page)
            except ValueError:
                pool.release([page])
                break
            self._mirror_l2_moves(h, was_l2, fx)
            if cp is not None:
                src = self.l1[cp.slot * self.page_bytes:(cp.slot + 1) * self.page_bytes]
                dst = self._page_view(page)
                if self.stream is not None:
                    with torch.cuda.stream(self.stream):
                        dst.copy_(src, non_blocking=True)
                else:
                    dst.copy_(src)
            pool.register(page, h)
            pool.release([page])  # resident and cached; admission takes its own reference
            self.tiers.drop_l0(h)  # L0 residency is the engine pool's; the tier engine keeps L1..L3
            promoted += 1
        if promoted:
            if self.stream is not None:
                self.stream.synchronize()
            self.authority.publish_location(self._ids([hashes[n_local]])[0], L0, self.node_id, 1, 0, True)
            self.authority.commit_pending()
        self.stats["promoted_blocks"] += promoted
        self.stats["promote_ms"] += (time.perf_counter() - t0) * 1000
        return promoted

    def _mirror_l2_moves(self, h: bytes, was_l2: bool, fx) -> None:
        """A promotion from L3 writes the block back to L2 (the node's recovery point for its
        working set) and may move the coldest L2 block to L3 under the cap; the control plane
        learns both, as the reference's engine mirrors them (rust/tiered-store/src/engine.rs:
        506-527)."""
        for v in fx.l2_demoted_to_l3:
            if v == h:
                continue
            vid = self._ids([v])[0]
            self.port.publish_location(vid, L2, self.storage_node_id, 0, 0, False)
            self.port.set_l3_present(vid, True)
        if not was_l2 and self.tiers.is_l2_durable(h):
            pl = self.tiers.l2_placement(h)
            self.port.publish_location(self._ids([h])[0], L2, self.storage_node_id, pl.segment_id, pl.offset, True)

    # ------------------------------------------------------------ fences
    def prepare_step(self, plan: PreparePlan) -> ReadyHandle:
        self._check_closed()
        reqs = self.eng.requests
        tables, slots, stats = {}, {}, {}
        for io in plan.write_set:
            r = reqs.get(io.req_id)
            if r is None:
                raise PoolError(PoolErrorCode.INVALID_ARG, f"unknown request {io.req_id}")
            need = (io.token_end + self.bs - 1) // self.bs
            if len(r.block_ids) < need:
                raise PoolError(PoolErrorCode.CAPACITY, f"{io.req_id}: {len(r.block_ids)} pages < {need}")
            tables[io.req_id] = list(r.block_ids)
            slots[io.req_id] = [r.block_ids[p // self.bs] * self.bs + p % self.bs
                                for p in range(io.token_start, io.token_end)]
            st = StepStats()
            if io.token_start == r.num_cached and r.num_cached:
                st.reused_blocks = r.num_cached // self.bs
            if io.token_start < len(r.prompt):
                st.prefill_blocks = (min(io.token_end, len(r.prompt)) - io.token_start + self.bs - 1) // self.bs
            stats[io.req_id] = st
        self._open(plan.step_id)
        return ReadyHandle(plan.step_id, stats, list(plan.read_set), list(plan.write_set), tables, slots)

    # ------------------------------------------------------------ writeback
    def _finish(self, finish: FinishRequest) -> None:
        req = self.eng.requests.get(finish.req_id)
        if req is None or self.writeback == "none":
            return
        self.write_back(req)

    def write_back(self, req) -> int:
        """Durably commit the request's full pages (prompt and decode-extended) to the pool."""
        t0 = time.perf_counter()
        toks = req.all_tokens
        n_full = min(req.num_computed, len(toks)) // self.bs
        hashes = chain_block_hashes(toks[: n_full * self.bs], self.bs, full_only=True)
        pages = req.meta.get("final_block_ids") or req.block_ids
        if not hashes or len(pages) < len(hashes):
            return 0
        todo = [(h, p) for h, p in zip(hashes, pages) if h not in self.written]
        if not todo:
            return 0
        sess = H.PutEndSession(req.rid, self.node_id, self.model_id, self.revision, self.storage_node_id)
        started = False
        for h, page in zip(hashes, pages):
            if h in self.written and not started:
                sess.add_prefix(h)  # already durable: only its place in the chain is needed
                continue
            started = True
            src = self._page_view(page)
            if src.is_cuda:
                self._staging.copy_(src, non_blocking=False)
                sess.put_start_ptr(h, self._staging.data_ptr(), self.page_bytes)
            else:
                sess.put_start(h, src.numpy().tobytes())
        sess.commit_through(self.port, self.tiers)
        self.written.update(hashes)
        self.stats["writeback_blocks"] += len(todo)
        self.stats["writeback_ms"] += (time.perf_counter() - t0) * 1000
        return len(todo)
