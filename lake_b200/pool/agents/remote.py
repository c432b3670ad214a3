"""Storage agent of a worker whose KV pool runs in other processes.

The pool is two gRPC services: the control plane (ControlPlaneService: the
location view, registration, references, request barriers) and a kv-pool byte
service (TcpDataService: opaque block bytes). This agent is what puts them on
the serving path:

  * admission (``prefetch``, called by the scheduler right before its prefix
    lookup): LookupPrefix for the prompt's full blocks; blocks the pool holds
    beyond the engine's own HBM prefix cache are pinned (REQUEST +1), pulled
    with GetBlocks, copied into fresh L0 pages (host -> device), registered in
    the engine's prefix cache and unpinned (REQUEST -1). The scheduler then
    counts them as cached tokens and prefills only the rest. A pull that would
    overrun the pull budget stops there: the remaining blocks are recomputed.
  * finish (D -> pool write-back, held until the step that may still touch the
    request closes): the request's full pages (prompt and decode-extended
    tokens) that the pool does not hold yet are copied device -> host, stored
    with PutBlocks, registered with RegisterBlocks (an L2 copy on the pool node
    plus this node's L0 copy, so the router can score this node for affinity),
    cycled through a WRITEBACK reference so the authority may evict them when
    idle, and the request's barrier is completed with RequestBarrier.

Block bytes are the page-first arena's page: every layer's K and V of 16
tokens, one contiguous span (``docs/block_format.md``).

Reference parity: python/lake/engine/agents/grpc_skeleton.py:49-253 (lookup,
GetBlocks on hits, PutBlocks + RegisterBlocks on misses, RequestBarrier on
finish; there the bytes are placeholders) and python/lake/runtime/worker.py:65-86
(the worker wires the agent from its control-plane and kv-pool addresses).
"""
from __future__ import annotations

import logging
import time

import torch

from ...api import proto
from ...engine.block_pool import chain_block_hashes
from ..types import FinishRequest, PoolError, PoolErrorCode, PreparePlan, PrefixHint, ReadyHandle, StepStats
from .fences import StepFences

LOG = logging.getLogger("lake_b200.pool.remote")
pb = proto.messages()

TARGET, REQUEST, WRITEBACK = 1, 1, 3
L0, L2 = 1, 3
BATCH_BYTES = 32 << 20  # bytes per GetBlocks / PutBlocks call


class RemotePoolAgent(StepFences):
    def __init__(self, engine, cp, kv, node_id: str = "worker-0", model_id: str | None = None,
                 revision: str = "", pool_node_id: str = "kv-pool", pull_budget_ms: float = 0.0,
                 writeback: bool = True, timeout_s: float = 10.0, clock=time.perf_counter):
        super().__init__()
        self.eng = engine
        self.cp, self.kv = cp, kv
        self.node_id = node_id
        self.model_id = model_id or engine.cfg.name
        self.revision = revision
        self.pool_node_id = pool_node_id
        self.pull_budget_ms = pull_budget_ms
        self.writeback = writeback
        self.timeout_s = timeout_s
        self.clock = clock
        self.bs = engine.ec.block_size
        self.page_bytes = engine.arena[0].numel() * engine.arena.element_size()
        cuda = engine.arena.is_cuda
        self.stream = torch.cuda.Stream(engine.arena.device) if cuda else None
        self._pin = cuda
        self.stats = {"lookups": 0, "pulled_blocks": 0, "pulled_bytes": 0, "pull_ms": 0.0, "budget_stops": 0,
                      "missing_bytes": 0, "written_blocks": 0, "written_bytes": 0, "writeback_ms": 0.0,
                      "register_rejects": 0, "rpc_errors": 0}
        self._rpc(cp.RegisterModel, pb.RegisterModelRequest(model=pb.ModelDescriptor(
            model_id=self.model_id, revision=revision, num_layers=engine.cfg.n_layers,
            block_spec=pb.BlockSpec(block_tokens=self.bs, bytes_per_block=self.page_bytes), hash_algo=1)),
            "RegisterModel", check=False)

    # ------------------------------------------------------------ helpers
    def _rpc(self, fn, req, what: str, check: bool = True):
        try:
            resp = fn(req, timeout=self.timeout_s)
        except Exception as e:  # grpc.RpcError and transport failures
            self.stats["rpc_errors"] += 1
            raise PoolError(PoolErrorCode.DOWNSTREAM, f"{what}: {e}") from e
        if check and hasattr(resp, "ok") and not resp.ok:
            raise PoolError(PoolErrorCode.DOWNSTREAM, f"{what}: {resp.err}")
        return resp

    def _ids(self, hashes):
        return [pb.KVBlockID(model_id=self.model_id, block_hash=h, pool_kind=TARGET, scope="public",
                             revision=self.revision) for h in hashes]

    def _page(self, page: int) -> torch.Tensor:
        return self.eng.arena[page].view(-1).view(torch.uint8)

    def _refs(self, ids, kind: int, delta: int) -> None:
        deltas = [pb.RefDelta(id=i, kind=kind, delta=delta, node_id=self.node_id) for i in ids]
        self._rpc(self.cp.ReportRef, iter(deltas), "ReportRef")

    def _lookup(self, hashes):
        self.stats["lookups"] += 1
        return self._rpc(self.cp.LookupPrefix, pb.LookupPrefixRequest(
            model_id=self.model_id, prefix_hashes=hashes, requester_node_id=self.node_id, revision=self.revision,
            pool_kind=TARGET), "LookupPrefix")

    # ------------------------------------------------------------ probe
    def probe_prefix(self, req) -> PrefixHint:
        hashes = chain_block_hashes(req.prompt, self.bs, full_only=True)
        if not hashes:
            return PrefixHint()
        local = self.eng.pool.peek(hashes)
        hit = max(int(self._lookup(hashes).hit_length), local)
        return PrefixHint(computed_tokens=min(hit * self.bs, len(req.prompt)), reused_blocks=hit,
                          local_hit=local > 0, prebuilt=local * self.bs >= len(req.prompt))

    # ------------------------------------------------------------ pool -> P (admission)
    def prefetch(self, req) -> int:
        usable = max(0, (len(req.prompt) - 1) // self.bs)  # the last prompt token is always computed
        hashes = chain_block_hashes(req.prompt[: usable * self.bs], self.bs, full_only=True)
        if not hashes:
            return 0
        pool = self.eng.pool
        n_local = pool.peek(hashes)
        if n_local == len(hashes):
            return 0
        t0 = self.clock()
        hit = int(self._lookup(hashes).hit_length)
        want = hashes[n_local:hit]
        if not want:
            return 0
        ids = self._ids(want)
        self._refs(ids, REQUEST, +1)  # pinned in the pool while the bytes are in transit
        pulled = 0
        try:
            per_call = max(1, BATCH_BYTES // self.page_bytes)
            for i in range(0, len(ids), per_call):
                if self.pull_budget_ms > 0 and (self.clock() - t0) * 1000 > self.pull_budget_ms:
                    self.stats["budget_stops"] += 1
                    break
                got = self._rpc(self.kv.GetBlocks, pb.GetBlocksRequest(ids=ids[i:i + per_call]), "GetBlocks")
                n = self._adopt(want[i:i + per_call], got.blocks)
                pulled += n
                if n < len(ids[i:i + per_call]):
                    break  # a block the pool lists but no longer stores: recompute from here
        finally:
            self._refs(ids, REQUEST, -1)
        self.stats["pulled_blocks"] += pulled
        self.stats["pulled_bytes"] += pulled * self.page_bytes
        self.stats["pull_ms"] += (self.clock() - t0) * 1000
        return pulled

    def _adopt(self, hashes, blocks) -> int:
        """Copy the leading blocks whose bytes arrived in order into fresh L0 pages."""
        pool = self.eng.pool
        todo = []
        for h, blk in zip(hashes, blocks):
            if bytes(blk.id.block_hash) != h or len(blk.data) != self.page_bytes:
                self.stats["missing_bytes"] += 1
                break
            if not pool.can_alloc(1):
                break
            todo.append((h, pool.alloc(1)[0], blk.data))
        if not todo:
            return 0
        host = torch.empty(len(todo), self.page_bytes, dtype=torch.uint8, pin_memory=self._pin)
        for j, (_, _, data) in enumerate(todo):
            host[j].copy_(torch.frombuffer(bytearray(data), dtype=torch.uint8))
        if self.stream is None:
            for j, (_, page, _) in enumerate(todo):
                self._page(page).copy_(host[j])
        else:
            dev = self.eng.arena.device
            self.stream.wait_event(torch.cuda.current_stream(dev).record_event())
            with torch.cuda.stream(self.stream):
                for j, (_, page, _) in enumerate(todo):
                    self._page(page).copy_(host[j], non_blocking=True)
            torch.cuda.current_stream(dev).wait_stream(self.stream)
            self.stream.synchronize()  # the pinned staging buffer is released on return
        for h, page, _ in todo:
            pool.register(page, h)
            pool.release([page])  # resident and cached; admission takes its own reference
        return len(todo)

    # ------------------------------------------------------------ fences
    def prepare_step(self, plan: PreparePlan) -> ReadyHandle:
        self._check_closed()
        reqs = self.eng.requests
        stats = {}
        for io in plan.write_set:
            r = reqs.get(io.req_id)
            st = StepStats()
            if r is not None:
                if io.token_start == r.num_cached and r.num_cached:
                    st.reused_blocks = r.num_cached // self.bs
                if io.token_start < len(r.prompt):
                    st.prefill_blocks = (min(io.token_end, len(r.prompt)) - io.token_start + self.bs - 1) // self.bs
            stats[io.req_id] = st
        self._open(plan.step_id)
        return ReadyHandle(plan.step_id, stats, list(plan.read_set), list(plan.write_set), {}, {})

    # ------------------------------------------------------------ D -> pool (finish)
    def _finish(self, finish: FinishRequest) -> None:
        req = self.eng.requests.get(finish.req_id)
        if req is not None and self.writeback:
            self.write_back(req)
        self._rpc(self.cp.RequestBarrier, pb.RequestBarrierRequest(request_id=finish.req_id, node_id=self.node_id),
                  "RequestBarrier")

    def write_back(self, req) -> int:
        t0 = self.clock()
        toks = req.all_tokens
        n_full = min(req.num_computed, len(toks)) // self.bs
        hashes = chain_block_hashes(toks[: n_full * self.bs], self.bs, full_only=True)
        pages = req.meta.get("final_block_ids") or req.block_ids
        n = min(len(hashes), len(pages))
        if n == 0:
            return 0
        hashes, pages = hashes[:n], pages[:n]
        have = int(self._lookup(hashes).hit_length)
        new = list(range(have, n))
        if not new:
            return 0
        # device -> host: the producing step has completed (finishes run after the compute fence)
        host = torch.empty(len(new), self.page_bytes, dtype=torch.uint8, pin_memory=self._pin)
        for j, i in enumerate(new):
            host[j].copy_(self._page(pages[i]), non_blocking=self._pin)
        if self._pin:
            torch.cuda.current_stream(self.eng.arena.device).synchronize()
        ids = self._ids([hashes[i] for i in new])
        per_call = max(1, BATCH_BYTES // self.page_bytes)
        for k in range(0, len(new), per_call):
            blocks = [pb.OpaqueBlock(id=ids[j], data=host[j].numpy().tobytes())
                      for j in range(k, min(len(new), k + per_call))]
            self._rpc(self.kv.PutBlocks, pb.PutBlocksRequest(node_id=self.pool_node_id, blocks=blocks), "PutBlocks")
        metas = [pb.BlockMeta(id=ids[j], block_kind=1, locations=[
            pb.Location(tier=L2, node_id=self.pool_node_id, segment_id=0, offset=0),
            pb.Location(tier=L0, node_id=self.node_id, segment_id=1, offset=int(pages[i]) * self.page_bytes)])
            for j, i in enumerate(new)]
        ack = self._rpc(self.cp.RegisterBlocks, pb.RegisterBlocksRequest(
            node_id=self.node_id, blocks=metas, prefix_hashes=hashes), "RegisterBlocks", check=False)
        if not ack.ok:  # quota / pool backpressure: the bytes stay unreferenced in the byte store
            self.stats["register_rejects"] += 1
            LOG.info("write-back of %s refused: %s", req.rid, ack.err)
            return 0
        self._refs(ids, WRITEBACK, +1)
        self._refs(ids, WRITEBACK, -1)  # idle: evictable by the pool's quota planning
        self.stats["written_blocks"] += len(new)
        self.stats["written_bytes"] += len(new) * self.page_bytes
        self.stats["writeback_ms"] += (self.clock() - t0) * 1000
        return len(new)


def connect(engine, cp_addr: str, kv_addr: str, **kw) -> RemotePoolAgent:
    """A RemotePoolAgent over fresh channels to the control plane and the kv-pool byte service."""
    import grpc

    cp = proto.Stub(grpc.insecure_channel(cp_addr, options=proto.message_options()), "ControlPlaneService")
    kv = proto.Stub(grpc.insecure_channel(kv_addr, options=proto.message_options()), "TcpDataService")
    return RemotePoolAgent(engine, cp, kv, **kw)
