"""ControlPlaneService: the gRPC face of the C++ block authority.

All 24 RPCs of lake.proto's ControlPlaneService are served over one
``lake_b200._host.Authority`` under a lock. Writers commit the authority's
pending view events as one ViewUpdate and broadcast it to every SubscribeView
stream.

SubscribeView protocol: the subscriber is attached to the broadcast first, then
the initial sequence is taken under the lock - the full snapshot (seq 0) plus
an empty anchor update carrying the last issued seq, or, for
resume_from_seq > 0, the replay of the missed updates (falling back to the
snapshot when the bounded replay log, ``LAKE_VIEW_LOG_CAP`` updates (default 1024), no
longer covers it, or when the resume point is ahead of what this process issued). Live updates with
seq <= the last delivered one are dropped (snapshot/broadcast overlap); a seq-0
update (a restored checkpoint) resets the watermark and is always forwarded.
A subscriber whose queue overflows is resynchronised with a fresh snapshot.

Lease (bidi): MOUNT/KEEPALIVE grant a lease of ``lease_ttl_ms`` for the node,
UNMOUNT releases it. ``reap_expired_leases()`` (run by the background thread
when ``start_reaper`` is called) reconciles nodes whose lease ran out as dead:
their locations are stripped and their refs cleared.

Reference parity: rust/controlplane/src/lib.rs:318-1090 (handlers),
checkpoint.rs:13-40 (store), view.rs (snapshot/replay/dedup), reconcile.rs.
"""
from __future__ import annotations

import logging
import os
import queue
import tempfile
import threading
import time

from .. import _host as H
from ..api import proto
from . import convert as C

LOG = logging.getLogger("lake_b200.controlplane")
pb = proto.messages()
DEFAULT_WARMUP_K = 256
SUBSCRIBER_QUEUE = 64


def ack(ok=True, err="", bp=None):
    return pb.Ack(ok=ok, err=err, backpressure=C.bp_out(bp))


# ------------------------------------------------------------------ checkpoint stores
class MemoryCheckpointStore:
    def __init__(self):
        self._snap = None

    def save(self, snap_pb) -> None:
        self._snap = snap_pb.SerializeToString()

    def load(self):
        return None if self._snap is None else pb.CheckpointSnapshot.FromString(self._snap)


class FileCheckpointStore:
    """One serialized CheckpointSnapshot per file, replaced atomically (write + fsync + rename)."""

    def __init__(self, path: str):
        self.path = path
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)

    def save(self, snap_pb) -> None:
        d = os.path.dirname(os.path.abspath(self.path))
        fd, tmp = tempfile.mkstemp(dir=d, prefix=".ckpt-")
        with os.fdopen(fd, "wb") as f:
            f.write(snap_pb.SerializeToString())
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, self.path)

    def load(self):
        if not os.path.exists(self.path):
            return None
        with open(self.path, "rb") as f:
            return pb.CheckpointSnapshot.FromString(f.read())


# ------------------------------------------------------------------ view broadcast
class _Subscriber:
    def __init__(self):
        self.q: "queue.Queue" = queue.Queue(maxsize=SUBSCRIBER_QUEUE)
        self.lagged = False


class ViewBroadcast:
    def __init__(self):
        self._subs: set[_Subscriber] = set()
        self._lock = threading.Lock()

    def attach(self) -> _Subscriber:
        s = _Subscriber()
        with self._lock:
            self._subs.add(s)
        return s

    def detach(self, s: _Subscriber) -> None:
        with self._lock:
            self._subs.discard(s)

    def send(self, update_pb) -> None:
        with self._lock:
            subs = list(self._subs)
        for s in subs:
            try:
                s.q.put_nowait(update_pb)
            except queue.Full:
                s.lagged = True

    @property
    def subscriber_count(self) -> int:
        with self._lock:
            return len(self._subs)


# ------------------------------------------------------------------ service
class ControlPlane:
    def __init__(self, authority: "H.Authority | None" = None, checkpoints=None, warmup_sink=None,
                 defrag_sink=None, lease_ttl_ms: int = 10_000, auto_defrag_threshold: float = 0.0,
                 defrag_slot_bytes: int = 0, clock=time.monotonic):
        self.auth = authority or H.Authority()
        self.lock = threading.RLock()
        self.view = ViewBroadcast()
        self.checkpoints = checkpoints or MemoryCheckpointStore()
        self.checkpoint_seq = 0
        self.warmup_sink = warmup_sink or (lambda node, ids: LOG.info("warmup %s: %d blocks", node, len(ids)))
        self.defrag_sink = defrag_sink or (lambda m, r, pk, moves: LOG.info("defrag %s: %d moves", m, len(moves)))
        self.lease_ttl_ms = lease_ttl_ms
        self.leases: dict[str, float] = {}  # node -> expiry (clock seconds)
        self.clock = clock
        self.auto_defrag_threshold = auto_defrag_threshold
        self.defrag_slot_bytes = defrag_slot_bytes
        self._reaper_stop = threading.Event()

    # ---------------------------------------------------------------- helpers
    def _commit(self) -> None:
        """Commit pending view events (under self.lock) and broadcast them."""
        if self.auth.pending_events() == 0:
            return
        self.view.send(C.update_out(self.auth.commit_pending()))

    def _snapshot_with_anchor(self):
        last = self.auth.last_seq()
        ups = [C.update_out(self.auth.snapshot())]
        if last > 0:
            ups.append(pb.ViewUpdate(seq=last))
        return ups, last

    # ---------------------------------------------------------------- view
    def SubscribeView(self, request, context):
        sub = self.view.attach()
        try:
            with self.lock:
                if request.resume_from_seq == 0:
                    initial, last = self._snapshot_with_anchor()
                else:
                    ups = self.auth.replay_after(request.resume_from_seq)
                    if ups is None:
                        initial, last = self._snapshot_with_anchor()
                    else:
                        initial = [C.update_out(u) for u in ups]
                        last = initial[-1].seq if initial else request.resume_from_seq
            yield from initial
            while context is None or context.is_active():
                if sub.lagged:
                    with self.lock:
                        while not sub.q.empty():
                            sub.q.get_nowait()
                        sub.lagged = False
                        ups, last = self._snapshot_with_anchor()
                    yield from ups
                    continue
                try:
                    u = sub.q.get(timeout=0.1)
                except queue.Empty:
                    if self._reaper_stop.is_set():
                        return
                    continue
                if u.seq == 0:  # restore broadcast: reset semantics, always forwarded
                    last = 0
                    yield u
                    continue
                if u.seq <= last:
                    continue
                last = u.seq
                yield u
        finally:
            self.view.detach(sub)

    # ---------------------------------------------------------------- lookups
    def LookupPrefix(self, request, context):
        with self.lock:
            r = self.auth.lookup_prefix(request.model_id, request.revision, int(request.pool_kind),
                                        [bytes(h) for h in request.prefix_hashes], request.requester_node_id)
        return pb.LookupPrefixResponse(
            blocks=[pb.ReusableBlock(id=C.kid_out(b.id), meta=C.meta_out(b.meta), local_hit=b.local_hit)
                    for b in r.blocks], hit_length=r.hit_length, all_local_hit=r.all_local_hit)

    def Locate(self, request, context):
        with self.lock:
            metas = self.auth.locate([C.kid_in(k) for k in request.ids])
        return pb.LocateResponse(blocks=[C.meta_out(m) for m in metas])

    # ---------------------------------------------------------------- registration
    @staticmethod
    def _admit_keys(request):
        ids = [b.id for b in request.blocks if b.HasField("id")]
        if not ids:
            raise ValueError("AdmitRegisterBlocks: no blocks")
        m, r, pk = ids[0].model_id, ids[0].revision, int(ids[0].pool_kind)
        for i in ids[1:]:
            if (i.model_id, i.revision, int(i.pool_kind)) != (m, r, pk):
                raise ValueError("AdmitRegisterBlocks: blocks span namespaces")
        return m, r, pk, [bytes(i.block_hash) for i in ids]

    def AdmitRegisterBlocks(self, request, context):
        try:
            m, r, pk, hashes = self._admit_keys(request)
            with self.lock:
                res = self.auth.preflight_register(m, r, pk, hashes)
        except Exception as e:
            return ack(False, str(e))
        if res.accepted:
            return ack()
        bp = res.backpressure
        return ack(False, f"AdmitRegisterBlocks: admission rejected reason={bp.reason} deficit={bp.deficit_bytes}",
                   bp)

    def RegisterBlocks(self, request, context):
        metas = [C.meta_in(b) for b in request.blocks]
        prefix = [bytes(h) for h in request.prefix_hashes]
        ns = next(((b.id.model_id, b.id.revision, int(b.id.pool_kind)) for b in request.blocks if b.HasField("id")),
                  None)
        preplace = defrag = None
        with self.lock:
            try:
                res = self.auth.register_blocks(request.node_id, prefix, metas)
            except Exception as e:
                self._commit()
                return ack(False, str(e))
            if res.accepted and ns is not None:
                preplace = self.auth.preplace_on_register(ns[0], ns[1], ns[2], prefix)
                defrag = self._plan_auto_defrag(*ns)
            self._commit()
        # sinks run outside the lock: they may call back into this service
        if preplace is not None and preplace.ids:
            self.warmup_sink(preplace.node_id, list(preplace.ids))
        if defrag:
            self.defrag_sink(ns[0], ns[1], ns[2], defrag)
        if res.accepted:
            return ack()
        bp = res.backpressure
        return ack(False, f"RegisterBlocks: admission rejected reason={bp.reason} deficit={bp.deficit_bytes}", bp)

    def _plan_auto_defrag(self, m, r, pk):
        if self.auto_defrag_threshold <= 0 or self.auth.background_paused():
            return None
        slot = self.defrag_slot_bytes
        if self.auth.l2_fragmentation_ratio(m, r, pk, slot) < self.auto_defrag_threshold:
            return None
        moves = self.auth.plan_defrag(m, r, pk, 3, slot)
        return moves or None

    def ReportRef(self, request_iterator, context):
        deltas = [C.ref_in(d) for d in request_iterator]
        with self.lock:
            try:
                self.auth.report_refs(deltas)
            except Exception as e:  # all-or-nothing: the ledger is left unchanged
                LOG.warning("report_ref rejected: %s", e)
                return ack(False, str(e))
            self._commit()
        return ack()

    def RequestBarrier(self, request, context):
        with self.lock:
            try:
                self.auth.complete_barrier(request.request_id, request.node_id)
            except Exception as e:
                return ack(False, str(e))
        return ack()

    # ---------------------------------------------------------------- leases
    def Lease(self, request_iterator, context):
        for hb in request_iterator:
            now = self.clock()
            with self.lock:
                if hb.op == 1:  # UNMOUNT
                    self.leases.pop(hb.node_id, None)
                    yield pb.LeaseAck(granted=False, ttl_ms=0)
                    continue
                if hb.op == 2 and hb.node_id not in self.leases:  # KEEPALIVE after expiry: must re-mount
                    yield pb.LeaseAck(granted=False, ttl_ms=0)
                    continue
                self.leases[hb.node_id] = now + self.lease_ttl_ms / 1000.0
            yield pb.LeaseAck(granted=True, ttl_ms=self.lease_ttl_ms)

    def reap_expired_leases(self) -> list[str]:
        now = self.clock()
        dead = []
        with self.lock:
            for node, exp in list(self.leases.items()):
                if exp < now:
                    del self.leases[node]
                    self.auth.reconcile_dead_node(node)
                    dead.append(node)
            if dead:
                self._commit()
        for n in dead:
            LOG.warning("lease of %s expired: node reconciled as dead", n)
        return dead

    def start_reaper(self, period_s: float = 1.0) -> threading.Thread:
        def loop():
            while not self._reaper_stop.wait(period_s):
                self.reap_expired_leases()

        t = threading.Thread(target=loop, name="lakeb-lease-reaper", daemon=True)
        t.start()
        return t

    def stop(self) -> None:
        self._reaper_stop.set()

    # ---------------------------------------------------------------- models / quota
    def RegisterModel(self, request, context):
        if not request.HasField("model"):
            return ack(False, "RegisterModel: model required")
        with self.lock:
            try:
                self.auth.register_model(C.model_in(request.model))
            except Exception as e:
                return ack(False, str(e))
        return ack()

    def DeregisterModel(self, request, context):
        with self.lock:
            try:
                self.auth.deregister_model(request.model_id, request.revision)
            except Exception as e:
                self._commit()
                return ack(False, str(e))
            self._commit()
        return ack()

    def SetModelQuota(self, request, context):
        if not request.HasField("quota"):
            return ack(False, "SetModelQuota: quota required")
        with self.lock:
            try:
                self.auth.set_quota(request.model_id, request.revision, C.quota_in(request.quota))
            except Exception as e:
                return ack(False, str(e))
        return ack()

    def GetModelQuota(self, request, context):
        with self.lock:
            try:
                q = self.auth.get_quota(request.model_id, request.revision)
                used = self.auth.used_bytes(request.model_id, request.revision)
            except Exception as e:
                return pb.GetModelQuotaResponse(ok=False, err=str(e))
        borrowed = max(0, used - q.soft_bytes) if q.soft_bytes > 0 else 0
        resp = pb.GetModelQuotaResponse(quota=C.quota_out(q), used_bytes=used, borrowed_bytes=borrowed, ok=True)
        if q.hard_bytes > 0 and used > q.hard_bytes:
            resp.backpressure.CopyFrom(pb.BackpressureSignal(
                model_id=request.model_id, revision=request.revision, used_bytes=used, soft_bytes=q.soft_bytes,
                hard_bytes=q.hard_bytes, deficit_bytes=used - q.hard_bytes, reason="HARD_QUOTA"))
        return resp

    # ---------------------------------------------------------------- reconcile / gc
    def ReconcileOrphans(self, request, context):
        discarded, stripped, cleared = [], [], 0
        with self.lock:
            try:
                if request.reports:
                    self.auth.report_orphans([C.orphan_in(r) for r in request.reports])
                discarded += self.auth.sweep_orphans(int(request.orphan_ttl_ms))
                if request.dead_node_id:
                    n, ids = self.auth.reconcile_dead_node(request.dead_node_id)
                    cleared += n
                    stripped += ids
                if request.gc_model_id and request.gc_cold_limit:
                    gone, cold = self.auth.gc_cold(request.gc_model_id, request.gc_revision,
                                                   int(request.gc_pool_kind), int(request.gc_cold_limit))
                    discarded += gone
                    stripped += cold
            except Exception as e:
                self._commit()
                return pb.ReconcileOrphansResponse(ok=False, err=str(e))
            self._commit()
        return pb.ReconcileOrphansResponse(discarded=[C.kid_out(k) for k in discarded],
                                           cold_stripped=[C.kid_out(k) for k in stripped], refs_cleared=cleared,
                                           ok=True)

    def DiscardBlocks(self, request, context):
        with self.lock:
            try:
                self.auth.discard_blocks([C.kid_in(k) for k in request.ids])
            except Exception as e:
                self._commit()
                return ack(False, str(e))
            self._commit()
        return ack()

    # ---------------------------------------------------------------- checkpoint
    def SaveCheckpoint(self, request, context):
        with self.lock:
            self.checkpoint_seq += 1
            snap = self.auth.export_snapshot()
            snap.seq = self.checkpoint_seq
            snap_pb = C.snapshot_out(snap)
        try:
            self.checkpoints.save(snap_pb)
        except Exception as e:
            return pb.SaveCheckpointResponse(ok=False, err=str(e))
        return pb.SaveCheckpointResponse(snapshot=snap_pb, ok=True)

    def RestoreCheckpoint(self, request, context):
        if request.HasField("snapshot"):
            snap_pb = request.snapshot
        else:
            try:
                snap_pb = self.checkpoints.load()
            except Exception as e:
                return ack(False, str(e))
            if snap_pb is None:
                return ack(False, "RestoreCheckpoint: store empty")
        with self.lock:
            try:
                self.auth.import_snapshot(C.snapshot_in(snap_pb))
            except Exception as e:
                return ack(False, str(e))
            ups, _ = self._snapshot_with_anchor()
            for u in ups:
                self.view.send(u)
        return ack()

    # ---------------------------------------------------------------- defrag / background
    def TriggerDefrag(self, request, context):
        mode = int(request.mode) or 3
        with self.lock:
            try:
                moves = self.auth.plan_defrag(request.model_id, request.revision, int(request.pool_kind), mode,
                                              int(request.slot_bytes))
            except Exception as e:
                return pb.TriggerDefragResponse(ok=False, err=str(e))
        return pb.TriggerDefragResponse(moves=[C.move_out(m) for m in moves], planned_moves=len(moves), ok=True)

    def PauseBackground(self, request, context):
        with self.lock:
            self.auth.set_background_paused(bool(request.paused))
        return ack()

    # ---------------------------------------------------------------- shard ring
    def GetShardMap(self, request, context):
        with self.lock:
            return pb.GetShardMapResponse(map=C.shard_map_out(self.auth.shard_map()), ok=True)

    def JoinShardNode(self, request, context):
        with self.lock:
            try:
                migs, _warm = self.auth.join_shard_node(request.node_id, int(request.vnode_count))
            except Exception as e:
                return pb.JoinShardNodeResponse(ok=False, err=str(e))
            smap = self.auth.shard_map()
            plan = self.auth.warmup_plan(request.node_id, DEFAULT_WARMUP_K)
        if plan:
            self.warmup_sink(request.node_id, list(plan))
        return pb.JoinShardNodeResponse(map=C.shard_map_out(smap), migrations=[C.migration_out(m) for m in migs],
                                        migration_count=len(migs), ok=True)

    def DrainShardNode(self, request, context):
        with self.lock:
            try:
                migs, push = self.auth.drain_shard_node(request.node_id)
            except Exception as e:
                return pb.DrainShardNodeResponse(ok=False, err=str(e))
            smap = self.auth.shard_map()
        return pb.DrainShardNodeResponse(map=C.shard_map_out(smap), migrations=[C.migration_out(m) for m in migs],
                                         push_l2=[C.kid_out(k) for k in push], migration_count=len(migs), ok=True)

    def RemoveShardNode(self, request, context):
        with self.lock:
            try:
                self.auth.remove_shard_node(request.node_id)
            except Exception as e:
                return ack(False, str(e))
        return ack()

    def ReportHits(self, request, context):
        with self.lock:
            plans = self.auth.report_hits(request.node_id, [C.kid_in(k) for k in request.ids])
        for p in plans:
            if p.ids:
                self.warmup_sink(p.node_id, list(p.ids))
        return ack()


def serve(bind: str = "0.0.0.0:50051", cp: ControlPlane | None = None, max_workers: int = 16):
    import grpc
    from concurrent import futures

    cp = cp or ControlPlane(checkpoints=FileCheckpointStore(os.environ["LAKE_CP_CHECKPOINT"])
                            if os.environ.get("LAKE_CP_CHECKPOINT") else None)
    if os.environ.get("LAKE_VIEW_LOG_CAP"):  # updates kept for resuming subscribers
        cp.auth.set_view_log_cap(int(os.environ["LAKE_VIEW_LOG_CAP"]))
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers), options=proto.message_options())
    proto.add_service(server, "ControlPlaneService", cp)
    port = server.add_insecure_port(bind)
    server.start()
    cp.start_reaper()
    return server, cp, port


def main() -> None:
    logging.basicConfig(level=os.environ.get("LAKE_LOG", "INFO"))
    server, _, port = serve(os.environ.get("LAKE_CP_ADDR", "0.0.0.0:50051"))
    LOG.info("controlplane listening on port %d", port)
    server.wait_for_termination()


if __name__ == "__main__":
    main()
