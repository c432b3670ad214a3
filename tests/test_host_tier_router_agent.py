"""Tier engine, router core and PutEnd protocol (C++) on CPU.

Fault injection follows the reference's test doubles (failing control-plane
ports in rust/storage-agent/src/putend.rs tests) but with ports written in
Python against the C++ interface."""
import ctypes
import time

import pytest
import torch

from lake_b200 import _host as H

BB = 4096  # block bytes for tests


def pinned(n_slots):
    t = torch.zeros(n_slots * BB, dtype=torch.uint8)
    return t, t.data_ptr()


def engine(tmp_path, caps=(4, 4, 3)):
    buf, ptr = pinned(caps[1])
    e = H.TierEngine(H.TierCaps(*caps), BB, ptr, str(tmp_path / "l2"), str(tmp_path / "l3"), "m")
    e._buf = buf  # keep the host buffer alive
    return e


def blk(i):
    return bytes([i % 251]) * BB


def h(i):
    return H.sha256(bytes([i]))


# ------------------------------------------------------------------ tier
def test_put_durable_l2_cap_demotes_to_l3_and_reads_back(tmp_path):
    e = engine(tmp_path, caps=(4, 4, 2))
    for i in range(3):
        tier, fx = e.put_durable_bytes(h(i), blk(i))
    assert e.l2_len() == 2
    assert fx.l2_demoted_to_l3 == [h(0)]
    assert e.l3_present(h(0)) and not e.is_l2_durable(h(0))
    assert e.read_bytes(h(0)) == blk(0)
    assert e.read_bytes(h(2)) == blk(2)
    assert e.probe(h(0)) == H.AccessKind.L3_HIT
    assert e.probe(h(9)) == H.AccessKind.MISS


def test_durable_records_detect_torn_foreign_and_flipped_bytes(tmp_path):
    """An L2 slot or L3 object holds a header (magic, version, block hash, payload length,
    checksum) before the payload: a record whose bytes changed on disk reads as missing."""
    e = engine(tmp_path, caps=(4, 4, 2))
    e.put_durable_bytes(h(0), blk(0))
    e.put_durable_bytes(h(1), blk(1))
    assert e.read_bytes(h(0)) == blk(0) and e.corrupt_reads() == 0
    seg, off = e.l2_placement(h(0)).segment_id, e.l2_placement(h(0)).offset
    assert e.l2_placement(h(1)).offset == off + e.record_bytes()  # slots are header + payload
    path = tmp_path / "l2" / f"seg_{seg}.bin"
    raw = bytearray(path.read_bytes())
    raw[off + 64 + 100] ^= 0x10  # one flipped payload bit
    path.write_bytes(bytes(raw))
    assert e.read_bytes(h(0)) is None and e.corrupt_reads() == 1
    assert e.read_bytes(h(1)) == blk(1)  # the neighbouring slot is intact
    raw[off + 64 + 100] ^= 0x10
    raw[off + 24] ^= 0x01  # a header naming another block
    path.write_bytes(bytes(raw))
    assert e.read_bytes(h(0)) is None and e.corrupt_reads() == 2
    # L3: an object cut short (a torn write) is rejected too
    f = engine(tmp_path / "l3case", caps=(4, 4, 1))
    f.put_durable_bytes(h(3), blk(3))
    f.put_durable_bytes(h(4), blk(4))  # L2 cap 1: h(3) moves to L3
    assert f.l3_present(h(3)) and f.read_bytes(h(3)) == blk(3)
    obj = tmp_path / "l3case" / "l3" / "m" / h(3).hex()
    obj.write_bytes(obj.read_bytes()[: 64 + BB // 2])
    assert f.read_bytes(h(3)) is None and f.corrupt_reads() == 1


def test_pinned_l2_blocks_are_not_demoted(tmp_path):
    e = engine(tmp_path, caps=(4, 4, 1))
    e.put_durable_bytes(h(0), blk(0))
    e.pin(h(0))
    # the pinned block stays; the unpinned newcomer is demoted straight to L3
    tier, fx = e.put_durable_bytes(h(1), blk(1))
    assert tier == H.TierId.L3 and e.is_l2_durable(h(0)) and e.l3_present(h(1))
    e.pin(h(2))
    with pytest.raises(ValueError, match="pinned"):
        e.put_durable_bytes(h(2), blk(2))
    # two-phase: the failed put left no trace
    assert not e.is_l2_durable(h(2)) and e.is_l2_durable(h(0))
    e.unpin(h(2))
    e.unpin(h(0))
    with pytest.raises(ValueError):
        e.unpin(h(0))


def test_promote_l3_to_l0_through_l1_and_pressure_eviction(tmp_path):
    e = engine(tmp_path, caps=(2, 4, 8))
    pages = iter(range(100))
    for i in range(3):
        e.put_durable_bytes(h(i), blk(i))
    c0, ev, fx = e.promote_to_l0(h(0), lambda: next(pages))
    assert c0.to_device and c0.slot >= 0 and e.l0_page(h(0)) == c0.page
    # the staged L1 slot holds the block bytes (the caller copies it to the GPU page)
    slot_bytes = ctypes.string_at(e._buf.data_ptr() + c0.slot * BB, BB)
    assert slot_bytes == blk(0)
    e.promote_to_l0(h(1), lambda: next(pages))
    assert e.is_one_shot(h(1))
    # L0 full: the third promotion demotes a one-shot block
    c2, ev, fx = e.promote_to_l0(h(2), lambda: -1)
    assert len(ev) == 1 and not ev[0].to_device
    assert e.l0_len() == 2
    assert e.begin_promote(h(2)) == H.BeginPromote.ALREADY_L0
    assert e.begin_promote(h(7)) == H.BeginPromote.MISSING


def test_segment_arena_compact_and_relocate():
    a = H.SegmentArena(4096, 4)
    for i in range(4):
        a.alloc(h(i))
    a.free(h(1))
    assert a.has_holes(1)
    moves = a.compact(1)
    assert len(moves) == 1 and moves[0].dst.offset == 4096
    assert not a.has_holes(1) and a.dense_prefix_slots(1) == 3


def test_bandwidth_pool_window_and_pause():
    bw = H.BandwidthPool(1000, 1000)
    assert bw.try_consume(600, 0)
    assert not bw.try_consume(600, 10)
    assert bw.try_consume(600, 1000)  # new window
    bw.set_paused(True)
    assert not bw.try_consume(1, 5000)


def test_pipeline_tick_promotes_and_emits_events(tmp_path):
    e = engine(tmp_path, caps=(4, 4, 8))
    e.put_durable_bytes(h(0), blk(0))
    bw = H.BandwidthPool(1 << 30, 1000)
    p = H.TierPipeline(e, bw, "node-a")
    p.enqueue(H.Action(H.ActionKind.PROMOTE, h(0)))
    p.enqueue(H.Action(H.ActionKind.DEMOTE_L2, h(0)))
    pages = iter(range(10))
    n, events, copies = p.tick(8, 0, lambda: next(pages))
    assert n == 2
    assert any(ev.kind == H.LocKind.PRESENT and ev.tier == 1 for ev in events)
    assert any(ev.kind == H.LocKind.L3_PRESENT for ev in events)
    assert copies and copies[0].to_device


def test_writeback_batcher():
    w = H.WritebackBatcher(2)
    assert w.push(b"a") == []
    assert w.push(b"b") == [b"a", b"b"]
    w.push(b"c")
    assert w.drain() == [b"c"] and w.flushes() == 2


# ------------------------------------------------------------------ router
def test_select_exec_mode():
    R = H.Role
    assert H.select_exec_mode(H.PrefixHint(16, 1, 1, True), 32, R.HYBRID, 10) == H.ExecMode.D_DIRECT
    assert H.select_exec_mode(H.PrefixHint(16, 1, 0, False), 32, R.PREFILL, 0.5) == H.ExecMode.COLOCATED
    assert H.select_exec_mode(H.PrefixHint(), 32, R.DECODE, 10) == H.ExecMode.PD_DISAGG
    assert H.select_exec_mode(H.PrefixHint(), 32, R.HYBRID, 10) == H.ExecMode.COLOCATED


def test_mirror_snapshot_gap_dedupe_and_lookup():
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, 100))
    hs = [h(1), h(2)]
    a.register_blocks("n0", hs, [H.BlockMeta(H.KVBlockID("m", x), [H.Location(1, "n0")]) for x in hs])
    u1 = a.commit_pending()
    mirror = H.ViewMirror()
    assert mirror.apply(a.snapshot()) == 0
    assert mirror.apply(u1) == 0 and mirror.last_seq() == 1
    a.publish_location(H.KVBlockID("m", hs[1]), 1, "n1", 1, 0, True)
    a.commit_pending()
    a.publish_location(H.KVBlockID("m", hs[0]), 1, "n1", 1, 0, True)
    u3 = a.commit_pending()
    assert mirror.apply(u3) == 2  # gap: wants seq 2
    for u in a.replay_after(mirror.last_seq()):
        assert mirror.apply(u) == 0
    assert mirror.apply(u3) == 0  # duplicate ignored
    got = mirror.prefix_lookup("m", "", 1, hs, "n1")
    assert [b.local_hit for b in got] == [True, True]


def test_pick_node_affinity_guard_and_hrw():
    nodes = H.NodeRegistry(["w0", "w1", "w2"])
    key = b"anchor"
    cold = H.pick_node(nodes, None, "m", [], key, 8)
    best = max(["w0", "w1", "w2"], key=lambda n: (H.hrw_score(key, n), [-ord(c) for c in n]))
    assert cold == best
    mirror = H.ViewMirror()
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, 100))
    a.register_blocks("w2", [h(5)], [H.BlockMeta(H.KVBlockID("m", h(5)), [H.Location(1, "w2")])])
    mirror.apply(a.snapshot())
    assert H.pick_node(nodes, mirror, "m", [h(5)], key, 8) == "w2"
    for _ in range(8):
        nodes.inc_inflight("w2")
    assert H.pick_node(nodes, mirror, "m", [h(5)], key, 8) != "w2"


def test_pq_priority_preempt_backpressure_and_load():
    pq = H.PQScheduler(1, 0.2)
    t1, pre = pq.submit(0, "a")
    assert pq.start_eligible() == [t1] and pre is None
    t2, pre = pq.submit(0, "a")
    assert pre is None  # same priority does not preempt
    t3, pre = pq.submit(5, "a")
    assert pre == t1
    pq.finish(t1, preempted=True)  # requeued
    assert pq.start_eligible() == [t3]
    pq.finish(t3)
    assert pq.start_eligible() == [t1]  # FIFO among priority 0: t1 (requeued) keeps its seq
    pq.finish(t1)
    pq.set_backpressure("a")
    assert pq.start_eligible() == []
    time.sleep(0.25)
    assert pq.start_eligible() == [t2]
    snap = pq.load_snapshot("n0")
    assert snap.in_flight == 1 and snap.remaining_cap == 0
    assert pq.cancel(pq.submit(0, "b")[0])


def test_autoscaler_sustain_and_cooldown():
    s = H.Autoscaler(H.AutoscaleConfig(1, 3, 4, 0, 2, 10.0))
    assert s.evaluate(0, 5, 2, 1) == H.ScaleDecision.NONE
    assert s.evaluate(1, 5, 2, 1) == H.ScaleDecision.SCALE_OUT
    assert s.evaluate(2, 5, 2, 2) == H.ScaleDecision.NONE  # sustain reset
    assert s.evaluate(3, 5, 2, 2) == H.ScaleDecision.NONE  # cooldown
    assert s.evaluate(20, 0, 0, 2) == H.ScaleDecision.NONE
    assert s.evaluate(21, 0, 0, 2) == H.ScaleDecision.SCALE_IN


# ------------------------------------------------------------------ PutEnd
def _setup(tmp_path):
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, BB))
    e = engine(tmp_path, caps=(4, 4, 8))
    return a, e


def _session(n=2):
    s = H.PutEndSession("req-1", "n0", "m")
    hs = [h(i) for i in range(n)]
    for i, x in enumerate(hs):
        s.put_start(x, blk(i))
    return s, hs


def test_putend_happy_path_releases_refs(tmp_path):
    a, e = _setup(tmp_path)
    s, hs = _session()
    s.commit_through(H.AuthorityPort(a), e)
    assert a.barrier_completed("req-1")
    assert a.lookup_prefix("m", "", 0, hs, "").hit_length == 2
    assert a.refs_by_kind(H.KVBlockID("m", hs[0])) == (0, 0)
    assert e.pin_count(hs[0]) == 0 and e.is_l2_durable(hs[0])
    assert not s.writeback_open() and not s.register_hold_open()


class Delegate(H.ControlPlanePort):
    def __init__(self, a):
        super().__init__()
        self.inner = H.AuthorityPort(a)
        self.calls = []

    def admit_register_blocks(self, node, prefix, metas):
        self.calls.append("admit")
        self.inner.admit_register_blocks(node, prefix, metas)

    def register_blocks(self, node, prefix, metas):
        self.calls.append("register")
        self.inner.register_blocks(node, prefix, metas)

    def report_refs(self, deltas):
        self.calls.append(("refs", deltas[0].kind, deltas[0].delta))
        self.inner.report_refs(deltas)

    def request_barrier(self, rid, node):
        self.calls.append("barrier")
        self.inner.request_barrier(rid, node)

    def publish_location(self, id, tier, node, seg, off, present):
        self.inner.publish_location(id, tier, node, seg, off, present)

    def set_l3_present(self, id, present):
        self.inner.set_l3_present(id, present)


def test_putend_protocol_order(tmp_path):
    a, e = _setup(tmp_path)
    s, hs = _session()
    port = Delegate(a)
    s.commit_through(port, e)
    assert port.calls == ["admit", "register", ("refs", 1, 1), ("refs", 3, 1), "barrier", ("refs", 3, -1),
                          ("refs", 1, -1)]


def test_putend_register_failure_discards_and_unpins(tmp_path):
    a, e = _setup(tmp_path)

    class FailRegister(Delegate):
        def register_blocks(self, node, prefix, metas):
            raise RuntimeError("register down")

    s, hs = _session()
    with pytest.raises(RuntimeError, match="register down"):
        s.commit_through(FailRegister(a), e)
    assert e.pin_count(hs[0]) == 0 and not s.all_durable()
    assert a.lookup_prefix("m", "", 0, hs, "").hit_length == 0


def test_putend_barrier_failure_keeps_hold_then_retry_succeeds(tmp_path):
    a, e = _setup(tmp_path)

    class BarrierOnceFail(Delegate):
        failed = False

        def request_barrier(self, rid, node):
            if not BarrierOnceFail.failed:
                BarrierOnceFail.failed = True
                raise RuntimeError("barrier timeout")
            super().request_barrier(rid, node)

    s, hs = _session()
    port = BarrierOnceFail(a)
    with pytest.raises(RuntimeError, match="register-hold retained"):
        s.commit_through(port, e)
    assert s.register_hold_open() and not s.writeback_open()
    assert a.refs_by_kind(H.KVBlockID("m", hs[0])) == (1, 0)  # frozen by the hold
    s.commit_through(port, e)  # retry-safe
    assert a.refs_by_kind(H.KVBlockID("m", hs[0])) == (0, 0)


def test_putend_admit_rejection_writes_nothing(tmp_path):
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, BB, 1, H.Quota(BB, BB, False)))
    e = engine(tmp_path)
    s, hs = _session(2)
    with pytest.raises(RuntimeError, match="HARD_QUOTA"):
        s.commit_through(H.AuthorityPort(a), e)
    assert e.l2_len() == 0


def test_apply_location_events_skips_unknown(tmp_path):
    a, e = _setup(tmp_path)
    s, hs = _session(1)
    s.commit_through(H.AuthorityPort(a), e)
    evs = [H.LocationEvent(H.LocKind.PRESENT, hs[0], 1, "n0", 0, 5), H.LocationEvent(H.LocKind.PRESENT, h(99), 1, "n0")]
    assert H.apply_location_events(H.AuthorityPort(a), "m", "", 1, evs) == 1
    r = a.lookup_prefix("m", "", 0, hs, "n0")
    assert r.all_local_hit


def test_backpressure_memory_ttl():
    b = H.BackpressureMemory(0.1)
    assert b.fresh() is None
    s = H.BackpressureSignal()
    s.reason = "HARD_QUOTA"
    b.record(s)
    assert b.fresh().reason == "HARD_QUOTA"
    time.sleep(0.15)
    assert b.fresh() is None
