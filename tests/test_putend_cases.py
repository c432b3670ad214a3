"""PutEnd commit protocol (C++ agent over the C++ authority and a real L0-L3 tier engine) under
the scenarios the reference's storage-agent tests pin (rust/storage-agent/src/putend.rs:556-1706):
where a committed block settles (L2 only, L2 cap demotions mirrored to the control plane), which
refs a failing control-plane port leaves behind and how a retry or a dead-node reconcile clears
them, idempotent location-event application, and the arena coordinates RegisterBlocks carries.
The failing ports are Python subclasses of the C++ port interface."""
import pytest

from lake_b200 import _host as H

BB = 4096
L0, L1, L2, L3 = 1, 2, 3, 4
REQUEST, WRITEBACK = 1, 3


def _engine(tmp_path, caps):
    import torch

    buf = torch.zeros(caps[1] * BB, dtype=torch.uint8)
    e = H.TierEngine(H.TierCaps(*caps), BB, buf.data_ptr(), str(tmp_path / "l2"), str(tmp_path / "l3"), "m")
    e._buf = buf
    return e


def _auth():
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, BB))
    return a


def _h(name: str) -> bytes:
    return H.sha256(name.encode())


def _blk(name: str) -> bytes:
    return (name.encode() * BB)[:BB]


def _session(rid, names):
    s = H.PutEndSession(rid, "n0", "m")
    for n in names:
        s.put_start(_h(n), _blk(n))
    return s


def _meta(a, name):
    return a.locate([H.KVBlockID("m", _h(name))])[0]


def _has_l0_on(a, name, node="n0"):
    return any(l.tier == L0 and l.node_id == node for l in _meta(a, name).locations)


class Port(H.ControlPlanePort):
    """Pass-through to an in-process authority; subclasses fail chosen calls."""

    def __init__(self, a):
        super().__init__()
        self.inner = H.AuthorityPort(a)

    def admit_register_blocks(self, node, prefix, metas):
        self.inner.admit_register_blocks(node, prefix, metas)

    def register_blocks(self, node, prefix, metas):
        self.inner.register_blocks(node, prefix, metas)

    def report_refs(self, deltas):
        self.inner.report_refs(deltas)

    def request_barrier(self, rid, node):
        self.inner.request_barrier(rid, node)

    def publish_location(self, id, tier, node, seg, off, present):
        self.inner.publish_location(id, tier, node, seg, off, present)

    def set_l3_present(self, id, present):
        self.inner.set_l3_present(id, present)


def test_commit_settles_on_l2_only_and_becomes_evictable(tmp_path):
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))
    _session("r1", ["h0"]).commit_through(H.AuthorityPort(a), e)
    assert e.is_l2_durable(_h("h0")) and not e.l3_present(_h("h0"))  # PutEnd writes no L3
    assert a.barrier_completed("r1")
    m = _meta(a, "h0")
    assert any(l.tier == L2 for l in m.locations) or m.l3_present  # published => settled
    assert e.has_durable_backing(_h("h0"))
    # a later request's hold and release leave the block at zero refs: evictable
    d = H.RefDelta(H.KVBlockID("m", _h("h0")), REQUEST, 1, "n0")
    a.report_refs([d])
    d.delta = -1
    a.report_refs([d])
    assert a.evict_n("m", "", 1, 1) == 1


def test_promotion_published_as_l0_location(tmp_path):
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))
    _session("r2", ["p"]).commit_through(H.AuthorityPort(a), e)
    pages = iter(range(8))
    e.promote_to_l0(_h("p"), lambda: next(pages))
    H.AuthorityPort(a).publish_location(H.KVBlockID("m", _h("p")), L0, "n0", 0, 0, True)
    assert e.l0_page(_h("p")) >= 0
    assert _has_l0_on(a, "p")


def test_l2_cap_demotion_of_an_earlier_block_is_mirrored_on_the_control_plane(tmp_path):
    a, e = _auth(), _engine(tmp_path, (4, 8, 1))
    _session("r-a", ["x"]).commit_through(H.AuthorityPort(a), e)
    assert e.is_l2_durable(_h("x")) and not e.l3_present(_h("x"))
    _session("r-b", ["y"]).commit_through(H.AuthorityPort(a), e)
    assert not e.is_l2_durable(_h("x")) and e.l3_present(_h("x"))  # exactly one of L2 / L3
    assert e.is_l2_durable(_h("y")) and not e.l3_present(_h("y"))
    mx = _meta(a, "x")
    assert mx.l3_present and not any(l.tier == L2 and l.node_id == "n0" for l in mx.locations)


def test_multi_block_commit_over_a_one_slot_l2(tmp_path):
    a, e = _auth(), _engine(tmp_path, (4, 8, 1))
    s = _session("r-mb", ["x", "y"])
    s.commit_through(H.AuthorityPort(a), e)
    assert not e.is_l2_durable(_h("x")) and e.l3_present(_h("x"))
    assert e.is_l2_durable(_h("y")) and not e.l3_present(_h("y"))
    assert e.l2_len() == 1
    assert e.pin_count(_h("x")) == 0 and e.pin_count(_h("y")) == 0
    assert _meta(a, "x").l3_present and any(l.tier == L2 for l in _meta(a, "y").locations)
    assert a.lookup_prefix("m", "", 1, [_h("x"), _h("y")], "").hit_length == 2


def test_barrier_error_with_failed_writeback_rollback_keeps_both_refs(tmp_path):
    """Barrier fails and so does the WRITEBACK -1 rollback: the error names both, the
    register-hold and the writeback ref both stay (the block cannot be evicted)."""
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))

    class FailingRollback(Port):
        def report_refs(self, deltas):
            if any(d.delta < 0 for d in deltas):
                raise RuntimeError("rollback unavailable")
            super().report_refs(deltas)

        def request_barrier(self, rid, node):
            raise RuntimeError("barrier unavailable")

    s = _session("r-rollback", ["h0"])
    with pytest.raises(RuntimeError) as ei:
        s.commit_through(FailingRollback(a), e)
    msg = str(ei.value)
    assert "barrier unavailable" in msg and "writeback rollback failed" in msg
    assert a.refs_by_kind(H.KVBlockID("m", _h("h0"))) == (1, 1)
    assert a.evict_n("m", "", 1, 1) == 0
    assert s.writeback_open() and s.register_hold_open()
    assert e.pin_count(_h("h0")) == 0


def test_writeback_release_failure_after_barrier_keeps_the_phantom_ref_until_reconcile(tmp_path):
    """Barrier succeeds, WRITEBACK -1 fails: the session says the writeback is still open, the
    register-hold is released, the phantom ref freezes the block until the node is reconciled."""
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))

    class MinusOneFails(Port):
        def report_refs(self, deltas):
            if any(d.delta < 0 and d.kind == WRITEBACK for d in deltas):
                raise RuntimeError("writeback -1 unavailable")
            super().report_refs(deltas)

    s = _session("r-m1", ["h0"])
    with pytest.raises(RuntimeError, match="WRITEBACK -1 failed"):
        s.commit_through(MinusOneFails(a), e)
    assert s.writeback_open() and not s.register_hold_open()
    assert a.refs_by_kind(H.KVBlockID("m", _h("h0"))) == (0, 1)
    assert a.evict_n("m", "", 1, 1) == 0
    a.reconcile_dead_node("n0")  # node-level reconcile clears the phantom
    assert a.refs_by_kind(H.KVBlockID("m", _h("h0"))) == (0, 0)


def test_writeback_release_failure_then_retry_converges(tmp_path):
    """The retry does not stack a second WRITEBACK +1: its -1 closes the phantom and the block
    ends evictable."""
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))

    class MinusOneOnce(Port):
        failed = False

        def report_refs(self, deltas):
            if not MinusOneOnce.failed and any(d.delta < 0 and d.kind == WRITEBACK for d in deltas):
                MinusOneOnce.failed = True
                raise RuntimeError("writeback -1 unavailable")
            super().report_refs(deltas)

    port = MinusOneOnce(a)
    s = _session("r-m1retry", ["h0"])
    with pytest.raises(RuntimeError, match="WRITEBACK -1 failed"):
        s.commit_through(port, e)
    assert a.refs_by_kind(H.KVBlockID("m", _h("h0"))) == (0, 1)
    s.commit_through(port, e)
    assert a.refs_by_kind(H.KVBlockID("m", _h("h0"))) == (0, 0)
    assert not s.writeback_open() and not s.register_hold_open()
    assert a.evict_n("m", "", 1, 1) == 1


def test_location_events_continue_past_a_failure_and_retry_idempotently(tmp_path):
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))
    for n in ("a", "fail", "b"):
        _session("r-" + n, [n]).commit_through(H.AuthorityPort(a), e)

    class TransientFail(Port):
        armed = True

        def publish_location(self, id, tier, node, seg, off, present):
            if TransientFail.armed and id.block_hash == _h("fail"):
                TransientFail.armed = False
                raise RuntimeError("transient")
            super().publish_location(id, tier, node, seg, off, present)

    port = TransientFail(a)
    evs = [H.LocationEvent(H.LocKind.PRESENT, _h(n), L0, "n0") for n in ("a", "fail", "b")]
    assert H.apply_location_events(port, "m", "", 1, evs) == 2  # the failing event did not stop the batch
    assert _has_l0_on(a, "a") and not _has_l0_on(a, "fail") and _has_l0_on(a, "b")
    assert H.apply_location_events(port, "m", "", 1, evs) == 3  # retry lands it; re-publishing is a refresh
    for n in ("a", "fail", "b"):
        assert sum(1 for l in _meta(a, n).locations if l.tier == L0 and l.node_id == "n0") == 1


def test_pipeline_promotion_events_move_the_single_l0_location(tmp_path):
    """With one L0 page, promoting b through the tier pipeline evicts a; applying the tick's
    events leaves the control plane with b in L0 and a no longer a local L0 hit."""
    a, e = _auth(), _engine(tmp_path, (1, 8, 8))
    for n in ("a", "b"):
        _session("r-" + n, [n]).commit_through(H.AuthorityPort(a), e)
    pipe = H.TierPipeline(e, H.BandwidthPool(1 << 30, 1000), "n0")
    pages = iter(range(16))
    pipe.enqueue(H.Action(H.ActionKind.PROMOTE, _h("a")))
    n, events, _ = pipe.tick(1, 0, lambda: next(pages))
    assert n == 1
    H.apply_location_events(H.AuthorityPort(a), "m", "", 1, events)
    assert _has_l0_on(a, "a")
    pipe.enqueue(H.Action(H.ActionKind.PROMOTE, _h("b")))
    n, events, _ = pipe.tick(1, 1, lambda: next(pages))
    assert n == 1
    H.apply_location_events(H.AuthorityPort(a), "m", "", 1, events)
    assert _has_l0_on(a, "b") and not _has_l0_on(a, "a")
    assert not a.lookup_prefix("m", "", 1, [_h("a")], "n0").all_local_hit


def test_register_request_carries_each_blocks_arena_slot(tmp_path):
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))
    s = _session("r-place", ["a", "b"])
    s.flush_durable(e)
    pa, pb = e.l2_placement(_h("a")), e.l2_placement(_h("b"))
    assert (pa.segment_id, pa.offset) != (pb.segment_id, pb.offset)
    coords = {}
    for m in s.metas(e):
        loc = [l for l in m.locations if l.tier == L2][0]
        coords[m.id.block_hash] = (loc.segment_id, loc.offset)
    assert coords[_h("a")] == (pa.segment_id, pa.offset) and coords[_h("b")] == (pb.segment_id, pb.offset)
    s.commit_through(H.AuthorityPort(a), e)
    la = [l for l in _meta(a, "a").locations if l.tier == L2][0]
    assert (la.segment_id, la.offset) == (pa.segment_id, pa.offset)


def test_a_session_names_the_storage_node_for_l2_and_the_committing_node_for_the_rest(tmp_path):
    """Engines sharing a pool node commit as themselves (refs, hold, barrier) while the L2
    locations name the pool node whose tiers hold the bytes."""
    a, e = _auth(), _engine(tmp_path, (4, 4, 8))
    seen = []

    class Rec(Port):
        def request_barrier(self, rid, node):
            seen.append(("barrier", node))
            super().request_barrier(rid, node)

        def report_refs(self, deltas):
            seen.extend(("ref", d.node_id) for d in deltas)
            super().report_refs(deltas)

    s = H.PutEndSession("r-shared", "eng-0", "m", "", "pool-0")
    s.put_start(_h("x"), _blk("x"))
    s.commit_through(Rec(a), e)
    assert [(l.tier, l.node_id) for l in _meta(a, "x").locations if l.tier == L2] == [(L2, "pool-0")]
    assert seen and all(node == "eng-0" for _, node in seen)
