"""ControlPlaneService view subscription under the scenarios the reference's control-plane
handler tests pin (rust/controlplane/src/lib.rs:1756-2050): a snapshot then an anchor on
connect, no zero-seq anchor when nothing was issued yet (a receiver resets on seq 0), a live
increment after RegisterBlocks, a restore on a fresh process, a restore broadcast to a live
subscriber, a resume that replays the missed updates, and resume points too old or ahead of
what this process issued falling back to a snapshot; and the handlers' sinks
(lib.rs:3150-3800): automatic defrag off by default, gated by its fragmentation threshold and by
PauseBackground, delivered outside the authority lock; hit reports warming a block with its
ancestors once (hysteresis), RegisterBlocks pre-placing a chain on its HRW home, and a join
warming the new node with the hot blocks. The servicer is called directly; its stream, a
generator, is drained by a reader thread."""
import queue
import threading

from lake_b200.api import proto
from lake_b200.engine.block_pool import chain_block_hashes
from lake_b200.services.controlplane import ControlPlane

pb = proto.messages()
M = "m"
REGISTERED, INVALIDATED, MOVED = 0, 1, 2


class _Ctx:
    def __init__(self):
        self.active = True

    def is_active(self):
        return self.active


def _cp():
    cp = ControlPlane()
    cp.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
        model_id=M, num_layers=2, block_spec=pb.BlockSpec(block_tokens=16, bytes_per_block=1000), hash_algo=1)), None)
    return cp


def _hashes(n, seed=0):
    return chain_block_hashes(list(range(seed, seed + 16 * n)), 16)


def _kid(k):
    from lake_b200 import _host as H

    return H.KVBlockID(k.model_id, bytes(k.block_hash), int(k.pool_kind), k.revision)


def _register(cp, hashes, node="n0"):
    ack = cp.RegisterBlocks(pb.RegisterBlocksRequest(node_id=node, prefix_hashes=hashes, blocks=[
        pb.BlockMeta(id=pb.KVBlockID(model_id=M, block_hash=h, pool_kind=1), block_kind=1,
                     locations=[pb.Location(tier=3, node_id=node, segment_id=1, offset=i * 1000)])
        for i, h in enumerate(hashes)]), None)
    assert ack.ok, ack.err


class _Sub:
    """A SubscribeView stream drained by a daemon reader thread into a queue."""

    def __init__(self, cp, resume=0):
        self.ctx = _Ctx()
        self.q = queue.Queue()
        gen = cp.SubscribeView(pb.SubscribeRequest(subscriber_id="r0", resume_from_seq=resume), self.ctx)
        threading.Thread(target=lambda: [self.q.put(u) for u in gen], daemon=True).start()

    def expect(self, timeout=5.0):
        return self.q.get(timeout=timeout)

    def expect_nothing(self, wait=0.3):
        try:
            u = self.q.get(timeout=wait)
        except queue.Empty:
            return
        raise AssertionError(f"unexpected update seq={u.seq} ({len(u.events)} events)")

    def close(self):
        self.ctx.active = False


def test_connect_gets_a_snapshot_then_the_anchor():
    cp = _cp()
    _register(cp, _hashes(2))
    s = _Sub(cp)
    snap = s.expect()
    assert snap.seq == 0 and [e.kind for e in snap.events] == [REGISTERED, REGISTERED]
    anchor = s.expect()
    assert anchor.seq == 1 and not anchor.events
    s.expect_nothing()
    s.close()
    cp.stop()


def test_no_zero_anchor_before_anything_was_issued_then_a_live_increment():
    cp = _cp()
    s = _Sub(cp)
    snap = s.expect()
    assert snap.seq == 0 and not snap.events
    s.expect_nothing()  # a seq-0 anchor would make a receiver reset again
    _register(cp, _hashes(1))
    live = s.expect()
    assert live.seq == 1 and [e.kind for e in live.events] == [REGISTERED]
    s.expect_nothing()
    s.close()
    cp.stop()


def _donor_snapshot(hashes):
    donor = _cp()
    _register(donor, hashes)
    resp = donor.SaveCheckpoint(pb.SaveCheckpointRequest(), None)
    donor.stop()
    assert resp.ok
    return resp.snapshot


def test_a_restore_on_a_fresh_process_sends_the_snapshot_and_no_zero_anchor():
    snap = _donor_snapshot(_hashes(2))
    cp = ControlPlane()
    assert cp.RestoreCheckpoint(pb.RestoreCheckpointRequest(snapshot=snap), None).ok
    assert cp.auth.last_seq() == 0
    s = _Sub(cp)
    first = s.expect()
    assert first.seq == 0 and len(first.events) == 2
    s.expect_nothing()
    s.close()
    cp.stop()


def test_a_live_subscriber_receives_the_restored_snapshot():
    cp = _cp()
    old = _hashes(1, seed=1000)
    _register(cp, old)
    s = _Sub(cp)
    assert s.expect().seq == 0 and s.expect().seq == 1
    new = _hashes(1, seed=2000)
    assert cp.RestoreCheckpoint(pb.RestoreCheckpointRequest(snapshot=_donor_snapshot(new)), None).ok
    reset = s.expect()
    assert reset.seq == 0 and [bytes(e.id.block_hash) for e in reset.events] == new  # the restored state
    anchor = s.expect()
    assert anchor.seq >= 1 and not anchor.events
    s.expect_nothing()
    s.close()
    cp.stop()


def test_a_resume_replays_the_missed_updates():
    cp = _cp()
    hs = _hashes(1)
    _register(cp, hs)  # seq 1
    kid = pb.KVBlockID(model_id=M, block_hash=hs[0], pool_kind=1)
    with cp.lock:  # while the subscriber is away: an L0 copy appears (seq 2), then the block goes (seq 3)
        cp.auth.publish_location(_kid(kid), 1, "n0", 0, 0, True)
        cp._commit()  # noqa: SLF001
    assert cp.DiscardBlocks(pb.DiscardBlocksRequest(ids=[kid]), None).ok
    s = _Sub(cp, resume=1)
    r1 = s.expect()
    assert r1.seq == 2 and r1.events[0].kind == MOVED and len(r1.events[0].locations) == 2  # every location
    r2 = s.expect()
    assert r2.seq == 3 and r2.events[0].kind == INVALIDATED
    s.expect_nothing()
    s.close()
    cp.stop()


def test_a_resume_point_older_than_the_replay_window_gets_a_snapshot():
    cp = _cp()
    cp.auth.set_view_log_cap(2)
    for i in range(4):  # seq 1..4; the window keeps 3 and 4
        _register(cp, _hashes(1, seed=100 * i + 1))
    s = _Sub(cp, resume=1)
    first = s.expect()
    assert first.seq == 0 and len(first.events) == 4
    assert s.expect().seq == 4
    s.expect_nothing()
    s.close()
    cp.stop()


def test_a_resume_point_ahead_of_what_was_issued_gets_a_snapshot():
    cp = _cp()
    _register(cp, _hashes(1))  # this process issued seq 1
    s = _Sub(cp, resume=100)  # a sequence from an earlier process
    first = s.expect()
    assert first.seq == 0 and len(first.events) == 1
    anchor = s.expect()
    assert anchor.seq == 1 and not anchor.events
    s.expect_nothing()
    s.close()
    cp.stop()


# ------------------------------------------------------------------ handler sinks (lib.rs:3150-3800)
SLOT = 4096


def _register_at(cp, placements, node="n0"):
    """placements: [(name, segment, offset)] registered as one chain with L2 copies there."""
    hs = [_name_hash(n) for n, _, _ in placements]
    ack = cp.RegisterBlocks(pb.RegisterBlocksRequest(node_id=node, prefix_hashes=hs, blocks=[
        pb.BlockMeta(id=pb.KVBlockID(model_id=M, block_hash=h, pool_kind=1), block_kind=1,
                     locations=[pb.Location(tier=3, node_id=node, segment_id=seg, offset=off)])
        for h, (_, seg, off) in zip(hs, placements)]), None)
    assert ack.ok, ack.err
    return hs


def _name_hash(name):
    from lake_b200 import _host as H

    return H.sha256(name.encode())


def _defrag_cp(threshold, sink):
    cp = ControlPlane(defrag_sink=sink, auto_defrag_threshold=threshold, defrag_slot_bytes=SLOT)
    cp.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
        model_id=M, num_layers=2, block_spec=pb.BlockSpec(block_tokens=16, bytes_per_block=1000), hash_algo=1)), None)
    return cp


FRAGMENTED = [("a", 1, 0), ("b", 1, 2 * SLOT)]  # a hole at slot 1


def test_auto_defrag_is_off_by_default():
    calls = []
    cp = _defrag_cp(0.0, lambda m, r, pk, moves: calls.append(len(moves)))
    _register_at(cp, FRAGMENTED)
    assert calls == []
    cp.stop()


def test_auto_defrag_below_its_threshold_does_not_fire():
    calls = []
    cp = _defrag_cp(0.5, lambda m, r, pk, moves: calls.append(len(moves)))
    _register_at(cp, FRAGMENTED + [("c", 2, 0), ("d", 2, SLOT), ("e", 3, 0), ("f", 3, SLOT)])
    assert calls == []
    assert abs(cp.auth.l2_fragmentation_ratio(M, "", 1, SLOT) - 1 / 3) < 1e-9  # one of three segments has a hole
    cp.stop()


def test_auto_defrag_at_its_threshold_fires_once_with_a_plan():
    calls = []
    cp = _defrag_cp(0.5, lambda m, r, pk, moves: calls.append(len(moves)))
    _register_at(cp, FRAGMENTED)
    assert len(calls) == 1 and calls[0] > 0
    cp.stop()


def test_auto_defrag_sink_runs_outside_the_authority_lock():
    got = []

    def try_lock():
        ok = cp.lock.acquire(timeout=2)
        if ok:
            cp.lock.release()
        got.append(ok)

    def sink(m, r, pk, moves):  # another thread must be able to take the lock meanwhile
        t = threading.Thread(target=try_lock)
        t.start()
        t.join(5)

    cp = _defrag_cp(0.5, sink)
    _register_at(cp, FRAGMENTED)
    assert got == [True]
    cp.stop()


def test_auto_defrag_is_skipped_while_background_work_is_paused():
    calls = []
    cp = _defrag_cp(0.5, lambda m, r, pk, moves: calls.append(len(moves)))
    assert cp.PauseBackground(pb.PauseBackgroundRequest(paused=True), None).ok
    _register_at(cp, FRAGMENTED)
    assert calls == []
    cp.stop()


def _warm_cp(calls):
    cp = ControlPlane(warmup_sink=lambda node, ids: calls.append((node, [bytes(i.block_hash) for i in ids])))
    cp.RegisterModel(pb.RegisterModelRequest(model=pb.ModelDescriptor(
        model_id=M, num_layers=2, block_spec=pb.BlockSpec(block_tokens=16, bytes_per_block=1000), hash_algo=1)), None)
    return cp


def _hits(cp, node, hashes):
    assert cp.ReportHits(pb.ReportHitsRequest(node_id=node, ids=[
        pb.KVBlockID(model_id=M, block_hash=h, pool_kind=1) for h in hashes]), None).ok


def test_report_hits_warm_the_block_and_its_ancestors_once():
    calls = []
    cp = _warm_cp(calls)
    a, c = _register_at(cp, [("a", 1, 0), ("c", 1, SLOT)])
    calls.clear()
    for _ in range(2):
        _hits(cp, "n5", [c])
    assert calls == [("n5", [a, c])]  # the ancestor travels with it, root first
    for _ in range(2):
        _hits(cp, "n5", [c])
    assert calls == [("n5", [a, c])]  # hysteresis: not sent again
    cp.stop()


def test_register_preplaces_the_chain_on_its_hrw_home():
    calls = []
    cp = _warm_cp(calls)
    assert cp.JoinShardNode(pb.JoinShardNodeRequest(node_id="n0", vnode_count=16), None).ok
    calls.clear()
    a, b = _register_at(cp, [("a", 1, 0), ("b", 1, SLOT)])
    assert calls == [("n0", [a, b])]  # the only ready node is the home of the whole chain
    cp.stop()


def test_a_join_warms_the_new_node_with_the_hot_blocks():
    calls = []
    cp = _warm_cp(calls)
    (hot,) = _register_at(cp, [("hot", 1, 0)])
    _hits(cp, "router-0", [hot])
    calls.clear()
    assert cp.JoinShardNode(pb.JoinShardNodeRequest(node_id="n1", vnode_count=16), None).ok
    assert calls == [("n1", [hot])]
    cp.stop()
