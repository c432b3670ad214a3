"""Tier engine (C++, real L1 slots, L2 segment files and L3 objects) under the scenarios the
reference's tiered-store engine tests pin (rust/tiered-store/src/engine.rs:700-1020): promote
and demote through L0/L1, L0 pressure reporting its collateral demotion, an L3 read miss that
lands back in L2, L3-only backing allowing an L0 demotion, pins blocking demotion, the L2 cap
moving a cold block to L3 (exactly one of L2 / L3), pinned blocks keeping their LRU position,
an all-pinned cap failure rolling back with the LRU order unchanged, hit counts, one-shot
admission and eviction order, and promote de-duplication; and the tier pipeline's cases
(pipeline.rs:315-445, storage-agent putend.rs:1706-1790): collateral L0 events, the bandwidth
window, requeue then drop of a failing action, compaction and a control-plane co-locate plan
held by PauseBackground. Storage failures are made on the host: a directory sits where the
engine wants to create a segment file or an L3 object."""
import pytest

from lake_b200 import _host as H

BB = 64


def _engine(tmp_path, caps):
    import torch

    buf = torch.zeros(caps[1] * BB, dtype=torch.uint8)
    e = H.TierEngine(H.TierCaps(*caps), BB, buf.data_ptr(), str(tmp_path / "l2"), str(tmp_path / "l3"), "m")
    e._buf = buf
    return e


def _h(name: str) -> bytes:
    return H.sha256(name.encode())


def _blk(name: str, tag: str = "") -> bytes:
    return ((tag + name).encode() * BB)[:BB]


def _put(e, name, tag=""):
    return e.put_durable_bytes(_h(name), _blk(name, tag))


def _pages(n=64):
    it = iter(range(n))
    return lambda: next(it)


def _l3_tmp_path(tmp_path, name):
    return tmp_path / "l3" / "m" / (_h(name).hex() + ".tmp")


# ------------------------------------------------------------------ promote / demote
def test_durable_promote_demote(tmp_path):
    e = _engine(tmp_path, (2, 4, 8))
    tier, fx = _put(e, "a")
    assert tier == H.TierId.L2 and not e.l3_present(_h("a"))  # PutEnd writes no L3 copy
    cp, evict, fx = e.promote_to_l0(_h("a"), _pages())
    assert e.local_tier(_h("a")) == H.TierId.L0 and cp.to_device and evict == []
    assert bytes(e._buf[cp.slot * BB:(cp.slot + 1) * BB].numpy()) == _blk("a")
    back = e.demote_l0(_h("a"))
    assert e.local_tier(_h("a")) == H.TierId.L1 and not back.to_device and back.page == cp.page


def test_l0_pressure_reports_collateral(tmp_path):
    e = _engine(tmp_path, (1, 8, 8))
    _put(e, "c0")
    _put(e, "c1")
    c0, _, _ = e.promote_to_l0(_h("c0"), _pages())
    c1, evict, fx = e.promote_to_l0(_h("c1"), _pages())
    assert fx.l0_demoted == [_h("c0")] and e.l0_len() == 1
    assert [(x.hash, x.page, x.to_device) for x in evict] == [(_h("c0"), c0.page, False)]
    assert c1.page == c0.page  # the victim's page is the one the new block lands in


def test_read_miss_from_l3_lands_back_in_l2(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    _put(e, "z")
    assert e.demote_l2_to_l3(_h("z"))
    assert not e.is_l2_durable(_h("z")) and e.l3_present(_h("z"))
    cp, _, fx = e.promote_to_l0(_h("z"), _pages())
    assert e.local_tier(_h("z")) == H.TierId.L0
    assert e.is_l2_durable(_h("z")) and fx.l2_demoted_to_l3 == []
    assert bytes(e._buf[cp.slot * BB:(cp.slot + 1) * BB].numpy()) == _blk("z")
    e.drop_l0(_h("z"))
    e.discard(_h("z"))  # drops the local copies; L3 stays the source of truth
    assert e.local_tier(_h("z")) == H.TierId.L3 and e.read_bytes(_h("z")) == _blk("z")


def test_l3_rehydration_demotes_the_coldest_l2_block_under_the_cap(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    _put(e, "a")
    e.demote_l2_to_l3(_h("a"))
    _put(e, "b")
    _, _, fx = e.promote_to_l0(_h("a"), _pages())
    assert fx.l2_demoted_to_l3 == [_h("b")]
    assert e.is_l2_durable(_h("a")) and not e.is_l2_durable(_h("b")) and e.l3_present(_h("b"))
    assert e.read_bytes(_h("b")) == _blk("b")


def test_l3_rehydration_skipped_when_every_l2_resident_is_pinned(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    _put(e, "a")
    e.demote_l2_to_l3(_h("a"))
    _put(e, "b")
    e.pin(_h("b"))
    order = e.l2_order()
    _, _, fx = e.promote_to_l0(_h("a"), _pages())
    assert e.local_tier(_h("a")) == H.TierId.L0 and not e.is_l2_durable(_h("a")) and e.l3_present(_h("a"))
    assert fx.l2_demoted_to_l3 == [] and e.l2_order() == order and e.is_l2_durable(_h("b"))
    assert e.l2_placement(_h("a")) is None  # its trial slot was given back


def test_pipeline_fill_miss_publishes_the_rehydrated_l2_copy_and_its_demotion(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    _put(e, "a")
    e.demote_l2_to_l3(_h("a"))
    _put(e, "b")
    pipe = H.TierPipeline(e, H.BandwidthPool(1 << 30, 1000), "n0")
    pipe.enqueue(H.Action(H.ActionKind.FILL_MISS, _h("a")))
    n, events, copies = pipe.tick(1, 0, _pages())
    assert n == 1 and [c.hash for c in copies] == [_h("a")]
    got = {(ev.kind, ev.hash, ev.tier) for ev in events}
    assert (H.LocKind.ABSENT, _h("b"), 3) in got and (H.LocKind.L3_PRESENT, _h("b"), 4) in got
    assert (H.LocKind.PRESENT, _h("a"), 3) in got and (H.LocKind.PRESENT, _h("a"), 1) in got
    pa = e.l2_placement(_h("a"))
    l2_event = [ev for ev in events if ev.hash == _h("a") and ev.tier == 3][0]
    assert (l2_event.segment_id, l2_event.offset) == (pa.segment_id, pa.offset)


def test_l0_demote_allows_l3_only_backing(tmp_path):
    e = _engine(tmp_path, (1, 8, 8))
    _put(e, "p")
    e.promote_to_l0(_h("p"), _pages())
    assert e.demote_l2_to_l3(_h("p"))
    assert not e.is_l2_durable(_h("p")) and e.l3_present(_h("p"))
    _put(e, "q")
    _, _, fx = e.promote_to_l0(_h("q"), _pages())
    assert fx.l0_demoted == [_h("p")] and e.l0_len() == 1
    assert e.local_tier(_h("p")) == H.TierId.L1


def test_pin_blocks_demote_like_a_lock_ref(tmp_path):
    e = _engine(tmp_path, (1, 8, 8))
    _put(e, "p")
    e.promote_to_l0(_h("p"), _pages())
    e.pin(_h("p"))
    _put(e, "q")
    with pytest.raises(ValueError, match="pinned"):
        e.promote_to_l0(_h("q"), _pages())
    with pytest.raises(ValueError, match="pinned"):
        e.demote_l0(_h("p"))
    e.unpin(_h("p"))
    _, _, fx = e.promote_to_l0(_h("q"), _pages())
    assert fx.l0_demoted == [_h("p")]


# ------------------------------------------------------------------ L2 cap
def test_put_durable_is_l2_only_and_the_cap_moves_the_cold_block_to_l3(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    tier, fx = _put(e, "x")
    assert tier == H.TierId.L2 and not e.l3_present(_h("x")) and fx.l2_demoted_to_l3 == []
    tier, fx = _put(e, "y")
    assert tier == H.TierId.L2 and fx.l2_demoted_to_l3 == [_h("x")]
    assert not e.is_l2_durable(_h("x")) and e.l3_present(_h("x"))  # exactly one of L2 / L3
    assert e.is_l2_durable(_h("y")) and not e.l3_present(_h("y"))
    assert e.read_bytes(_h("x")) == _blk("x")


def test_a_pinned_cold_block_is_skipped_and_the_new_write_may_land_in_l3(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    _put(e, "x")
    e.pin(_h("x"))
    tier, fx = _put(e, "y")
    assert tier == H.TierId.L3 and fx.l2_demoted_to_l3 == [_h("y")]
    assert e.is_l2_durable(_h("x")) and e.l3_present(_h("y")) and e.has_durable_backing(_h("y"))
    assert e.read_bytes(_h("y")) == _blk("y")


def test_a_pinned_victim_keeps_its_l2_lru_position(tmp_path):
    e = _engine(tmp_path, (4, 8, 3))
    for n in ("x", "a", "b"):
        _put(e, n)
    e.pin(_h("x"))  # the coldest block, passed over by the cap scan but not rotated
    _put(e, "c")
    assert e.l3_present(_h("a")) and not e.is_l2_durable(_h("a"))
    assert e.l2_order() == [_h("x"), _h("b"), _h("c")]


def test_all_pinned_over_cap_errors_and_rolls_back(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    _put(e, "x")
    e.pin(_h("x"))
    e.pin(_h("y"))  # a reader's pin taken before the write lands
    order = e.l2_order()
    with pytest.raises(ValueError, match="pinned"):
        _put(e, "y")
    assert not e.is_l2_durable(_h("y")) and not e.l3_present(_h("y")) and not e.has_durable_backing(_h("y"))
    assert e.l2_len() == 1 and e.is_l2_durable(_h("x")) and e.l2_order() == order
    assert e.l2_placement(_h("y")) is None
    e.unpin(_h("x"))
    tier, fx = _put(e, "y")  # with the pin gone the same write settles
    assert tier == H.TierId.L2 and fx.l2_demoted_to_l3 == [_h("x")]


def test_a_failed_put_on_a_large_pinned_l2_keeps_the_order_bit_for_bit(tmp_path):
    e = _engine(tmp_path, (4, 8, 160))
    names = [f"b{i:04d}" for i in range(160)]
    for n in names:
        _put(e, n)
        e.pin(_h(n))
    e.pin(_h("y"))
    order = e.l2_order()
    assert order == [_h(n) for n in names]
    with pytest.raises(ValueError, match="pinned"):
        _put(e, "y")
    assert e.l2_order() == order and not e.has_durable_backing(_h("y"))
    tier, fx = _put(e, "b0000", tag="again")  # an overwrite keeps the resident count: it settles
    assert tier == H.TierId.L2 and fx.l2_demoted_to_l3 == []
    assert e.l2_order() == order[1:] + order[:1]  # and becomes the most recent write


def test_an_l3_write_failure_during_cap_demotion_changes_nothing(tmp_path):
    e = _engine(tmp_path, (4, 8, 1))
    _put(e, "x")
    blocker = _l3_tmp_path(tmp_path, "x")
    blocker.mkdir(parents=True)  # the L3 object cannot be created
    with pytest.raises(ValueError, match="L3"):
        _put(e, "y")
    assert e.is_l2_durable(_h("x")) and not e.l3_present(_h("x")) and e.l2_order() == [_h("x")]
    assert not e.has_durable_backing(_h("y")) and e.l2_placement(_h("y")) is None
    blocker.rmdir()
    tier, fx = _put(e, "y")
    assert tier == H.TierId.L2 and fx.l2_demoted_to_l3 == [_h("x")] and e.read_bytes(_h("x")) == _blk("x")


# ------------------------------------------------------------------ L2 write failures
def _fill_first_segment(e):
    names = [f"s{i:02d}" for i in range(64)]  # 64 slots per segment file
    for n in names:
        _put(e, n)
    assert {e.l2_placement(_h(n)).segment_id for n in names} == {1}
    return names


def test_a_failed_overwrite_keeps_the_previous_record(tmp_path):
    e = _engine(tmp_path, (4, 8, 128))
    names = _fill_first_segment(e)
    before = e.l2_placement(_h("s00"))
    order = e.l2_order()
    (tmp_path / "l2" / "seg_2.bin").mkdir()  # the spare slot's segment file cannot be opened
    with pytest.raises(ValueError, match="previous record is kept"):
        _put(e, "s00", tag="new")
    assert e.read_bytes(_h("s00")) == _blk("s00") and e.corrupt_reads() == 0
    after = e.l2_placement(_h("s00"))
    assert (after.segment_id, after.offset) == (before.segment_id, before.offset) and e.l2_order() == order
    (tmp_path / "l2" / "seg_2.bin").rmdir()
    _put(e, "s00", tag="new")
    moved = e.l2_placement(_h("s00"))
    assert e.read_bytes(_h("s00")) == _blk("s00", "new") and moved.segment_id == 2
    _put(e, "fresh")  # the old slot was given back: the next new block takes it
    reused = e.l2_placement(_h("fresh"))
    assert (reused.segment_id, reused.offset) == (before.segment_id, before.offset)
    assert all(e.read_bytes(_h(n)) == _blk(n) for n in names[1:])


def test_a_failed_new_write_leaves_no_slot_behind(tmp_path):
    e = _engine(tmp_path, (4, 8, 128))
    _fill_first_segment(e)
    (tmp_path / "l2" / "seg_2.bin").mkdir()
    with pytest.raises(ValueError, match="L2 write failed"):
        _put(e, "z")
    assert e.l2_placement(_h("z")) is None and not e.has_durable_backing(_h("z")) and e.l2_len() == 64
    (tmp_path / "l2" / "seg_2.bin").rmdir()
    tier, _ = _put(e, "z")
    assert tier == H.TierId.L2 and e.l2_placement(_h("z")).segment_id == 2 and e.read_bytes(_h("z")) == _blk("z")


# ------------------------------------------------------------------ hits / admission
def test_hit_count_counts_hits_only(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    _put(e, "a")
    assert e.probe(_h("a")) == H.AccessKind.L2_HIT and e.hit_count(_h("a")) == 1
    assert e.probe(_h("nobody")) == H.AccessKind.MISS and e.hit_count(_h("nobody")) == 0


def test_admitted_promote_marks_cold_blocks_one_shot_and_they_graduate(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    _put(e, "cold")
    _put(e, "hot")
    e.probe(_h("cold"))  # one hit, below the admission threshold of two
    e.promote_to_l0(_h("cold"), _pages())
    assert e.is_one_shot(_h("cold"))
    e.probe(_h("hot"))
    e.probe(_h("hot"))
    e.promote_to_l0(_h("hot"), _pages(8))
    assert not e.is_one_shot(_h("hot"))
    assert e.probe(_h("cold")) == H.AccessKind.L0_HIT  # the second hit graduates it
    assert not e.is_one_shot(_h("cold"))


@pytest.mark.parametrize("hot_first", [False, True])
def test_one_shot_blocks_are_evicted_before_hot_ones(tmp_path, hot_first):
    """Whichever of the two was promoted first (the LRU one), the one-shot block goes."""
    e = _engine(tmp_path, (2, 8, 8))
    for n in ("cold", "hot", "new"):
        _put(e, n)
    pages = _pages()
    e.probe(_h("cold"))
    e.probe(_h("hot"))
    e.probe(_h("hot"))
    for n in (("hot", "cold") if hot_first else ("cold", "hot")):
        e.promote_to_l0(_h(n), pages)
    _, _, fx = e.promote_to_l0(_h("new"), pages)
    assert fx.l0_demoted == [_h("cold")]
    assert e.local_tier(_h("cold")) == H.TierId.L1 and e.local_tier(_h("hot")) == H.TierId.L0


def test_async_promote_dedups_in_flight_requests(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    _put(e, "a")
    assert e.begin_promote(_h("a")) == H.BeginPromote.STARTED
    assert e.begin_promote(_h("a")) == H.BeginPromote.ALREADY_IN_FLIGHT
    assert e.promote_inflight_len() == 1
    e.promote_to_l0(_h("a"), _pages())
    e.finish_promote(_h("a"))
    assert e.promote_inflight_len() == 0 and e.local_tier(_h("a")) == H.TierId.L0
    assert e.begin_promote(_h("a")) == H.BeginPromote.ALREADY_L0
    assert e.begin_promote(_h("nobody")) == H.BeginPromote.MISSING


def test_an_engine_needs_an_l2_directory(tmp_path):
    with pytest.raises(ValueError, match="L2 directory"):
        H.TierEngine(H.TierCaps(1, 0, 1), BB, 0, "", str(tmp_path / "l3"), "m")


# ------------------------------------------------------------------ pipeline (rust/tiered-store/src/pipeline.rs:315-445)
def _pipe(e, budget=1 << 30):
    bw = H.BandwidthPool(budget, 1000)
    return H.TierPipeline(e, bw, "n0"), bw


def test_pipeline_promotion_emits_the_collateral_l0_absent(tmp_path):
    e = _engine(tmp_path, (1, 8, 8))
    _put(e, "a")
    _put(e, "b")
    p, _ = _pipe(e)
    pages = _pages()
    p.enqueue(H.Action(H.ActionKind.PROMOTE, _h("a")))
    assert p.tick(1, 0, pages)[0] == 1
    p.enqueue(H.Action(H.ActionKind.PROMOTE, _h("b")))
    n, events, copies = p.tick(1, 0, pages)
    assert n == 1
    assert any(ev.kind == H.LocKind.ABSENT and ev.hash == _h("a") and ev.tier == 1 for ev in events)
    assert [(c.hash, c.to_device) for c in copies] == [(_h("a"), False), (_h("b"), True)]  # copy out first


def test_pipeline_waits_for_the_next_window_when_the_budget_is_spent(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    _put(e, "a")
    _put(e, "b")
    p, _ = _pipe(e, budget=3 * BB)  # an L2 promotion is charged two block moves
    pages = _pages()
    p.enqueue(H.Action(H.ActionKind.PROMOTE, _h("a")))
    p.enqueue(H.Action(H.ActionKind.PROMOTE, _h("b")))
    n, _, _ = p.tick(8, 0, pages)
    assert n == 1 and p.pending() == 1 and e.local_tier(_h("b")) != H.TierId.L0
    assert p.tick(8, 500, pages)[0] == 0  # same window
    assert p.tick(8, 1000, pages)[0] == 1 and e.local_tier(_h("b")) == H.TierId.L0


def test_pipeline_requeues_a_failed_action_then_drops_it(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    p, _ = _pipe(e)
    p.enqueue(H.Action(H.ActionKind.PROMOTE, _h("missing")))
    assert p.tick(1, 0, _pages())[0] == 0 and p.pending() == 1  # failed: back in the queue
    assert p.tick(1, 0, _pages())[0] == 0 and p.pending() == 1
    assert p.tick(1, 0, _pages())[0] == 0 and p.pending() == 0  # third failure: dropped


def test_pipeline_compaction_waits_while_paused_then_emits_moves(tmp_path):
    e = _engine(tmp_path, (4, 8, 8))
    for n in ("a", "b", "c", "d"):
        _put(e, n)
    e.discard(_h("b"))  # a hole at slot 1
    p, bw = _pipe(e)
    p.enqueue(H.Action(H.ActionKind.COMPACT_SEGMENT, segment_id=1))
    H.sync_background_pause(bw, True)
    assert p.tick(8, 0, _pages())[0] == 0 and p.pending() == 1
    assert e.l2_placement(_h("d")).offset == 3 * e.record_bytes()
    H.sync_background_pause(bw, False)
    n, events, _ = p.tick(8, 0, _pages())
    assert n == 1
    assert [(ev.kind, ev.hash, ev.segment_id, ev.offset) for ev in events] == [
        (H.LocKind.MOVED, _h("d"), 1, e.record_bytes())]
    assert e.l2_placement(_h("d")).offset == e.record_bytes()
    assert all(e.read_bytes(_h(n)) == _blk(n) for n in ("a", "c", "d")) and e.corrupt_reads() == 0


def test_a_colocate_plan_runs_on_the_pipeline_and_moves_the_authority_location(tmp_path):
    """The control plane plans a co-locate move for a chain whose second block sits in another
    segment than its parent; the node queues it (paused background bandwidth holds it), runs it, and the
    MOVED event puts the block's L2 location next to its parent (putend.rs:1706-1790)."""
    e = _engine(tmp_path, (4, 8, 128))
    _put(e, "h0")
    for i in range(1, 64):
        _put(e, f"x{i}")  # fills segment 1
    _put(e, "h1")
    assert e.l2_placement(_h("h1")).segment_id == 2
    e.discard(_h("x1"))  # the slot next to h0 is free on the node
    slot = e.record_bytes()
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, BB))
    metas = [H.BlockMeta(H.KVBlockID("m", _h(n)), [H.Location(3, "n0", e.l2_placement(_h(n)).segment_id,
                                                              e.l2_placement(_h(n)).offset)])
             for n in ("h0", "h1")]
    a.register_blocks("n0", [_h("h0"), _h("h1")], metas)
    moves = a.plan_defrag("m", "", 1, 2, slot)  # COLOCATE
    assert [(m.id.block_hash, m.to_segment, m.to_offset) for m in moves] == [(_h("h1"), 1, slot)]
    other = H.DefragMove()
    other.node_id = "n1"
    other.compact_segment = True
    other.segment_id = 1
    p, bw = _pipe(e)
    H.sync_background_pause(bw, True)
    assert H.enqueue_defrag_moves(p, moves + [other]) == 1  # the other node's move is not ours
    assert p.tick(8, 0, _pages())[0] == 0
    H.sync_background_pause(bw, False)
    n, events, _ = p.tick(8, 0, _pages())
    assert n == 1
    assert H.apply_location_events(H.AuthorityPort(a), "m", "", 1, events) == 1
    loc = [l for l in a.locate([H.KVBlockID("m", _h("h1"))])[0].locations if l.tier == 3]
    assert [(l.segment_id, l.offset) for l in loc] == [(1, slot)]
    pl = e.l2_placement(_h("h1"))
    assert (pl.segment_id, pl.offset) == (1, slot) and e.read_bytes(_h("h1")) == _blk("h1")
