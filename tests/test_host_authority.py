"""Control-plane authority (C++), test cases modelled on the reference's
rust/controlplane unit tests (behaviour, not code)."""
import pytest

from lake_b200 import _host as H
from lake_b200.engine.block_pool import chain_block_hashes

M = "m"
BPB = 1000


def chain(n, seed=0):
    return chain_block_hashes(list(range(seed, seed + n * 16)), 16)


def meta(h, node="n0", tier=3, seg=1, off=0, l3=False):
    return H.BlockMeta(H.KVBlockID(M, h), [H.Location(tier, node, seg, off)], l3)


def auth(quota=None, cap=4096, pool=0):
    a = H.Authority(cap, pool)
    a.register_model(H.ModelDescriptor(M, "", 2, 16, BPB, 1, quota or H.Quota()))
    return a


def ref(h, kind, d, node=""):
    return H.RefDelta(H.KVBlockID(M, h), kind, d, node)


REQUEST, WRITEBACK, IN_FLIGHT = 1, 3, 2
L0, L1, L2 = 1, 2, 3


def test_register_requires_model_and_contiguity_and_durability():
    a = H.Authority()
    hs = chain(3)
    with pytest.raises(ValueError, match="not registered"):
        a.register_blocks("n0", hs, [meta(hs[0])])
    a = auth()
    with pytest.raises(ValueError, match="contiguous"):
        a.register_blocks("n0", hs, [meta(hs[0]), meta(hs[2])])
    with pytest.raises(ValueError, match="durable"):
        a.register_blocks("n0", hs, [H.BlockMeta(H.KVBlockID(M, hs[0]))])
    assert a.register_blocks("n0", hs, [meta(h) for h in hs]).accepted
    assert a.block_count(M, "") == 3
    assert a.used_bytes(M, "") == 3 * BPB
    # idempotent re-register charges nothing
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    assert a.used_bytes(M, "") == 3 * BPB


def test_lookup_prefix_gap_lineage_and_local_hit():
    a = auth()
    hs = chain(4)
    a.register_blocks("n0", hs[:2], [meta(hs[0], tier=L0), meta(hs[1])])
    r = a.lookup_prefix(M, "", 0, hs, "n0")
    assert r.hit_length == 2 and not r.all_local_hit
    assert [b.local_hit for b in r.blocks] == [True, False]
    r = a.lookup_prefix(M, "", 0, hs[:1], "n0")
    assert r.all_local_hit
    # same flat hash reached through a different prefix: lineage mismatch -> miss
    other = [b"\x01" * 32, hs[1]]
    assert a.lookup_prefix(M, "", 0, other, "n0").hit_length == 0
    # draft pool is a separate namespace
    assert a.lookup_prefix(M, "", 2, hs, "n0").hit_length == 0


def test_refs_by_kind_underflow_all_or_nothing_and_freeze():
    a = auth()
    hs = chain(2)
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    a.report_refs([ref(hs[0], REQUEST, 1, "n0"), ref(hs[0], WRITEBACK, 1, "n0")])
    assert a.refs_by_kind(H.KVBlockID(M, hs[0])) == (1, 1)
    # batch with an underflow leaves state untouched
    with pytest.raises(ValueError, match="underflow"):
        a.report_refs([ref(hs[0], REQUEST, -1), ref(hs[1], REQUEST, -1)])
    assert a.refs_by_kind(H.KVBlockID(M, hs[0])) == (1, 1)
    with pytest.raises(ValueError, match="unsupported ref_kind"):
        a.report_refs([ref(hs[0], IN_FLIGHT, 1)])
    # referenced block cannot be evicted; after release it becomes inactive and evictable (leaf first)
    a.report_refs([ref(hs[1], REQUEST, 1), ref(hs[1], REQUEST, -1)])
    a.report_refs([ref(hs[0], REQUEST, -1, "n0"), ref(hs[0], WRITEBACK, -1, "n0")])
    assert a.inactive_len(M, "", 1) == 2
    assert a.evict_n(M, "", 1, 1) == 1
    # the leaf (hs[1]) went first; root remains
    assert a.lookup_prefix(M, "", 0, hs, "").hit_length == 1


def test_view_log_snapshot_replay_and_events():
    a = auth()
    hs = chain(2)
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    u1 = a.commit_pending()
    assert u1.seq == 1 and [e.kind for e in u1.events] == [0, 0]  # REGISTERED
    a.publish_location(H.KVBlockID(M, hs[0]), L0, "n1", 1, 0, True)
    u2 = a.commit_pending()
    assert u2.events[0].kind == 2  # MOVED
    assert [u.seq for u in a.replay_after(1)] == [2]
    assert a.replay_after(0) is None
    snap = a.snapshot()
    assert snap.seq == 0 and len(snap.events) == 2


def test_quota_hard_reject_without_mutation_and_soft_eviction():
    a = auth(H.Quota(2 * BPB, 3 * BPB, False))
    hs = chain(5)
    assert a.register_blocks("n0", hs[:3], [meta(h) for h in hs[:3]]).accepted
    r = a.register_blocks("n0", hs[:4], [meta(hs[3])])
    assert not r.accepted and r.backpressure.reason == "HARD_QUOTA"
    assert r.backpressure.deficit_bytes == BPB
    assert a.block_count(M, "") == 3
    # free an inactive leaf: the admission now evicts it to fit
    a.report_refs([ref(hs[2], REQUEST, 1), ref(hs[2], REQUEST, -1)])
    hs2 = chain(1, seed=999)
    r = a.register_blocks("n0", hs2, [meta(hs2[0])])
    assert r.accepted and a.block_count(M, "") == 3
    assert not a.preflight_register(M, "", 1, [b"z" * 32, b"y" * 32]).accepted


def test_borrow_reclaims_from_over_soft_namespace():
    a = H.Authority(4096, 4 * BPB)
    a.register_model(H.ModelDescriptor("a", "", 2, 16, BPB, 1, H.Quota(1 * BPB, 0, True)))
    a.register_model(H.ModelDescriptor("b", "", 2, 16, BPB, 1, H.Quota(1 * BPB, 0, True)))
    ha = chain_block_hashes(list(range(48)), 16)
    a.register_blocks("n0", ha, [H.BlockMeta(H.KVBlockID("a", h), [H.Location(L2, "n0")]) for h in ha])
    for h in ha:
        a.report_refs([H.RefDelta(H.KVBlockID("a", h), REQUEST, 1), H.RefDelta(H.KVBlockID("a", h), REQUEST, -1)])
    hb = chain_block_hashes(list(range(1000, 1048)), 16)
    r = a.register_blocks("n0", hb, [H.BlockMeta(H.KVBlockID("b", h), [H.Location(L2, "n0")]) for h in hb])
    assert r.accepted
    assert a.used_bytes("a", "") < 3 * BPB  # borrower gave bytes back


def test_orphans_gc_dead_node_and_discard():
    a = auth()
    now = [1000]
    a.set_clock(lambda: now[0])
    a.report_orphans([H.OrphanReport("n0", [H.KVBlockID(M, b"o" * 32)], 0)])
    assert a.orphan_count() == 1
    assert a.sweep_orphans(30000) == []
    now[0] += 30001
    assert len(a.sweep_orphans(30000)) == 1
    hs = chain(2)
    a.register_blocks("n0", hs, [meta(hs[0], tier=L0), meta(hs[1], tier=L0)])
    a.publish_location(H.KVBlockID(M, hs[1]), L2, "n0", 1, 0, True)
    a.report_refs([ref(hs[0], REQUEST, 1, "n1"), ref(hs[1], REQUEST, 1, "n1")])
    cleared, stripped = a.reconcile_dead_node("n1")
    assert cleared == 2 and stripped == []
    cleared, stripped = a.reconcile_dead_node("n0")
    assert len(stripped) == 2  # L0 copies on n0 removed
    # cold GC: hs[1] durable (L2) -> stripped; hs[0] not durable -> discarded
    discarded, stripped = a.gc_cold(M, "", 1, 8)
    assert len(discarded) + len(stripped) >= 1
    with pytest.raises(ValueError, match="referenced"):
        a2 = auth()
        a2.register_blocks("n0", hs[:1], [meta(hs[0])])
        a2.report_refs([ref(hs[0], REQUEST, 1)])
        a2.discard_blocks([H.KVBlockID(M, hs[0])])


def test_checkpoint_roundtrip_rebuilds_radix():
    a = auth()
    hs = chain(3)
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    snap = a.export_snapshot()
    b = H.Authority()
    b.import_snapshot(snap)
    assert b.lookup_prefix(M, "", 0, hs, "").hit_length == 3
    assert b.has_namespace(M, "")


def test_shard_join_drain_remove_and_warmup():
    a = auth()
    hs = chain(40)
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    a.join_shard_node("s0", 64)
    migs, warm = a.join_shard_node("s1", 64)
    assert 0 < len(migs) < 40 and all(m.to_node == "s1" for m in migs)
    assert a.shard_map().generation == 2
    migs, push = a.drain_shard_node("s1")
    assert all(m.from_node == "s1" for m in migs)
    with pytest.raises(ValueError):
        a.remove_shard_node("s0")  # not drained
    a.remove_shard_node("s1")
    assert a.ready_nodes() == ["s0"]


def test_hrw_vectors_and_preplacement():
    # cross-language anchors (rust/controlplane/src/placement.rs:277-295)
    assert H.fnv1a64(b"") == 14695981039346656037
    assert H.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert H.fnv1a64(b"lake") == 0x0471D1AD906F0DDE
    assert H.hrw_score(b"anchor-0", "n0") == 0xC8E4E7B063E4EF7F
    assert H.hrw_score(b"key!", "worker-1") == 0xD485E7E9B3D80A5F
    a = auth()
    a.join_shard_node("n0", 8)
    a.join_shard_node("n1", 8)
    hs = chain(3)
    a.register_blocks("nx", hs, [meta(h, node="nx") for h in hs])
    plan = a.preplace_on_register(M, "", 1, hs)
    assert plan is not None and len(plan.ids) == 3
    assert a.preplace_on_register(M, "", 1, hs) is None  # hysteresis marks


def test_follow_traffic_and_hits():
    a = auth()
    hs = chain(2)
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    ids = [H.KVBlockID(M, h) for h in hs]
    assert a.report_hits("n5", ids) == []
    plans = a.report_hits("n5", ids)
    assert plans and plans[0].node_id == "n5"
    assert a.hit_count_on(ids[0], "n5") == 2


def test_defrag_plans_and_relocate():
    a = auth()
    hs = chain(3)
    metas = [meta(hs[0], seg=1, off=0), meta(hs[1], seg=1, off=2 * 4096), meta(hs[2], seg=2, off=0)]
    a.register_blocks("n0", hs, metas)
    assert a.l2_fragmentation_ratio(M, "", 1, 4096) > 0
    moves = a.plan_defrag(M, "", 1, 1, 4096)  # COMPACT
    assert len(moves) == 1 and moves[0].to_offset == 4096
    assert a.relocate_in_view(moves) == 1
    assert a.l2_fragmentation_ratio(M, "", 1, 4096) == 0.0
    col = a.plan_defrag(M, "", 1, 2, 4096)  # COLOCATE: hs[2] moves next to its parent
    assert any(m.to_segment == 1 for m in col)


def test_frequency_buckets_order_inactive_eviction():
    """Inactive blocks leave in frequency-bucket order (lookups touch the counter; thresholds
    3 / 8 / 15), least recently used first inside a bucket."""
    a = auth()
    A, B, C = chain(1, seed=0), chain(1, seed=1000), chain(1, seed=2000)
    for X in (A, B, C):
        a.register_blocks("n0", X, [meta(h) for h in X])
        a.report_refs([ref(X[0], REQUEST, 1), ref(X[0], REQUEST, -1)])
    assert a.inactive_len(M, "", 1) == 3
    for _ in range(10):
        a.lookup_prefix(M, "", 0, A, "")
    for _ in range(4):
        a.lookup_prefix(M, "", 0, C, "")
    assert a.evict_n(M, "", 1, 1) == 1  # B: never looked up
    assert a.evict_n(M, "", 1, 1) == 1  # C: lower bucket than A
    assert [a.lookup_prefix(M, "", 0, X, "").hit_length for X in (A, B, C)] == [1, 0, 0]


def test_quota_locate_l3_barrier_pause_and_deregister():
    a = auth()
    hs = chain(2)
    a.register_blocks("n0", hs, [meta(h) for h in hs])
    q = H.Quota()
    q.soft_bytes, q.hard_bytes, q.borrow_enabled = 5 * BPB, 8 * BPB, True
    a.set_quota(M, "", q)
    g = a.get_quota(M, "")
    assert (g.soft_bytes, g.hard_bytes, g.borrow_enabled) == (5 * BPB, 8 * BPB, True)
    # locate reports every location and the L3 flag (which the object store sets separately)
    loc = a.locate([H.KVBlockID(M, hs[0])])
    assert [(l.tier, l.node_id) for l in loc[0].locations] == [(L2, "n0")] and not loc[0].l3_present
    a.set_l3_present(H.KVBlockID(M, hs[0]), True)
    assert a.locate([H.KVBlockID(M, hs[0])])[0].l3_present
    # request barrier: complete once a node acknowledges
    assert not a.barrier_completed("req-1")
    a.complete_barrier("req-1", "n0")
    assert a.barrier_completed("req-1")
    a.set_background_paused(True)
    assert a.background_paused()
    a.set_background_paused(False)
    assert not a.background_paused()
    # deregistering drops the namespace with its blocks
    assert a.has_namespace(M, "")
    a.deregister_model(M, "")
    assert not a.has_namespace(M, "")
    with pytest.raises(ValueError, match="not registered"):
        a.register_blocks("n0", hs, [meta(h) for h in hs])
