"""Control-plane authority: one test per behaviour that the reference's control-plane
unit tests pin (rust/controlplane/src/lib.rs:1108-3992), written against this
framework's C++ authority through its Python binding. The cases reproduce the
reference's inputs and expected outcomes; where this authority deliberately behaves
differently the test says so (zero-ref blocks past the inactive-index cap wait in an
overflow queue instead of never becoming evictable)."""
import pytest

from lake_b200 import _host as H

REQUEST, IN_FLIGHT, WRITEBACK = 1, 2, 3
TARGET, DRAFT = 1, 2
L0, L1, L2 = 1, 2, 3
REGISTERED, INVALIDATED, MOVED = 0, 1, 2
COMPACT, COLOCATE = 1, 2


def model(a, m="m", rev="", soft=0, hard=0, borrow=False, bpb=0, layers=32):
    a.register_model(H.ModelDescriptor(m, rev, layers, 128, bpb, 1, H.Quota(soft, hard, borrow)))


def bid(h, m="m", rev="", pk=TARGET):
    return H.KVBlockID(m, h, pk, rev)


def meta(h, m="m", rev="", node="n0", seg=1, off=0, pk=TARGET, l0=False):
    locs = [H.Location(L2, node, seg, off)]
    if l0:
        locs.append(H.Location(L0, node, 0, 0))
    return H.BlockMeta(bid(h, m, rev, pk), locs)


def reg(a, chain, metas, node="n0"):
    return a.register_blocks(node, list(chain), metas)


def ref(a, h, d, m="m", kind=REQUEST, node="n0", rev=""):
    a.report_refs([H.RefDelta(bid(h, m, rev), kind, d, node)])


def hit(a, chain, m="m", rev="", pk=TARGET, node="n0"):
    return a.lookup_prefix(m, rev, pk, list(chain), node).hit_length


def total_refs(a, h, m="m"):
    req, wb = a.refs_by_kind(bid(h, m))
    return req + wb


def release_cycle(a, h, m="m"):
    ref(a, h, 1, m)
    ref(a, h, -1, m)


# ------------------------------------------------------------------ lookup / register
def test_lookup_prefix_contiguous_then_gap():
    a = H.Authority()
    model(a)
    reg(a, [b"h0", b"h1", b"h2"], [meta(b"h0"), meta(b"h1"), meta(b"h2")])
    r = a.lookup_prefix("m", "", TARGET, [b"h0", b"gap", b"h2"], "n0")
    assert r.hit_length == 1 and len(r.blocks) == 1 and not r.all_local_hit


def test_lookup_full_hit_is_not_local_without_l0():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b"], [meta(b"a"), meta(b"b")])
    r = a.lookup_prefix("m", "", TARGET, [b"a", b"b"], "n0")
    assert r.hit_length == 2 and not r.all_local_hit


def test_cross_model_isolation():
    a = H.Authority()
    model(a, "m1")
    model(a, "m2")
    reg(a, [b"shared"], [meta(b"shared", "m1")])
    reg(a, [b"shared"], [meta(b"shared", "m2")])
    assert hit(a, [b"shared"], "m1") == 1 and hit(a, [b"shared"], "m2") == 1
    assert hit(a, [b"other"], "m1") == 0


def test_register_requires_prefix_hashes():
    a = H.Authority()
    model(a)
    with pytest.raises(ValueError, match="prefix_hashes"):
        reg(a, [], [meta(b"a")])


def test_register_requires_registered_model():
    a = H.Authority()
    with pytest.raises(ValueError, match="not registered"):
        reg(a, [b"a"], [meta(b"a")])


def test_register_missing_suffix_with_full_chain():
    a = H.Authority()
    model(a)
    full = [b"h0", b"h1", b"h2"]
    reg(a, full, [meta(b"h0"), meta(b"h1")])
    reg(a, full, [meta(b"h2")])
    assert hit(a, full) == 3


def test_register_rejects_non_contiguous_subset():
    a = H.Authority()
    model(a)
    with pytest.raises(ValueError, match="contiguous"):
        reg(a, [b"h0", b"h1", b"h2"], [meta(b"h0"), meta(b"h2")])


def test_lookup_stops_on_lineage_mismatch():
    a = H.Authority()
    model(a)
    reg(a, [b"A", b"B"], [meta(b"A"), meta(b"B")])
    r = a.lookup_prefix("m", "", TARGET, [b"B"], "n0")
    assert r.hit_length == 0 and not r.blocks


def test_register_rejects_a_block_without_a_durable_copy():
    a = H.Authority()
    model(a)
    with pytest.raises(ValueError, match="durable"):
        reg(a, [b"bare"], [H.BlockMeta(bid(b"bare"))])


def test_publish_l0_enables_local_hit():
    a = H.Authority()
    model(a)
    reg(a, [b"loc"], [meta(b"loc")])
    a.publish_location(bid(b"loc"), L0, "n0", 0, 0, True)
    assert a.lookup_prefix("m", "", TARGET, [b"loc"], "n0").all_local_hit
    a.publish_location(bid(b"loc"), L0, "n0", 0, 0, False)
    assert not a.lookup_prefix("m", "", TARGET, [b"loc"], "n0").all_local_hit


# ------------------------------------------------------------------ refs / eviction
def test_ref_freeze_and_evict():
    a = H.Authority()
    model(a)
    reg(a, [b"x"], [meta(b"x")])
    ref(a, b"x", 1)
    assert total_refs(a, b"x") == 1 and a.inactive_len("m", "", TARGET) == 0
    ref(a, b"x", -1)
    assert total_refs(a, b"x") == 0 and a.inactive_len("m", "", TARGET) == 1
    ref(a, b"x", 1)
    assert a.inactive_len("m", "", TARGET) == 0
    ref(a, b"x", -1)
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert hit(a, [b"x"]) == 0


def test_report_ref_batch_all_or_nothing_on_unknown_block():
    a = H.Authority()
    model(a)
    reg(a, [b"p"], [meta(b"p")])
    ref(a, b"p", 1)
    with pytest.raises(ValueError, match="unknown block_hash"):
        a.report_refs([H.RefDelta(bid(b"p"), REQUEST, -1, "n0"), H.RefDelta(bid(b"missing"), REQUEST, -1, "n0")])
    assert total_refs(a, b"p") == 1


def test_referenced_block_is_not_evicted():
    a = H.Authority()
    model(a)
    reg(a, [b"y"], [meta(b"y")])
    ref(a, b"y", 1)
    assert a.evict_n("m", "", TARGET, 10) == 0
    assert hit(a, [b"y"]) == 1


def test_frequency_evicts_colder_leaf_first():
    a = H.Authority()
    model(a)
    reg(a, [b"cold"], [meta(b"cold")])
    reg(a, [b"hot"], [meta(b"hot")])
    for _ in range(64):
        a.lookup_prefix("m", "", TARGET, [b"hot"], "n0")
    for h in (b"cold", b"hot"):
        release_cycle(a, h)
    assert a.inactive_len("m", "", TARGET) == 2
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert hit(a, [b"cold"]) == 0 and hit(a, [b"hot"]) == 1


def test_leaf_is_evicted_before_its_prefix_parent():
    a = H.Authority()
    model(a)
    reg(a, [b"parent", b"child"], [meta(b"parent"), meta(b"child")])
    for h in (b"parent", b"child"):
        release_cycle(a, h)
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert hit(a, [b"parent"]) == 1
    assert hit(a, [b"parent", b"child"]) == 1
    # the parent became a leaf: the next eviction may take it
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert hit(a, [b"parent"]) == 0


def test_one_batch_walks_a_chain_leaf_to_root():
    a = H.Authority()
    model(a)
    chain = [b"c0", b"c1", b"c2", b"c3"]
    reg(a, chain, [meta(h) for h in chain])
    for h in chain:
        release_cycle(a, h)
    assert a.evict_n("m", "", TARGET, 4) == 4
    assert a.block_count("m", "") == 0


def test_inactive_cap_overflow_keeps_every_release_evictable():
    """The reference skips the insert at the cap, so those blocks stay registered with zero
    refs and can never be evicted. Here they wait in an overflow queue: the index stays at its
    cap, no view entry is dropped, and every one of them is evicted once room frees up."""
    cap = 4
    a = H.Authority(cap)
    model(a)
    flats = [f"leaf{i:02d}".encode() for i in range(2 * cap)]
    for i, f in enumerate(flats):
        reg(a, [f], [meta(f)])
        release_cycle(a, f)
        assert a.inactive_len("m", "", TARGET) <= cap
    assert a.inactive_len("m", "", TARGET) == cap
    assert hit(a, [flats[0]]) == 1
    assert a.evict_n("m", "", TARGET, cap) == cap
    assert a.inactive_len("m", "", TARGET) == cap  # the waiting releases moved in
    assert a.evict_n("m", "", TARGET, cap) == cap
    assert a.block_count("m", "") == 0


def test_ref_batch_does_not_evict_a_peer_mid_batch():
    a = H.Authority(1)
    model(a)
    reg(a, [b"held"], [meta(b"held")])
    reg(a, [b"cand"], [meta(b"cand")])
    release_cycle(a, b"cand")
    ref(a, b"held", 1)
    assert a.inactive_len("m", "", TARGET) == 1
    a.report_refs([H.RefDelta(bid(b"held"), REQUEST, -1, "n0"), H.RefDelta(bid(b"cand"), REQUEST, 1, "n0")])
    assert total_refs(a, b"held") == 0 and total_refs(a, b"cand") == 1
    assert hit(a, [b"cand"]) == 1
    # held is the zero-ref one now, and it is evictable (not stranded past the cap)
    assert a.evict_n("m", "", TARGET, 5) == 1
    assert hit(a, [b"held"]) == 0 and hit(a, [b"cand"]) == 1


def test_writeback_ref_freezes_until_cleared():
    a = H.Authority()
    model(a)
    reg(a, [b"wb0"], [meta(b"wb0")])
    ref(a, b"wb0", 1, kind=WRITEBACK)
    assert total_refs(a, b"wb0") == 1
    assert a.evict_n("m", "", TARGET, 10) == 0
    ref(a, b"wb0", -1, kind=WRITEBACK)
    a.complete_barrier("req-wb", "n0")
    assert a.barrier_completed("req-wb")
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert hit(a, [b"wb0"]) == 0


def test_request_barrier_requires_ids():
    a = H.Authority()
    with pytest.raises(ValueError):
        a.complete_barrier("", "n0")
    with pytest.raises(ValueError):
        a.complete_barrier("r", "")


def test_ref_accounts_split_by_kind():
    a = H.Authority()
    model(a)
    reg(a, [b"k"], [meta(b"k")])
    ref(a, b"k", 1, kind=REQUEST)
    ref(a, b"k", 1, kind=WRITEBACK)
    assert a.refs_by_kind(bid(b"k")) == (1, 1)
    ref(a, b"k", -1, kind=WRITEBACK)
    assert a.refs_by_kind(bid(b"k")) == (1, 0)
    assert a.inactive_len("m", "", TARGET) == 0
    ref(a, b"k", -1, kind=REQUEST)
    assert a.refs_by_kind(bid(b"k")) == (0, 0)
    assert a.inactive_len("m", "", TARGET) == 1


def test_ref_underflow_is_scoped_by_kind():
    a = H.Authority()
    model(a)
    reg(a, [b"u"], [meta(b"u")])
    ref(a, b"u", 1, kind=WRITEBACK)
    with pytest.raises(ValueError, match=r"ref_count underflow \(kind=REQUEST\)"):
        ref(a, b"u", -1, kind=REQUEST, node="")
    assert a.refs_by_kind(bid(b"u")) == (0, 1)
    with pytest.raises(ValueError, match="unsupported ref_kind"):
        ref(a, b"u", 1, kind=IN_FLIGHT)
    with pytest.raises(ValueError, match="unsupported ref_kind"):
        a.report_refs([H.RefDelta(bid(b"u"), REQUEST, 1, "n0"), H.RefDelta(bid(b"u"), IN_FLIGHT, 1, "n0")])
    assert a.refs_by_kind(bid(b"u")) == (0, 1)


def test_dead_node_reconcile_clears_each_kind():
    a = H.Authority()
    model(a)
    reg(a, [b"z"], [meta(b"z")])
    ref(a, b"z", 1, kind=REQUEST)
    ref(a, b"z", 1, kind=WRITEBACK)
    assert a.evict_n("m", "", TARGET, 1) == 0
    cleared, _ = a.reconcile_dead_node("n0")
    assert cleared == 1
    assert a.refs_by_kind(bid(b"z")) == (0, 0)
    assert a.evict_n("m", "", TARGET, 1) == 1


def test_underflow_is_rejected_and_leaves_nothing_inactive():
    a = H.Authority()
    model(a)
    reg(a, [b"under"], [meta(b"under")])
    with pytest.raises(ValueError, match="underflow"):
        ref(a, b"under", -1)
    assert total_refs(a, b"under") == 0 and a.inactive_len("m", "", TARGET) == 0


def test_underflow_in_a_batch_is_all_or_nothing():
    a = H.Authority()
    model(a)
    reg(a, [b"ok", b"bad"], [meta(b"ok"), meta(b"bad")])
    with pytest.raises(ValueError, match="underflow"):
        a.report_refs([H.RefDelta(bid(b"ok"), REQUEST, 1, "n0"), H.RefDelta(bid(b"bad"), REQUEST, -1, "n0")])
    assert total_refs(a, b"ok") == 0 and total_refs(a, b"bad") == 0


def test_node_underflow_in_a_batch_is_all_or_nothing():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b"], [meta(b"a"), meta(b"b")])
    ref(a, b"a", 1)
    with pytest.raises(ValueError, match="node_ref underflow"):
        a.report_refs([H.RefDelta(bid(b"b"), REQUEST, 1, "n0"), H.RefDelta(bid(b"a"), REQUEST, -1, "n1")])
    assert total_refs(a, b"a") == 1 and total_refs(a, b"b") == 0
    # the node ledgers were restored too: n0 can still release its reference
    ref(a, b"a", -1)
    assert total_refs(a, b"a") == 0


def test_view_events_cover_mutation_paths():
    a = H.Authority()
    model(a)
    reg(a, [b"h0", b"h1"], [meta(b"h0"), meta(b"h1")])
    u = a.commit_pending()
    assert u.seq == 1 and len(u.events) == 2 and all(e.kind == REGISTERED for e in u.events)
    a.publish_location(bid(b"h0"), L0, "n0", 0, 0, True)
    u = a.commit_pending()
    assert len(u.events) == 1 and u.events[0].kind == MOVED and len(u.events[0].locations) == 2
    a.discard_blocks([bid(b"h0")])
    u = a.commit_pending()
    assert [e.kind for e in u.events] == [INVALIDATED]
    release_cycle(a, b"h1")
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert any(e.kind == INVALIDATED for e in a.commit_pending().events)


def test_relocate_in_view_emits_moved():
    a = H.Authority()
    model(a)
    reg(a, [b"h0"], [meta(b"h0")])
    a.commit_pending()
    mv = H.DefragMove()
    mv.id, mv.node_id, mv.from_segment, mv.from_offset, mv.to_segment, mv.to_offset = bid(b"h0"), "n0", 1, 0, 7, 42
    assert a.relocate_in_view([mv]) == 1
    u = a.commit_pending()
    assert len(u.events) == 1 and u.events[0].kind == MOVED
    assert (u.events[0].locations[0].segment_id, u.events[0].locations[0].offset) == (7, 42)


# ------------------------------------------------------------------ namespaces
def test_two_models_same_hash_no_crosstalk():
    a = H.Authority()
    model(a, "llama")
    model(a, "qwen")
    reg(a, [b"same"], [meta(b"same", "llama")])
    assert hit(a, [b"same"], "qwen") == 0
    reg(a, [b"same"], [meta(b"same", "qwen")])
    assert hit(a, [b"same"], "llama") == 1 and hit(a, [b"same"], "qwen") == 1
    a.deregister_model("llama", "")
    assert hit(a, [b"same"], "llama") == 0 and hit(a, [b"same"], "qwen") == 1


def test_deregister_cascades_the_view():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b"], [meta(b"a"), meta(b"b")])
    a.commit_pending()
    a.deregister_model("m", "")
    assert not a.has_namespace("m", "") and a.block_count("m", "") == 0
    assert sum(e.kind == INVALIDATED for e in a.commit_pending().events) == 2
    model(a)
    reg(a, [b"a", b"b"], [meta(b"a")])
    assert hit(a, [b"a"]) == 1


def test_revision_isolation():
    a = H.Authority()
    model(a, rev="r1")
    model(a, rev="r2")
    reg(a, [b"pfx"], [meta(b"pfx", rev="r1")])
    reg(a, [b"pfx"], [meta(b"pfx", rev="r2")])
    assert hit(a, [b"pfx"], rev="r1") == 1 and hit(a, [b"pfx"], rev="r2") == 1
    a.deregister_model("m", "r1")
    assert hit(a, [b"pfx"], rev="r1") == 0 and hit(a, [b"pfx"], rev="r2") == 1
    assert a.has_namespace("m", "r2") and not a.has_namespace("m", "r1")


def test_register_model_is_idempotent_and_updates_quota():
    a = H.Authority()
    model(a)
    reg(a, [b"keep"], [meta(b"keep")])
    model(a, soft=1, hard=2, borrow=True)
    assert hit(a, [b"keep"]) == 1
    q = a.get_quota("m", "")
    assert (q.soft_bytes, q.hard_bytes, q.borrow_enabled) == (1, 2, True)


def test_register_model_rejects_an_identity_change():
    a = H.Authority()
    model(a)
    with pytest.raises(ValueError, match="conflicts"):
        model(a, layers=64)
    reg(a, [b"x"], [meta(b"x")])
    assert hit(a, [b"x"]) == 1


def test_target_and_draft_pools_do_not_crosstalk():
    a = H.Authority()
    model(a)
    reg(a, [b"shared"], [meta(b"shared")])
    reg(a, [b"shared"], [meta(b"shared", pk=DRAFT)])
    assert hit(a, [b"shared"], pk=TARGET) == 1 and hit(a, [b"shared"], pk=DRAFT) == 1
    assert len(a.locate([bid(b"shared", pk=TARGET)])) == 1 and len(a.locate([bid(b"shared", pk=DRAFT)])) == 1
    release_cycle(a, b"shared")  # TARGET only
    assert a.evict_n("m", "", TARGET, 1) == 1
    assert hit(a, [b"shared"], pk=TARGET) == 0 and hit(a, [b"shared"], pk=DRAFT) == 1


# ------------------------------------------------------------------ quota
def test_hard_quota_of_one_model_does_not_affect_another():
    a = H.Authority()
    model(a, "A", soft=100, hard=200, bpb=100)
    model(a, "B", soft=100, hard=200, bpb=100)
    assert reg(a, [b"a0"], [meta(b"a0", "A")]).accepted
    assert reg(a, [b"a1"], [meta(b"a1", "A")]).accepted
    r = reg(a, [b"a2"], [meta(b"a2", "A")])
    assert not r.accepted and r.backpressure.reason == "HARD_QUOTA" and r.backpressure.model_id == "A"
    assert r.backpressure.deficit_bytes > 0
    assert a.used_bytes("A", "") == 200 and a.block_count("A", "") == 2
    assert reg(a, [b"b0"], [meta(b"b0", "B")]).accepted
    assert a.used_bytes("B", "") == 100 and hit(a, [b"b0"], "B") == 1


def test_borrow_over_soft_and_reclaim_for_another_borrower():
    a = H.Authority(4096, 300)
    model(a, "A", soft=100, hard=300, borrow=True, bpb=100)
    model(a, "B", soft=100, hard=300, borrow=True, bpb=100)
    assert reg(a, [b"a0"], [meta(b"a0", "A")]).accepted
    assert reg(a, [b"a1"], [meta(b"a1", "A")]).accepted
    assert a.used_bytes("A", "") == 200
    release_cycle(a, b"a1", "A")
    assert reg(a, [b"b0"], [meta(b"b0", "B")]).accepted
    assert reg(a, [b"b1"], [meta(b"b1", "B")]).accepted
    assert a.used_bytes("A", "") <= 100 and a.used_bytes("B", "") == 200
    assert hit(a, [b"a1"], "A") == 0


def test_pool_capacity_reject_is_not_hard_quota():
    a = H.Authority(4096, 200)
    model(a, soft=100, hard=300, borrow=True, bpb=100)
    assert reg(a, [b"a0"], [meta(b"a0")]).accepted
    assert reg(a, [b"a1"], [meta(b"a1")]).accepted
    r = reg(a, [b"a2"], [meta(b"a2")])
    assert not r.accepted and r.backpressure.reason == "POOL_CAPACITY"
    assert r.backpressure.hard_bytes == 300 and r.backpressure.deficit_bytes > 0
    assert a.block_count("m", "") == 2


def test_set_quota_then_hard_backpressure():
    a = H.Authority()
    model(a, bpb=50)
    assert reg(a, [b"x"], [meta(b"x")]).accepted
    a.set_quota("m", "", H.Quota(50, 50, False))
    assert a.used_bytes("m", "") == 50 and a.get_quota("m", "").hard_bytes == 50
    r = reg(a, [b"y"], [meta(b"y")])
    assert not r.accepted and r.backpressure.reason == "HARD_QUOTA" and r.backpressure.hard_bytes == 50


def test_hard_reject_has_no_side_effects():
    a = H.Authority()
    model(a, soft=200, hard=200, bpb=100)
    assert reg(a, [b"a0"], [meta(b"a0")]).accepted
    assert reg(a, [b"a1"], [meta(b"a1")]).accepted
    a.set_quota("m", "", H.Quota(100, 100, False))
    release_cycle(a, b"a1")
    assert a.inactive_len("m", "", TARGET) == 1
    assert not reg(a, [b"a2"], [meta(b"a2")]).accepted
    assert hit(a, [b"a1"]) == 1 and a.block_count("m", "") == 2 and a.used_bytes("m", "") == 200


def test_soft_quota_evicts_own_zero_ref_blocks_first():
    a = H.Authority()
    model(a, soft=200, hard=400, bpb=100)
    for h in (b"s0", b"s1"):
        assert reg(a, [h], [meta(h)]).accepted
        release_cycle(a, h)
    assert reg(a, [b"s2"], [meta(b"s2")]).accepted
    assert a.used_bytes("m", "") == 200 and a.block_count("m", "") == 2
    assert hit(a, [b"s0"]) == 0  # the oldest release went first


def test_register_model_rejects_invalid_quota():
    a = H.Authority()
    with pytest.raises(ValueError, match="soft_bytes"):
        model(a, "bad", soft=200, hard=100)


def test_preflight_matches_register_without_mutating():
    a = H.Authority()
    model(a, soft=100, hard=100, bpb=100)
    assert a.preflight_register("m", "", TARGET, [b"p0"]).accepted
    assert a.block_count("m", "") == 0
    reg(a, [b"p0"], [meta(b"p0")])
    assert a.preflight_register("m", "", TARGET, [b"p0"]).accepted  # already registered: no charge
    r = a.preflight_register("m", "", TARGET, [b"p1", b"p1"])
    assert not r.accepted and r.backpressure.deficit_bytes == 100


# ------------------------------------------------------------------ reconcile / GC / checkpoint
def test_cold_gc_strips_l0_and_keeps_l2():
    a = H.Authority()
    model(a)
    reg(a, [b"c0"], [meta(b"c0", l0=True)])
    release_cycle(a, b"c0")
    discarded, stripped = a.gc_cold("m", "", TARGET, 1)
    assert len(stripped) == 1 and not discarded
    assert all(l.tier != L0 for l in a.locate([bid(b"c0")])[0].locations)
    assert hit(a, [b"c0"]) == 1


def test_cold_gc_reinserts_durable_blocks():
    a = H.Authority()
    model(a)
    reg(a, [b"c0"], [meta(b"c0", l0=True)])
    release_cycle(a, b"c0")
    assert a.inactive_len("m", "", TARGET) == 1
    _, stripped = a.gc_cold("m", "", TARGET, 1)
    assert len(stripped) == 1 and a.inactive_len("m", "", TARGET) == 1
    _, stripped = a.gc_cold("m", "", TARGET, 1)
    assert len(stripped) == 1 and a.inactive_len("m", "", TARGET) == 1


def test_orphan_ttl_discard():
    now = [1000]
    a = H.Authority()
    a.set_clock(lambda: now[0])
    model(a)
    a.report_orphans([H.OrphanReport("n0", [bid(b"zombie")], 1000)])
    assert a.sweep_orphans(30000) == []
    now[0] = 31000
    gone = a.sweep_orphans(30000)
    assert len(gone) == 1 and gone[0].block_hash == b"zombie"


def test_orphan_mark_is_cleared_by_a_later_register():
    now = [1000]
    a = H.Authority()
    a.set_clock(lambda: now[0])
    model(a)
    a.report_orphans([H.OrphanReport("n0", [bid(b"late")], 1000)])
    reg(a, [b"late"], [meta(b"late")])
    now[0] = 31000
    assert a.sweep_orphans(30000) == []
    assert hit(a, [b"late"]) == 1


def test_discard_rejects_a_referenced_block():
    a = H.Authority()
    model(a)
    reg(a, [b"live"], [meta(b"live")])
    ref(a, b"live", 1)
    with pytest.raises(ValueError, match="global_refs"):
        a.discard_blocks([bid(b"live")])
    assert hit(a, [b"live"]) == 1


def test_dead_node_clears_writeback_ref():
    a = H.Authority()
    model(a)
    reg(a, [b"wb"], [meta(b"wb")])
    ref(a, b"wb", 1, kind=WRITEBACK)
    assert a.evict_n("m", "", TARGET, 1) == 0
    cleared, _ = a.reconcile_dead_node("n0")
    assert cleared == 1 and total_refs(a, b"wb") == 0
    assert a.evict_n("m", "", TARGET, 1) == 1


def test_dead_node_l0_presence_is_per_node():
    a = H.Authority()
    model(a)
    reg(a, [b"l0"], [meta(b"l0")])
    a.publish_location(bid(b"l0"), L0, "n0", 0, 0, True)
    a.publish_location(bid(b"l0"), L0, "n1", 0, 0, True)
    a.reconcile_dead_node("n0")
    l0 = lambda: sorted(l.node_id for l in a.locate([bid(b"l0")])[0].locations if l.tier == L0)  # noqa: E731
    assert l0() == ["n1"]
    a.reconcile_dead_node("n1")
    assert l0() == []


def test_dead_node_clears_reference_counts_beyond_int32():
    a = H.Authority()
    model(a)
    reg(a, [b"big"], [meta(b"big")])
    for d in (2**31 - 1, 2):
        ref(a, b"big", d)
    assert total_refs(a, b"big") == 2**31 + 1
    cleared, _ = a.reconcile_dead_node("n0")
    assert cleared == 1 and total_refs(a, b"big") == 0


def test_checkpoint_roundtrip_keeps_multi_block_lineage():
    a = H.Authority()
    model(a)
    full = [b"h0", b"h1"]
    reg(a, full, [meta(b"h0"), meta(b"h1")])
    snap = a.export_snapshot()
    assert len(snap.blocks) == 2 and any(len(b.prefix_chain) == 2 for b in snap.blocks)
    b = H.Authority()
    b.import_snapshot(snap)
    assert b.has_namespace("m", "") and hit(b, full) == 2


def test_checkpoint_restore_rejects_quota_loss():
    a = H.Authority()
    model(a, bpb=100)
    reg(a, [b"q"], [meta(b"q")])
    snap = a.export_snapshot()
    snap.models[0].quota = H.Quota(50, 50, False)
    b = H.Authority()
    with pytest.raises(ValueError, match="import_snapshot register rejected"):
        b.import_snapshot(snap)
    assert b.block_count("m", "") == 0


# ------------------------------------------------------------------ defrag
def test_compact_plan_on_holes():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b", b"c"], [meta(b"a", off=0), meta(b"b", off=200), meta(b"c", off=300)])
    moves = a.plan_defrag("m", "", TARGET, COMPACT, 100)
    assert len(moves) == 1 and moves[0].compact_segment and moves[0].segment_id == 1
    assert (moves[0].from_offset, moves[0].to_offset) == (300, 100)


def test_compact_skips_a_segment_with_a_referenced_block():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b", b"c"], [meta(b"a", off=0), meta(b"b", off=200), meta(b"c", off=300)])
    ref(a, b"b", 1)
    assert a.plan_defrag("m", "", TARGET, COMPACT, 100) == []


def test_colocate_packs_a_scattered_chain_on_one_node():
    a = H.Authority()
    model(a)
    reg(a, [b"h0", b"h1"], [meta(b"h0", seg=1), meta(b"h1", seg=2)])
    moves = a.plan_defrag("m", "", TARGET, COLOCATE, 64)
    assert any(not m.compact_segment and m.to_segment == 1 for m in moves)
    assert all(m.node_id == "n0" for m in moves)


def test_colocate_skips_cross_node_chains():
    a = H.Authority()
    model(a)
    reg(a, [b"h0", b"h1"], [meta(b"h0", node="n0"), meta(b"h1", node="n1")])
    assert a.plan_defrag("m", "", TARGET, COLOCATE, 64) == []


def test_colocate_avoids_occupied_slots():
    a = H.Authority()
    model(a)
    reg(a, [b"x"], [meta(b"x", seg=1, off=0)])
    reg(a, [b"h0", b"h1"], [meta(b"h0", seg=1, off=128), meta(b"h1", seg=2, off=0)])
    moves = a.plan_defrag("m", "", TARGET, COLOCATE, 64)
    assert moves
    taken = {(1, 0), (1, 128)}
    assert all((m.to_segment, m.to_offset) not in taken for m in moves)


def test_l2_fragmentation_ratio_counts_movable_segments():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b", b"c", b"d"],
        [meta(b"a", seg=1, off=0), meta(b"b", seg=1, off=100), meta(b"c", seg=2, off=0), meta(b"d", seg=2, off=200)])
    assert a.l2_fragmentation_ratio("m", "", TARGET, 100) == 0.5
    ref(a, b"c", 1)  # segment 2 is frozen: not counted
    assert a.l2_fragmentation_ratio("m", "", TARGET, 100) == 0.0


# ------------------------------------------------------------------ shard ring / hits / placement
def test_shard_membership_and_map():
    a = H.Authority()
    a.join_shard_node("n0", 16)
    a.join_shard_node("n1", 16)
    m = a.shard_map()
    assert len(m.nodes) == 2 and m.generation >= 2
    assert a.shard_owner(b"any-key") in ("n0", "n1")


def test_join_moves_a_bounded_subset():
    a = H.Authority()
    model(a)
    a.join_shard_node("n0", 32)
    a.join_shard_node("n1", 32)
    for i in range(80):
        h = f"b{i:03d}".encode()
        reg(a, [h], [meta(h)])
    migs, _ = a.join_shard_node("n2", 32)
    assert 0 < len(migs) < 80
    assert all(m.to_node == "n2" and m.from_node in ("n0", "n1") and not m.push_l2_first for m in migs)


def test_report_hits_feed_the_warmup_plan():
    a = H.Authority()
    model(a)
    reg(a, [b"hot", b"cold"], [meta(b"hot"), meta(b"cold")])
    a.report_hits("router-0", [bid(b"hot")] * 3 + [bid(b"cold"), bid(b"ghost")])
    assert (a.hit_count(bid(b"hot")), a.hit_count(bid(b"cold")), a.hit_count(bid(b"ghost"))) == (3, 1, 0)
    plan = a.warmup_plan("n1", 10)
    assert [p.block_hash for p in plan] == [b"hot", b"cold"]
    a.publish_location(bid(b"hot"), L0, "n0", 0, 0, True)
    assert [p.block_hash for p in a.warmup_plan("n0", 10)] == [b"cold"]


def test_follow_traffic_threshold_and_hysteresis():
    a = H.Authority()
    model(a)
    reg(a, [b"solo"], [meta(b"solo")])
    assert a.report_hits("n5", [bid(b"solo")]) == []
    assert a.hit_count_on(bid(b"solo"), "n5") == 1
    plans = a.report_hits("n5", [bid(b"solo")])
    assert len(plans) == 1 and plans[0].node_id == "n5" and [i.block_hash for i in plans[0].ids] == [b"solo"]
    assert a.report_hits("n5", [bid(b"solo")]) == []
    assert a.report_hits("n7", [bid(b"solo")]) == []
    assert len(a.report_hits("n7", [bid(b"solo")])) == 1
    assert a.hit_count(bid(b"solo")) == 5


def test_follow_traffic_colocates_ancestors_root_first():
    a = H.Authority()
    model(a)
    reg(a, [b"a", b"b", b"c"], [meta(b"a"), meta(b"b"), meta(b"c")])
    a.publish_location(bid(b"a"), L0, "n5", 0, 0, True)
    assert a.report_hits("n5", [bid(b"c")]) == []
    plans = a.report_hits("n5", [bid(b"c")])
    assert [i.block_hash for i in plans[0].ids] == [b"b", b"c"]


def test_follow_traffic_skips_blocks_already_in_l0():
    a = H.Authority()
    model(a)
    reg(a, [b"solo"], [meta(b"solo")])
    a.publish_location(bid(b"solo"), L0, "n5", 0, 0, True)
    for _ in range(3):
        assert a.report_hits("n5", [bid(b"solo")]) == []
    assert a.hit_count_on(bid(b"solo"), "n5") == 3


def test_l0_eviction_clears_the_placement_mark():
    a = H.Authority()
    model(a)
    reg(a, [b"solo"], [meta(b"solo")])
    assert a.report_hits("n5", [bid(b"solo")]) == []
    assert len(a.report_hits("n5", [bid(b"solo")])) == 1
    assert a.report_hits("n5", [bid(b"solo")]) == []
    a.publish_location(bid(b"solo"), L0, "n5", 0, 0, True)
    a.publish_location(bid(b"solo"), L0, "n5", 0, 0, False)
    plans = a.report_hits("n5", [bid(b"solo")])
    assert len(plans) == 1 and plans[0].node_id == "n5"
    assert a.report_hits("n5", [bid(b"solo")]) == []


def test_preplace_on_register_uses_the_hrw_home():
    a = H.Authority()
    model(a)
    full = [b"a", b"b"]
    assert a.preplace_on_register("m", "", TARGET, full) is None  # empty ring
    reg(a, full, [meta(b"a"), meta(b"b")])
    a.join_shard_node("n0", 16)
    plan = a.preplace_on_register("m", "", TARGET, full)
    assert plan.node_id == "n0" and [i.block_hash for i in plan.ids] == full
    assert a.preplace_on_register("m", "", TARGET, full) is None
    reg(a, [b"x"], [meta(b"x", l0=True)])
    assert a.preplace_on_register("m", "", TARGET, [b"x"]) is None


def test_drain_pushes_l2_first_then_remove():
    a = H.Authority()
    model(a)
    a.join_shard_node("n0", 16)
    a.join_shard_node("n1", 16)
    reg(a, [b"d0"], [meta(b"d0", node="n0")])
    migs, push = a.drain_shard_node("n0")
    assert [p.block_hash for p in push] == [b"d0"]
    assert any(m.push_l2_first and m.to_node == "n1" for m in migs)
    with pytest.raises(ValueError, match="placements remain"):
        a.remove_shard_node("n0")
    a.publish_location(bid(b"d0"), L2, "n0", 1, 0, False)
    a.publish_location(bid(b"d0"), L2, "n1", 1, 0, True)
    a.remove_shard_node("n0")
    assert a.ready_nodes() == ["n1"]


def test_drain_of_many_blocks_moves_ownership_and_remove_waits_for_the_copies():
    """rust/controlplane/src/lib.rs:3864-3907: every L2 block on the drained node is a push
    candidate, none is owned by it any more, and removal waits until its copies are gone."""
    a = H.Authority()
    model(a)
    a.join_shard_node("n0", 32)
    a.join_shard_node("n1", 32)
    names = [f"d{i:02}".encode() for i in range(20)]
    for n in names:
        reg(a, [n], [meta(n, node="n1")], node="n1")
    migs, push = a.drain_shard_node("n1")
    assert sorted(p.block_hash for p in push) == sorted(names)
    assert migs and all(m.from_node == "n1" and m.push_l2_first for m in migs)
    assert all(a.shard_owner(p.block_hash) != "n1" for p in push)
    with pytest.raises(ValueError, match="placements remain"):
        a.remove_shard_node("n1")
    for p in push:
        a.publish_location(p, L2, "n1", 1, 0, False)
    a.remove_shard_node("n1")
    assert a.ready_nodes() == ["n0"]


def test_remove_is_refused_while_an_l2_copy_remains_and_the_node_stays_draining():
    a = H.Authority()
    model(a)
    a.join_shard_node("n0", 16)
    a.join_shard_node("n1", 16)
    reg(a, [b"stuck"], [meta(b"stuck", node="n1")], node="n1")
    a.drain_shard_node("n1")
    with pytest.raises(ValueError, match="placements remain"):
        a.remove_shard_node("n1")
    assert a.ready_nodes() == ["n0"] and [(e.node_id, e.draining) for e in a.shard_map().nodes if e.node_id == "n1"] == [("n1", True)]


def test_drain_keeps_target_and_draft_identities_apart():
    a = H.Authority()
    model(a)
    a.join_shard_node("n0", 16)
    a.join_shard_node("n1", 16)
    reg(a, [b"same"], [meta(b"same", node="n1")], node="n1")
    reg(a, [b"same"], [meta(b"same", node="n1", pk=DRAFT)], node="n1")
    _, push = a.drain_shard_node("n1")
    assert sorted(p.pool_kind for p in push if p.block_hash == b"same") == [TARGET, DRAFT]
