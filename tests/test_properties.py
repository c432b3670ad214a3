"""Property tests (random operation sequences, hypothesis) of the C++ authority and tier engine,
in the spirit of the reference's vendored block-manager property tests
(rust/vendor/kvbm-logical/src/pools/block_proptest.rs):

* authority: ref counts never go below zero (an underflowing batch changes nothing), a block
  with a reference is never evicted, eviction frees at most what was asked, and a prefix lookup
  finds a contiguous run of registered blocks;
* tier engine: L2 never holds more than its cap, every written block stays durable and reads
  back its own bytes, and a pinned block never leaves L2;
* router priority queue: no request is lost (each one is started and finished, or cancelled),
  in flight never exceeds the slots, and a preempted request is requeued."""
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

from lake_b200 import _host as H  # noqa: E402

REQUEST, WRITEBACK = 1, 3
CHAINS = 4  # chains of up to 3 blocks; block j of chain c is named (c, j)


def _h(c, j):
    return H.sha256(f"{c}/{j}".encode())


def _bid(c, j):
    return H.KVBlockID("m", _h(c, j))


auth_ops = st.lists(st.one_of(
    st.tuples(st.just("register"), st.integers(0, CHAINS - 1), st.integers(1, 3)),
    st.tuples(st.just("ref"), st.integers(0, CHAINS - 1), st.integers(0, 2), st.sampled_from([REQUEST, WRITEBACK]),
              st.sampled_from([1, -1])),
    st.tuples(st.just("evict"), st.integers(1, 4)),
), max_size=40)


@settings(max_examples=60, deadline=None)
@given(auth_ops)
def test_authority_refs_eviction_and_lookup_invariants(ops):
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, 100))
    refs = {}  # (c, j, kind) -> count, the model of the ledger
    registered = set()
    for op in ops:
        if op[0] == "register":
            _, c, n = op
            chain = [_h(c, j) for j in range(n)]
            a.register_blocks("n0", chain, [H.BlockMeta(_bid(c, j), [H.Location(3, "n0", 1, 100 * j)])
                                            for j in range(n)])
            registered.update((c, j) for j in range(n))
        elif op[0] == "ref":
            _, c, j, kind, d = op
            if (c, j) not in registered:
                continue
            key = (c, j, kind)
            try:
                a.report_refs([H.RefDelta(_bid(c, j), kind, d, "n0")])
            except ValueError:
                assert refs.get(key, 0) + d < 0  # only an underflow is refused ...
            else:
                assert refs.get(key, 0) + d >= 0
                refs[key] = refs.get(key, 0) + d
        else:
            _, n = op
            held = {(c, j) for (c, j, _), v in refs.items() if v > 0}
            freed = a.evict_n("m", "", 1, n)
            assert 0 <= freed <= n
            for c, j in held:  # ... and a referenced block survives eviction
                assert a.locate([_bid(c, j)])[0].id.block_hash == _h(c, j)
            gone = {cj for cj in registered if not a.locate([_bid(*cj)])}
            assert len(gone) <= freed and not gone & held
            registered -= gone
            refs = {k: v for k, v in refs.items() if k[:2] not in gone}
        for (c, j, kind), v in refs.items():  # the ledger matches the model after every step
            if (c, j) in registered and a.locate([_bid(c, j)]):
                req, wb = a.refs_by_kind(_bid(c, j))
                assert (req if kind == REQUEST else wb) == v
    for c in range(CHAINS):
        chain = [_h(c, j) for j in range(3)]
        r = a.lookup_prefix("m", "", 1, chain, "n0")
        assert 0 <= r.hit_length <= 3
        assert [b.id.block_hash for b in r.blocks] == chain[:r.hit_length]  # a contiguous run from the root


tier_ops = st.lists(st.one_of(
    st.tuples(st.just("put"), st.integers(0, 11)),
    st.tuples(st.just("pin"), st.integers(0, 11)),
    st.tuples(st.just("unpin"), st.integers(0, 11)),
    st.tuples(st.just("promote"), st.integers(0, 11)),
    st.tuples(st.just("demote_l2"), st.integers(0, 11)),
), max_size=40)


@settings(max_examples=40, deadline=None)
@given(tier_ops)
def test_tier_engine_cap_durability_and_pin_invariants(tmp_path_factory, ops):
    import torch

    bb, caps = 64, (2, 4, 3)
    root = tmp_path_factory.mktemp("tiers")
    buf = torch.zeros(caps[1] * bb, dtype=torch.uint8)
    e = H.TierEngine(H.TierCaps(*caps), bb, buf.data_ptr(), str(root / "l2"), str(root / "l3"), "m")
    data = {i: (f"block-{i}-".encode() * bb)[:bb] for i in range(12)}
    written, pins = set(), {}
    pages = iter(range(10_000))
    for op, i in ops:
        h = _h(9, i)
        pinned_in_l2 = {j for j in written if pins.get(j) and e.is_l2_durable(_h(9, j))}
        try:
            if op == "put":
                e.put_durable_bytes(h, data[i])
                written.add(i)
            elif op == "pin":
                e.pin(h)
                pins[i] = pins.get(i, 0) + 1
            elif op == "unpin" and pins.get(i):
                e.unpin(h)
                pins[i] -= 1
            elif op == "promote" and i in written:
                e.promote_to_l0(h, lambda: next(pages))
            elif op == "demote_l2" and i in written:
                e.demote_l2_to_l3(h)
        except ValueError as err:  # refusals the engine documents: all pinned, L0 full of pinned
            assert "pinned" in str(err) or "no free L1 slot" in str(err), err
        assert e.l2_len() <= caps[2] and len(e.l2_order()) == e.l2_len()
        for j in written:
            hj = _h(9, j)
            assert e.has_durable_backing(hj)
            assert e.read_bytes(hj) == data[j]
        assert all(e.is_l2_durable(_h(9, j)) for j in pinned_in_l2)  # a pinned block stayed in L2
    assert e.corrupt_reads() == 0


pq_ops = st.lists(st.one_of(
    st.tuples(st.just("submit"), st.integers(0, 3), st.sampled_from(["m", "x"])),
    st.tuples(st.just("finish"), st.integers(0, 30), st.booleans()),
    st.tuples(st.just("cancel"), st.integers(0, 30)),
    st.tuples(st.just("start"),),
), max_size=60)


@settings(max_examples=80, deadline=None)
@given(st.integers(1, 3), pq_ops)
def test_priority_queue_loses_no_request_and_respects_its_slots(slots, ops):
    """Every submitted ticket ends started-and-finished or cancelled; in flight never exceeds
    the slots; a preempted ticket is requeued, not dropped (reference: go/router/pq.go no-shed)."""
    pq = H.PQScheduler(slots, 1.0)
    waiting, running, cancelled, done = set(), set(), set(), set()
    for op in ops:
        if op[0] == "submit":
            t, _ = pq.submit(op[1], op[2])
            waiting.add(t)
        elif op[0] == "start":
            for t in pq.start_eligible():
                assert t in waiting
                waiting.discard(t)
                running.add(t)
        elif op[0] == "finish" and running:
            t = sorted(running)[op[1] % len(running)]
            pq.finish(t, preempted=op[2])
            running.discard(t)
            if op[2] and t not in cancelled:
                waiting.add(t)  # a preempted request goes back to the queue
            else:
                done.add(t)
        elif op[0] == "cancel" and (waiting or running):
            pool = sorted(waiting | running)
            t = pool[op[1] % len(pool)]
            if pq.cancel(t):
                assert t in waiting
                waiting.discard(t)
                cancelled.add(t)
            else:
                assert t in running
                cancelled.add(t)  # abandoned: it is not requeued when it ends
        assert pq.in_flight() == len(running) <= slots
        assert pq.queue_len() == len(waiting)
    while waiting or running:  # drain: everything left starts and finishes
        for t in list(running):
            pq.finish(t, preempted=False)
            running.discard(t)
            done.add(t)
        for t in pq.start_eligible():
            waiting.discard(t)
            running.add(t)
        if not running and waiting:
            raise AssertionError(f"{len(waiting)} queued requests can never start")
