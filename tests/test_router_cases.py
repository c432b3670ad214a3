"""Router core (C++) under the scenarios the reference's Go router tests pin
(go/router/pq_test.go:83-370, affinity_test.go:43-184): priority order and FIFO within a
priority, preemption that requeues its victim, no preemption at equal priority or by a
backpressured model, no shedding under overload, backpressure that defers but never drops,
the load snapshot, cancellation, and the affinity / rendezvous node choice (L0 preference,
in-flight guard, deterministic cold path equal to the pure HRW argmax, minimal migration when
a node joins, overflow past the guard)."""
import random
import time

from lake_b200 import _host as H


# ------------------------------------------------------------------ priority queue
class Driver:
    """Runs the queue like the router's loop: start what is eligible, finish on request."""

    def __init__(self, max_inflight, ttl=1.0):
        self.pq = H.PQScheduler(max_inflight, ttl)
        self.order, self.names = [], {}

    def submit(self, prio, model, name):
        t, pre = self.pq.submit(prio, model)
        self.names[t] = name
        return t, pre

    def pump(self):
        started = self.pq.start_eligible()
        self.order += [self.names[t] for t in started]
        return started


def test_priority_order_then_fifo_within_a_priority():
    d = Driver(1)
    first, _ = d.submit(10, "m", "first")
    assert d.pump() == [first]
    d.submit(5, "m", "mid")
    d.submit(1, "m", "low")
    d.submit(5, "m", "mid2")
    assert d.pq.queue_len() == 3
    running = first
    while True:
        d.pq.finish(running)
        started = d.pump()
        if not started:
            break
        running = started[0]
    assert d.order == ["first", "mid", "mid2", "low"]


def test_preemption_requeues_the_victim_which_reruns():
    d = Driver(1)
    low, _ = d.submit(1, "m", "low")
    d.pump()
    high, pre = d.submit(10, "m", "high")
    assert pre == low  # the higher priority outranks the only running request
    d.pq.finish(low, preempted=True)  # the victim goes back to the queue, not away
    assert d.pump() == [high]
    d.pq.finish(high)
    assert d.pump() == [low]
    d.pq.finish(low)
    assert d.order == ["low", "high", "low"] and d.pq.queue_len() == 0 and d.pq.in_flight() == 0


def test_no_preemption_at_equal_priority():
    d = Driver(1)
    d.submit(5, "m", "first")
    d.pump()
    _, pre = d.submit(5, "m", "second")
    assert pre is None and d.pump() == []


def test_no_shedding_under_overload():
    d = Driver(2)
    tickets = [d.submit(i % 3, "m", f"r{i}")[0] for i in range(20)]
    done = set()
    running = d.pump()
    while running:
        t = running.pop(0)
        d.pq.finish(t)
        done.add(t)
        running += d.pump()
    assert done == set(tickets)  # every request ran: nothing rejected or dropped


def test_backpressure_defers_a_model_without_dropping_it():
    d = Driver(1, ttl=0.1)
    d.pq.set_backpressure("m")
    m, _ = d.submit(5, "m", "m")
    x, _ = d.submit(5, "x", "x")
    assert d.pump() == [x]  # the other model starts; m is skipped, not dropped
    d.pq.finish(x)
    assert d.pump() == [] and d.pq.queue_len() == 1
    assert 0.0 < d.pq.next_backpressure_expiry_s() <= 0.1
    time.sleep(0.12)
    assert d.pump() == [m]
    assert d.order == ["x", "m"]


def test_a_backpressured_model_does_not_preempt():
    d = Driver(1, ttl=0.15)
    low, _ = d.submit(1, "x", "low")
    d.pump()
    d.pq.set_backpressure("m")
    high, pre = d.submit(10, "m", "high")
    assert pre is None  # it could not start anyway: the running request keeps its slot
    d.pq.finish(low)
    assert d.pump() == []
    time.sleep(0.17)
    assert d.pump() == [high]


def test_load_snapshot_counts_running_queued_and_capacity():
    d = Driver(1)
    d.submit(10, "m", "a")
    d.pump()
    d.submit(1, "m", "b")
    d.submit(1, "m", "c")
    s = d.pq.load_snapshot("router")
    assert (s.node_id, s.in_flight, s.queue_len, s.remaining_cap) == ("router", 1, 2, 0)


def test_cancel_dequeues_a_waiting_request_and_abandons_a_running_one():
    d = Driver(1)
    a, _ = d.submit(1, "m", "runner")
    d.pump()
    q, _ = d.submit(1, "m", "quitter")
    assert d.pq.cancel(q) and d.pq.queue_len() == 0  # waiting: removed
    assert not d.pq.cancel(q)  # already gone
    assert not d.pq.cancel(a)  # running: not dequeued, marked abandoned
    _, pre = d.submit(10, "m", "high")
    assert pre is None  # an abandoned request is no preemption victim (its slot frees anyway)
    d.pq.finish(a, preempted=True)  # and it is not requeued
    assert d.pq.in_flight() == 0 and d.pq.queue_len() == 1
    assert [d.names[t] for t in d.pump()] == ["high"]


# ------------------------------------------------------------------ affinity / HRW
def _mirror_with_l0(blocks):
    """blocks: [(hash, [nodes holding an L0 copy])] registered through an authority snapshot."""
    a = H.Authority()
    a.register_model(H.ModelDescriptor("m", "", 2, 16, 100))
    prefix = []
    for hsh, nodes in blocks:
        prefix.append(hsh)
        a.register_blocks(nodes[0], list(prefix), [H.BlockMeta(H.KVBlockID("m", hsh), [H.Location(1, n) for n in nodes])])
    m = H.ViewMirror()
    assert m.apply(a.snapshot()) == 0
    return m


NODES = ["worker-0", "worker-1", "worker-2"]


def test_affinity_prefers_the_node_holding_the_longest_l0_prefix():
    h0, h1, h2 = H.sha256(b"h0"), H.sha256(b"h1"), H.sha256(b"h2")
    m = _mirror_with_l0([(h0, ["worker-1", "worker-2"]), (h1, ["worker-1"]), (h2, ["worker-1"])])
    assert H.pick_node(H.NodeRegistry(NODES), m, "m", [h0, h1, h2], b"key-x", 4) == "worker-1"


def test_guard_downgrades_an_overloaded_node_then_falls_to_the_cold_path():
    h0, h1 = H.sha256(b"h0"), H.sha256(b"h1")
    m = _mirror_with_l0([(h0, ["worker-1", "worker-2"]), (h1, ["worker-1"])])
    nodes = H.NodeRegistry(NODES)
    for _ in range(4):
        nodes.inc_inflight("worker-1")
    assert H.pick_node(nodes, m, "m", [h0, h1], b"key-x", 4) == "worker-2"  # next best prefix
    for _ in range(4):
        nodes.inc_inflight("worker-2")
    # both holders over the guard: the cold path, over the nodes still under it
    assert H.pick_node(nodes, m, "m", [h0, h1], b"key-x", 4) == "worker-0"


def test_cold_path_is_deterministic_and_spreads():
    nodes = H.NodeRegistry(NODES)
    for i in range(8):
        key = f"key-{i}".encode()
        first = H.pick_node(nodes, None, "m", [], key, 4)
        assert all(H.pick_node(nodes, None, "m", [], key, 4) == first for _ in range(4))
    assert len({H.pick_node(nodes, None, "m", [], f"spread-{i}".encode(), 4) for i in range(64)}) >= 2


def test_cold_path_equals_the_pure_hrw_argmax():
    nodes = H.NodeRegistry(NODES)
    for i in range(64):
        key = f"conv-{i}".encode()
        want = max(NODES, key=lambda n: (H.hrw_score(key, n), [-ord(c) for c in n]))  # ties: smaller id
        assert H.pick_node(nodes, None, "m", [], key, 4) == want


def test_a_joining_node_moves_about_a_quarter_of_the_keys():
    nodes = H.NodeRegistry(NODES)
    rnd = random.Random(7)
    keys = [bytes([i & 255, (i >> 8) & 255, rnd.randrange(256)]) for i in range(2000)]
    before = {k: H.pick_node(nodes, None, "m", [], k, 4) for k in keys}
    nodes.add("worker-3")
    moved = sum(H.pick_node(nodes, None, "m", [], k, 4) != v for k, v in before.items())
    assert 0 < moved <= len(keys) * 35 // 100  # rendezvous hashing: ~1/4 move, to the new node
    assert all(H.pick_node(nodes, None, "m", [], k, 4) in (v, "worker-3") for k, v in before.items())


def test_cold_path_overflows_past_the_guard_and_returns_home_when_all_are_full():
    nodes = H.NodeRegistry(NODES)
    key = b"overflow-key"
    home = H.pick_node(nodes, None, "m", [], key, 4)
    for _ in range(4):
        nodes.inc_inflight(home)
    second = H.pick_node(nodes, None, "m", [], key, 4)
    assert second != home and H.pick_node(nodes, None, "m", [], key, 4) == second
    for n in NODES:
        while nodes.inflight(n) < 4:
            nodes.inc_inflight(n)
    assert H.pick_node(nodes, None, "m", [], key, 4) == home
