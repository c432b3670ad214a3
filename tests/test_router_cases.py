"""Router core (C++) and the router loop under the scenarios the reference's Go router tests
pin (go/router/pq_test.go:83-370, affinity_test.go:43-184, modeselect_test.go:16-140,
mirror_test.go:28-200, autoscale_test.go:30-405): priority order and FIFO within a priority,
preemption that requeues its victim, no preemption at equal priority or by a backpressured
model, no shedding under overload, backpressure that defers but never drops, the load
snapshot, cancellation; the affinity / rendezvous node choice (L0 preference, in-flight guard,
deterministic cold path equal to the pure HRW argmax, minimal migration when a node joins,
overflow past the guard); the three execution modes and the bandwidth gate; the view mirror's
snapshot, anchor, de-duplication, gap and prefix lookup; the autoscaler's sustain, cooldown,
bounds and streak reset; the router loop's mirror-first prefix hint with authority fallback,
hit reports with autoscale off, and a queue-driven scale-out that widens admission; and the HTTP
front (server_test.go:268-405): the body limit, generic error texts that leak no backend
detail, D-direct dispatch from a mirror hit, and a cold request with the authority down; the
view sync loop resuming after a gap and taking a fallback snapshot, and the load sync loop
uploading reports and applying the backpressure an ack carries (viewsync_test.go:85-200,
loadsync_test.go:82-140)."""
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


# ------------------------------------------------------------------ mode select (modeselect_test.go:16-75)
R = H.Role
PD, COLO, DD = H.ExecMode.PD_DISAGG, H.ExecMode.COLOCATED, H.ExecMode.D_DIRECT


def test_a_pool_hit_on_a_dedicated_role_goes_pd():
    hint = H.PrefixHint(16, 2, 0, False)
    assert H.select_exec_mode(hint, 16, R.PREFILL, 0) == PD
    assert H.select_exec_mode(hint, 16, R.DECODE, 0) == PD
    assert H.select_exec_mode(hint, 16, R.PREFILL, 10) == PD  # the path is fast enough to move KV


def test_the_bandwidth_gate_recomputes_a_pool_hit_on_a_slow_path():
    hint = H.PrefixHint(16, 2, 0, False)
    assert H.TRANSFER_BW_THRESHOLD_GBPS == 1.0
    assert H.select_exec_mode(hint, 16, R.PREFILL, 0.5) == COLO
    assert H.select_exec_mode(hint, 16, R.DECODE, 0.99) == COLO
    # a local hit needs no transfer: the gate does not apply
    assert H.select_exec_mode(H.PrefixHint(8, 1, 1, True), 16, R.HYBRID, 0.3) == DD
    # a miss has nothing to move: the role decides
    assert H.select_exec_mode(H.PrefixHint(), 16, R.PREFILL, 0.3) == PD


def test_a_local_hit_goes_d_direct_on_every_role():
    for role in (R.HYBRID, R.PREFILL, R.DECODE):
        assert H.select_exec_mode(H.PrefixHint(8, 1, 1, True), 16, role, 0) == DD


def test_hybrid_workers_colocate_misses_and_pool_hits():
    assert H.select_exec_mode(H.PrefixHint(), 8, R.HYBRID, 0) == COLO
    assert H.select_exec_mode(H.PrefixHint(8, 1, 0, False), 16, R.HYBRID, 0) == COLO
    assert H.select_exec_mode(H.PrefixHint(0, 0, 0, True), 0, R.HYBRID, 0) == COLO  # empty prompt


# ------------------------------------------------------------------ view mirror (mirror_test.go:28-200)
REGISTERED, INVALIDATED, MOVED = 0, 1, 2


def _event(kind, hsh, nodes=(), pool_kind=1, block_kind=0):
    e = H.ViewEvent()
    e.kind = kind
    e.id = H.KVBlockID("m", hsh, pool_kind)
    e.locations = [H.Location(1, n, 1, 0) for n in nodes]
    e.l3_present = True
    e.block_kind = block_kind
    return e


def _update(seq, events=()):
    u = H.ViewUpdate()
    u.seq = seq
    u.events = list(events)
    return u


def _local(m, hsh, node, pool_kind=1):
    got = m.prefix_lookup("m", "", pool_kind, [hsh], node)
    return None if not got else got[0].local_hit


def test_mirror_snapshot_anchor_increment_dedupe_and_invalidation():
    m = H.ViewMirror()
    assert m.apply(_update(0, [_event(REGISTERED, b"h0"), _event(REGISTERED, b"h1", ["n0"])])) == 0
    assert m.apply(_update(3)) == 0 and m.last_seq() == 3  # an anchor moves the sequence only
    assert m.apply(_update(4, [_event(MOVED, b"h1", ["n1"])])) == 0
    assert _local(m, b"h1", "n1") is True and _local(m, b"h1", "n0") is False
    assert m.apply(_update(2, [_event(REGISTERED, b"h9")])) == 0  # seq <= last: dropped
    assert _local(m, b"h9", "") is None
    assert m.apply(_update(5, [_event(INVALIDATED, b"h0")])) == 0
    assert _local(m, b"h0", "") is None and m.size() == 1


def test_a_snapshot_resets_the_sequence_after_a_control_plane_restart():
    m = H.ViewMirror()
    m.apply(_update(0, [_event(REGISTERED, b"old")]))
    m.apply(_update(100))
    assert m.last_seq() == 100
    m.apply(_update(0, [_event(REGISTERED, b"new")]))  # the restarted authority counts from 1 again
    assert m.last_seq() == 0 and _local(m, b"old", "") is None
    m.apply(_update(1))
    assert m.apply(_update(2, [_event(REGISTERED, b"h2")])) == 0
    assert _local(m, b"h2", "") is False and m.last_seq() == 2


def test_a_gap_is_reported_and_changes_nothing():
    m = H.ViewMirror()
    m.apply(_update(0, [_event(REGISTERED, b"h0")]))
    m.apply(_update(1))
    assert m.apply(_update(3, [_event(REGISTERED, b"h1")])) == 2  # wants seq 2
    assert m.last_seq() == 1 and _local(m, b"h1", "") is None


def test_mirror_prefix_lookup_is_contiguous_per_requester_and_per_pool():
    m = H.ViewMirror()
    m.apply(_update(0, [_event(REGISTERED, b"h0", ["n0"]), _event(REGISTERED, b"h1"),
                        _event(REGISTERED, b"h2", ["n1"])]))
    got = m.prefix_lookup("m", "", 1, [b"h0", b"h1", b"h2"], "n0")
    assert [b.local_hit for b in got] == [True, False, False]  # all three found, only h0 on n0
    assert m.prefix_lookup("m", "", 1, [b"hx", b"h0"], "n0") == []  # the first miss ends the match
    assert m.prefix_lookup("m", "", 2, [b"h0"], "n0") == []  # the draft pool is its own namespace


# ------------------------------------------------------------------ autoscaler (autoscale_test.go:30-80)
def _scaler():
    return H.Autoscaler(H.AutoscaleConfig(1, 3, 4, 0, 3, 60.0))  # min, max, out at 4, in at 0, 3 periods, 60 s


def test_autoscale_decisions_sustain_cooldown_bounds_and_streak_reset():
    NONE, OUT, IN = H.ScaleDecision.NONE, H.ScaleDecision.SCALE_OUT, H.ScaleDecision.SCALE_IN
    a = _scaler()
    assert [a.evaluate(0, 5, 1, 1) for _ in range(3)] == [NONE, NONE, OUT]  # three hot periods
    assert a.evaluate(10, 5, 1, 2) == NONE  # cooldown
    assert a.evaluate(120, 5, 1, 3) == NONE  # at max nodes
    b = _scaler()
    b.evaluate(0, 5, 1, 1)
    b.evaluate(0, 2, 1, 1)  # a middle value resets the streak
    b.evaluate(0, 5, 1, 1)
    assert b.evaluate(0, 5, 1, 1) == NONE
    c = _scaler()
    assert [c.evaluate(0, 0, 0, 2) for _ in range(3)] == [NONE, NONE, IN]  # three idle periods
    assert all(c.evaluate(120 * (i + 1), 0, 0, 1) == NONE for i in range(5))  # never below min nodes


def test_node_registry_ids_grow_and_the_newest_ready_node_drains_first():
    n = H.NodeRegistry(["worker-0"])
    assert n.next_id() == "worker-1"
    n.add("worker-1")
    assert n.next_id() == "worker-2" and n.last_ready() == "worker-1"
    assert n.mark_draining("worker-1") and n.count() == 1 and n.draining() == ["worker-1"]
    assert n.ready_ids() == ["worker-0"]  # a draining node takes no new request
    n.unmark_draining("worker-1")
    assert n.count() == 2 and n.draining() == []


# ------------------------------------------------------------------ router loop (modeselect_test.go:77-140, autoscale_test.go:183-405)
class _FakeCP:
    """The control-plane calls the router makes, recorded; LookupPrefix answers from `lookup`."""

    def __init__(self, lookup=None):
        from lake_b200.api import proto

        self.pb = proto.messages()
        self.lookup, self.calls, self.hits = lookup, [], []

    async def LookupPrefix(self, req, timeout=None):
        self.calls.append("lookup")
        if self.lookup is None:
            raise AssertionError("the control plane was asked")
        return self.lookup(req)

    async def ReportHits(self, req, timeout=None):
        self.hits.append((req.node_id, [bytes(i.block_hash) for i in req.ids]))
        return self.pb.Ack(ok=True)

    async def JoinShardNode(self, req, timeout=None):
        self.calls.append(("join", req.node_id))
        return self.pb.JoinShardNodeResponse(ok=True)


class _FakeAgent:
    def __init__(self):
        self.placed = 0

    async def PlaceBlocks(self, req, timeout=None):
        self.placed += 1


def _router(cp, agent=None, **cfg):
    from lake_b200.router.server import Router, RouterConfig

    class R(Router):
        pass

    R.cp = property(lambda self: cp)
    R.agent = property(lambda self: agent)
    return R(RouterConfig(workers={"worker-0": "127.0.0.1:1"}, **cfg))


def _prompt_hashes(r, n_blocks=2):
    from lake_b200.engine.block_pool import chain_block_hashes

    tokens = list(range(1, n_blocks * r.cfg.block_size + 1))
    return tokens, chain_block_hashes(tokens, r.cfg.block_size, full_only=True)


def test_a_mirror_hit_makes_the_hint_without_a_control_plane_call():
    import asyncio

    cp = _FakeCP()
    r = _router(cp)
    tokens, hs = _prompt_hashes(r)
    r.mirror.apply(_update(0, [_event(REGISTERED, hs[0], ["worker-0"])]))
    hint = asyncio.run(r.prefix_hint("m", hs, len(tokens), "worker-0"))
    assert (hint.reused_blocks, hint.computed_tokens, hint.local_hit) == (1, r.cfg.block_size, True)
    hint = asyncio.run(r.prefix_hint("m", hs, len(tokens), "worker-1"))
    assert (hint.reused_blocks, hint.local_hit) == (1, False)  # the same block, held elsewhere: a pool hit
    assert cp.calls == []


def test_a_mirror_miss_falls_back_to_the_authority_and_a_double_miss_is_cold():
    import asyncio

    def answer(req):
        return cp.pb.LookupPrefixResponse(hit_length=1, blocks=[cp.pb.ReusableBlock(
            id=cp.pb.KVBlockID(model_id=req.model_id, block_hash=req.prefix_hashes[0]))])

    cp = _FakeCP(answer)
    r = _router(cp)
    tokens, hs = _prompt_hashes(r)
    hint = asyncio.run(r.prefix_hint("m", hs, len(tokens), "worker-0"))
    assert cp.calls == ["lookup"]
    assert (hint.reused_blocks, hint.computed_tokens, hint.local_hit) == (1, r.cfg.block_size, False)
    cold = _FakeCP(lambda req: cold.pb.LookupPrefixResponse())
    hint = asyncio.run(_router(cold).prefix_hint("m", hs, len(tokens), "worker-0"))
    assert (hint.reused_blocks, hint.computed_tokens, hint.local_hit) == (0, 0, False)


def test_the_tick_reports_hits_with_autoscale_off():
    import asyncio

    cp = _FakeCP()
    r = _router(cp, autoscale=False)
    tokens, hs = _prompt_hashes(r)
    r.mirror.apply(_update(0, [_event(REGISTERED, hs[0], ["worker-0"])]))
    asyncio.run(r.prefix_hint("m", hs, len(tokens), "worker-0"))
    asyncio.run(r.autoscale_tick())
    assert cp.hits == [("worker-0", [hs[0]])]
    assert not any(isinstance(c, tuple) for c in cp.calls)  # no scaling with autoscale off


def test_queue_depth_drives_a_scale_out_that_widens_admission_and_places_nothing():
    import asyncio

    cp, agent = _FakeCP(), _FakeAgent()
    r = _router(cp, agent, autoscale=True, max_inflight=1)
    r.scaler = H.Autoscaler(H.AutoscaleConfig(1, 3, 2, 0, 1, 0.0))
    r.pq = H.PQScheduler(1, 1.0)
    for _ in range(3):
        r.pq.submit(0, "m")
    r.pq.start_eligible()
    assert (r.pq.in_flight(), r.pq.queue_len()) == (1, 2)
    tokens, hs = _prompt_hashes(r)
    r.mirror.apply(_update(0, [_event(REGISTERED, hs[0], ["worker-0"])]))
    asyncio.run(r.prefix_hint("m", hs, len(tokens), "worker-0"))
    asyncio.run(r.autoscale_tick())
    assert cp.calls == [("join", "worker-1")] and r.nodes.count() == 2
    assert r.pq.load_snapshot("r").remaining_cap == 1  # two per-node slots, one in use
    assert len(r.pq.start_eligible()) == 1
    assert cp.hits == [("worker-0", [hs[0]])] and agent.placed == 0  # hits go to the pool side


# ------------------------------------------------------------------ HTTP front (server_test.go:268-405)
class _Call:
    """A finished unary call the router can await and cancel."""

    def __init__(self, resp):
        self.resp, self._cancelled = resp, False

    def __await__(self):
        return self.resp
        yield  # noqa: unreachable (makes this a generator)

    def cancel(self):
        self._cancelled = True

    def cancelled(self):
        return self._cancelled


def _rpc_error(code, details):
    import grpc

    return grpc.aio.AioRpcError(code, grpc.aio.Metadata(), grpc.aio.Metadata(), details=details)


class _DownCP(_FakeCP):
    async def LookupPrefix(self, req, timeout=None):
        import grpc

        raise _rpc_error(grpc.StatusCode.UNAVAILABLE, "control plane down")


def _http(dispatch, cp=None):
    """A router app whose agent answers Dispatch with `dispatch(pb, req)` and whose worker
    answers Generate with one token in the requested mode."""
    from lake_b200.api import proto
    from lake_b200.router.http import make_app
    from lake_b200.router.server import Router, RouterConfig

    pb = proto.messages()
    seen = {}

    class Agent:
        async def Dispatch(self, req, timeout=None):
            seen["dispatch"] = req
            return dispatch(pb, req)

    class Worker:
        def Generate(self, req, timeout=None):
            seen["generate"] = req
            return _Call(pb.GenerateResponse(request_id=req.request_id, mode=req.exec_mode, output_tokens=[5]))

    class R(Router):
        agent = property(lambda self: Agent())

        def worker(self, node):
            return Worker()

    R.cp = property(lambda self: cp or _DownCP())
    r = R(RouterConfig(workers={"worker-0": "127.0.0.1:1"}, request_timeout_s=5))
    return r, make_app(r), seen


def _post(app, **kw):
    import asyncio

    from aiohttp.test_utils import TestClient, TestServer

    async def run():
        async with TestClient(TestServer(app)) as c:
            resp = await c.post("/v1/chat/completions", **kw)
            return resp.status, await resp.text()

    return asyncio.run(run())


def _ok(pb, req):
    return pb.Ack(ok=True)


CHAT = {"model": "m", "messages": [{"role": "user", "content": "hi"}]}


def test_a_body_over_the_limit_is_413():
    from lake_b200.router.server import MAX_BODY

    _, app, _ = _http(_ok)
    assert _post(app, data=b"x" * (MAX_BODY + 1))[0] == 413


def test_invalid_json_gets_a_generic_message():
    _, app, _ = _http(_ok)
    status, text = _post(app, data=b"{")
    assert status == 400 and text == "invalid JSON request"  # no parser detail


def test_an_upstream_error_does_not_leak_its_message():
    import grpc

    def down(pb, req):
        raise _rpc_error(grpc.StatusCode.UNAVAILABLE, "secret backend details")

    _, app, _ = _http(down)
    status, text = _post(app, json=CHAT)
    assert status == 503 and "secret" not in text


def test_a_rejected_dispatch_does_not_leak_its_reason():
    _, app, _ = _http(lambda pb, req: pb.Ack(ok=False, err="secret quota details"))
    status, text = _post(app, json=CHAT)
    assert status == 502 and "secret" not in text


def test_a_mirror_hit_dispatches_d_direct_with_the_hint():
    import json

    r, app, seen = _http(_ok)
    prompt = list(range(100, 100 + 2 * r.cfg.block_size))
    hs = H.chain_block_hashes(prompt, r.cfg.block_size, True)
    r.mirror.apply(_update(0, [_event(REGISTERED, hs[0], ["worker-0"])]))
    status, text = _post(app, json={"model": "m", "prompt_token_ids": prompt, "max_tokens": 1})
    assert status == 200 and json.loads(text)["lake"]["mode"] == "D_DIRECT"
    assert seen["dispatch"].mode == "D_DIRECT"
    g = seen["generate"]
    assert (g.exec_mode, g.local_hit, g.reused_blocks, g.computed_tokens) == ("D_DIRECT", True, 1, r.cfg.block_size)


def test_a_cold_miss_with_the_authority_down_runs_colocated_without_reuse():
    import json

    r, app, seen = _http(_ok)
    status, text = _post(app, json={"model": "m", "prompt_token_ids": list(range(1, 40)), "max_tokens": 1})
    assert status == 200 and json.loads(text)["lake"]["mode"] == "COLOCATED"
    g = seen["generate"]
    assert (g.exec_mode, g.reused_blocks, g.computed_tokens, g.local_hit) == ("COLOCATED", 0, 0, False)


# ------------------------------------------------------------------ view / load sync loops (viewsync_test.go:85-200, loadsync_test.go:82-140)
class _Stream:
    """A server stream: yields `items` (raising an item that is an exception), then either ends
    with `end` raised or stays open until cancelled."""

    def __init__(self, items, end=None):
        self.items, self.end, self.cancelled = items, end, False

    def cancel(self):
        self.cancelled = True

    def __aiter__(self):
        return self._gen()

    async def _gen(self):
        import asyncio

        for it in self.items:
            if self.cancelled:
                return
            yield it
        if self.end is not None:
            raise self.end
        while not self.cancelled:
            await asyncio.sleep(0.001)


def _pb_update(pb, seq, regs=(), moved=()):
    ev = [pb.ViewEvent(kind=0, id=pb.KVBlockID(model_id="m", block_hash=h, pool_kind=1), l3_present=True)
          for h in regs]
    ev += [pb.ViewEvent(kind=2, id=pb.KVBlockID(model_id="m", block_hash=h, pool_kind=1),
                        locations=[pb.Location(tier=1, node_id=n, segment_id=1)]) for h, n in moved]
    return pb.ViewUpdate(seq=seq, events=ev)


def _run_view_sync(script):
    """Runs the router's view sync against a control plane answering SubscribeView call k with
    script(pb, k); returns the router and the resume sequence of each call."""
    import asyncio

    from lake_b200.api import proto

    pb = proto.messages()
    resumes = []

    class CP(_FakeCP):
        def SubscribeView(self, req, timeout=None):
            resumes.append(req.resume_from_seq)
            return script(pb, len(resumes) - 1)

    r = _router(CP())

    async def run(want_seq):
        t = asyncio.create_task(r._view_sync(reconnect_s=0.001))
        for _ in range(3000):
            if r.mirror.last_seq() == want_seq and len(resumes) >= 2:
                break
            await asyncio.sleep(0.001)
        t.cancel()
        try:
            await t
        except asyncio.CancelledError:
            pass

    return r, resumes, run


def test_view_sync_resumes_after_a_gap_and_replays_to_alignment():
    import asyncio
    import grpc

    def script(pb, k):
        if k == 0:  # snapshot, anchor 1, then seq 3: seq 2 was missed
            return _Stream([_pb_update(pb, 0, regs=[b"h0"]), _pb_update(pb, 1), _pb_update(pb, 3, regs=[b"h1"])],
                           end=_rpc_error(grpc.StatusCode.UNAVAILABLE, "drop"))
        assert k == 1
        return _Stream([_pb_update(pb, 2, moved=[(b"h0", "n0")]), _pb_update(pb, 3, regs=[b"h1"])])

    r, resumes, run = _run_view_sync(script)
    asyncio.run(run(3))
    assert r.mirror.last_seq() == 3 and resumes == [0, 1]
    assert _local(r.mirror, b"h0", "n0") is True and _local(r.mirror, b"h1", "") is False


def test_view_sync_takes_the_snapshot_a_control_plane_falls_back_to():
    import asyncio
    import grpc

    def script(pb, k):
        if k == 0:
            return _Stream([_pb_update(pb, 0, regs=[b"h0", b"h1"]), _pb_update(pb, 1)],
                           end=_rpc_error(grpc.StatusCode.UNAVAILABLE, "drop"))
        return _Stream([_pb_update(pb, 0, regs=[b"h1"]), _pb_update(pb, 5)])  # resume point evicted

    r, resumes, run = _run_view_sync(script)
    asyncio.run(run(5))
    assert r.mirror.last_seq() == 5 and resumes == [0, 1]
    assert _local(r.mirror, b"h0", "") is None and _local(r.mirror, b"h1", "") is False


def test_load_sync_uploads_reports_and_applies_backpressure_from_the_ack():
    import asyncio

    from lake_b200.api import proto

    pb = proto.messages()
    sent, bp_on = [], []

    class Bidi:
        def __init__(self):
            self.q = asyncio.Queue()

        async def write(self, rep):
            sent.append(rep)
            sig = pb.BackpressureSignal(model_id="m-bp", reason="HARD_QUOTA", deficit_bytes=64) if bp_on else None
            await self.q.put(pb.Ack(ok=True, backpressure=sig) if sig else pb.Ack(ok=True))

        def cancel(self):
            self.q.put_nowait(None)

        def __aiter__(self):
            return self

        async def __anext__(self):
            item = await self.q.get()
            if item is None:
                raise StopAsyncIteration
            return item

    class Agent:
        def ReportLoad(self):
            return Bidi()

    r = _router(_FakeCP(), Agent())
    r.pq = H.PQScheduler(1, 5.0)

    async def run():
        t = asyncio.create_task(r._load_sync(interval_s=0.001))
        for _ in range(2000):
            if sent:
                break
            await asyncio.sleep(0.001)
        assert sent and sent[0].node_id == "router"
        bp_on.append(True)
        for _ in range(2000):
            if r.pq.backpressured("m-bp"):
                break
            await asyncio.sleep(0.001)
        t.cancel()
        try:
            await t
        except asyncio.CancelledError:
            pass

    asyncio.run(run())
    assert r.pq.backpressured("m-bp") and not r.pq.backpressured("other")
    bp, _ = r.pq.submit(5, "m-bp")
    other, _ = r.pq.submit(5, "other")
    assert r.pq.start_eligible() == [other]  # the backpressured model waits, the other one runs
    assert r.pq.queue_len() == 1
