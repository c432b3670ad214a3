"""Engine <-> storage-pool contract: the step fences every agent shares (one open step,
paired done, finishes held while a step is open), PoolIface's handle validation and error
wrapping, and an engine whose steps run through the production in-process agent
(NativeAgent: L1/L2 tiers, PutEnd, authority). Modelled on the behaviours of the reference's
python/lake/engine/tests/test_pool_agent.py and test_executor.py."""
import pytest

from lake_b200.pool.agents.fences import StepFences
from lake_b200.pool.pool_iface import PoolIface
from lake_b200.pool.types import (FinishRequest, ForwardMode, PoolError, PoolErrorCode, PreparePlan, ReadyHandle,
                                  ReqIoSet)


def plan(step, writes=(("a", 0, 16),)):
    ws = [ReqIoSet(r, s, e) for r, s, e in writes]
    return PreparePlan(step, ForwardMode.EXTEND, [], ws, {io.req_id: io.token_end - io.token_start for io in ws},
                       0, False)


class _Recorder(StepFences):
    def __init__(self):
        super().__init__()
        self.finished = []

    def prepare_step(self, p):
        self._open(p.step_id)
        return ReadyHandle(p.step_id)

    def _finish(self, f):
        self.finished.append(f.req_id)


def test_step_fences_are_strictly_paired():
    ag = _Recorder()
    assert ag.prepare_step(plan(1)).step_id == 1
    with pytest.raises(PoolError) as e:
        ag.prepare_step(plan(2))
    assert e.value.code == PoolErrorCode.PROTOCOL_ERROR
    with pytest.raises(PoolError):
        ag.done(7)
    ag.done(1)
    with pytest.raises(PoolError):
        ag.done(1)  # nothing open
    ag.prepare_step(plan(2))
    ag.done(2)
    assert ag.fence_stats["steps"] == 2


def test_finishes_inside_an_open_step_run_at_done_in_order():
    ag = _Recorder()
    ag.on_request_finished(FinishRequest("x", "n0"))  # no open step: runs now
    ag.prepare_step(plan(1))
    ag.on_request_finished(FinishRequest("a", "n0"))
    ag.on_request_finished(FinishRequest("b", "n0"))
    assert ag.finished == ["x"]
    ag.done(1)
    assert ag.finished == ["x", "a", "b"] and ag.fence_stats["held_finishes"] == 2


class _Agent:
    """Scripted agent for PoolIface validation."""

    def __init__(self, handle=None, exc=None):
        self.handle, self.exc, self.finished, self.dones = handle, exc, [], []

    def prepare_step(self, p):
        if self.exc:
            raise self.exc
        return self.handle(p)

    def done(self, step_id):
        self.dones.append(step_id)

    def on_request_finished(self, f):
        self.finished.append(f.req_id)

    def commit_write_extent(self, req_id, token_end):
        pass


class _Out:
    def __init__(self, step_id, chunks):
        self.step_id, self.chunks, self.decode, self.prefill = step_id, chunks, [], chunks


class _Ch:
    def __init__(self, rid, start, n):
        self.req = type("R", (), {"rid": rid})()
        self.start, self.n = start, n


def test_pool_iface_validates_handles_and_wraps_errors():
    out = _Out(5, [_Ch("a", 0, 16), _Ch("b", 32, 1)])
    ok = PoolIface(_Agent(lambda p: ReadyHandle(p.step_id)))
    assert ok.prepare_step(out).step_id == 5
    bad_step = PoolIface(_Agent(lambda p: ReadyHandle(p.step_id + 1)))
    with pytest.raises(PoolError) as e:
        bad_step.prepare_step(out)
    assert e.value.code == PoolErrorCode.PROTOCOL_ERROR

    def shrink(p):
        return ReadyHandle(p.step_id, effective_write_set=[ReqIoSet("a", 0, 16)])

    with pytest.raises(PoolError, match="allow_partial_hit"):
        PoolIface(_Agent(shrink)).prepare_step(out)
    assert PoolIface(_Agent(shrink), allow_partial_hit=True).prepare_step(out).step_id == 5
    with pytest.raises(PoolError, match="unplanned"):
        PoolIface(_Agent(lambda p: ReadyHandle(p.step_id, effective_read_set=[ReqIoSet("zz", 0, 1)]))).prepare_step(out)
    boom = PoolIface(_Agent(exc=KeyError("x")))
    with pytest.raises(PoolError) as e:
        boom.prepare_step(out)
    assert e.value.code == PoolErrorCode.DOWNSTREAM and boom.stats.errors == 1
    # finish is idempotent
    req = type("R", (), {"rid": "a"})()
    ok.on_request_finished(req)
    ok.on_request_finished(req)
    assert ok.agent.finished == ["a"] and ok.stats.duplicate_finish_calls == 1


def test_engine_steps_through_the_native_agent_and_done_survives_a_failed_step(tmp_path):
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.pool.agents.native import NativeAgent

    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=64, max_model_len=256, num_blocks=64)
    ag = NativeAgent(eng, storage_dir=str(tmp_path))
    pool = PoolIface(ag)
    eng.attach_pool(pool)
    outs = eng.generate([[1, 2, 3, 4, 5] * 7, [9] * 20], max_new_tokens=5)
    assert all(len(o) == 5 for o in outs)
    assert pool.stats.prepare_calls == pool.stats.done_calls == ag.fence_stats["steps"] == eng.step_count
    assert pool.stats.finish_calls == len(eng.requests)  # every finished request reached the agent
    assert ag.stats["writeback_blocks"] == 2 + 1  # 35 + 5 and 20 + 5 tokens: full pages only
    # a forward that raises still closes the step's compute fence
    eng.add_request([7] * 10, max_new_tokens=3)

    def fail(*a, **k):
        raise RuntimeError("device lost")

    eng.runner.execute = fail
    with pytest.raises(RuntimeError, match="device lost"):
        eng.step()
    assert pool.stats.prepare_calls == pool.stats.done_calls


def test_promotion_from_l3_is_written_back_to_l2_and_mirrored_on_the_control_plane(tmp_path):
    """One pool node (L2 cap of 2 blocks) shared by two engines: the first writes a 5-page
    prompt back (3 pages end in L3), the second promotes all 5 at admission. Every promotion
    from L3 gives the page an L2 record again and moves the coldest L2 page to L3; afterwards
    the authority's L2 locations and L3 flags agree with the tier engine page by page."""
    from lake_b200 import _host as H
    from lake_b200.engine.block_pool import chain_block_hashes
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.pool.agents.native import NativeAgent, make_pool_node

    kw = dict(device="cpu", max_running=4, max_batched_tokens=128, max_model_len=256, num_blocks=64)
    a_eng, b_eng = LLMEngine("tiny", **kw), LLMEngine("tiny", **kw)
    page = a_eng.arena[0].numel() * a_eng.arena.element_size()
    node = make_pool_node("tiny", page, a_eng.pool.num_blocks, l1_blocks=8, l2_blocks=2, storage_dir=str(tmp_path))
    authority = H.Authority()
    a_ag = NativeAgent(a_eng, "n0", authority=authority, shared_tiers=node)
    b_ag = NativeAgent(b_eng, "n0", authority=authority, shared_tiers=node)
    a_eng.attach_pool(PoolIface(a_ag, node_id="n0"))
    b_eng.attach_pool(PoolIface(b_ag, node_id="n0"))
    prompt = list(range(3, 3 + 5 * 16 + 1))
    a_eng.generate([prompt], max_new_tokens=1)
    tiers = node[0]
    hashes = chain_block_hashes(prompt, 16, full_only=True)[:5]
    assert sum(tiers.is_l2_durable(h) for h in hashes) == 2 and sum(tiers.l3_present(h) for h in hashes) == 3
    b_eng.generate([prompt], max_new_tokens=1)
    assert b_ag.stats["promoted_blocks"] == 5
    assert [tiers.is_l2_durable(h) for h in hashes] == [False, False, False, True, True]  # the last two promoted
    for h in hashes:
        meta = authority.locate([H.KVBlockID("tiny", h)])[0]
        on_l2 = any(loc.tier == 3 and loc.node_id == "n0" for loc in meta.locations)
        assert on_l2 == tiers.is_l2_durable(h)
        assert meta.l3_present and tiers.l3_present(h)  # all five passed through L3


def test_a_shared_pool_node_owns_the_l2_locations_and_outlives_an_engine(tmp_path):
    """Two engines (worker-0, worker-1) share one pool node's tiers: what worker-0 writes back is
    registered with its L2 copy on the pool node, so reconciling worker-0 as dead leaves the
    durable copy in place and worker-1 still reuses the prefix from the pool."""
    from lake_b200 import _host as H
    from lake_b200.engine.block_pool import chain_block_hashes
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.pool.agents.native import NativeAgent, make_pool_node

    kw = dict(device="cpu", max_running=4, max_batched_tokens=128, max_model_len=256, num_blocks=64)
    a_eng, b_eng = LLMEngine("tiny", **kw), LLMEngine("tiny", **kw)
    page = a_eng.arena[0].numel() * a_eng.arena.element_size()
    node = make_pool_node("tiny", page, a_eng.pool.num_blocks, l1_blocks=8, l2_blocks=32, storage_dir=str(tmp_path))
    authority = H.Authority()
    for n, eng in (("worker-0", a_eng), ("worker-1", b_eng)):
        eng.attach_pool(PoolIface(NativeAgent(eng, n, authority=authority, shared_tiers=node,
                                              storage_node_id="pool-0"), node_id=n))
    prompt = list(range(3, 3 + 3 * 16 + 1))
    a_eng.generate([prompt], max_new_tokens=1)
    hashes = chain_block_hashes(prompt, 16, full_only=True)[:3]
    metas = authority.locate([H.KVBlockID("tiny", h) for h in hashes])
    assert all([(loc.tier, loc.node_id) for loc in m.locations if loc.tier == 3] == [(3, "pool-0")] for m in metas)
    authority.reconcile_dead_node("worker-0")
    metas = authority.locate([H.KVBlockID("tiny", h) for h in hashes])
    assert all(any(loc.tier == 3 and loc.node_id == "pool-0" for loc in m.locations) for m in metas)
    rid = b_eng.add_request(prompt, max_new_tokens=1)
    while b_eng.has_unfinished():
        b_eng.step()
    assert b_eng.requests[rid].num_cached == 3 * 16  # the three blocks came from the pool
