"""Engine <-> storage-pool contract (PoolIface over the in-memory agent): ready/done fences,
pull budget, partial hits, deferred finishes, the commit-vs-newer-prepare guard, handle
validation and error wrapping; and an engine whose steps run through the pool (modelled on the
reference's python/lake/engine/tests/test_pool_agent.py and test_executor.py behaviours)."""
import pytest

from lake_b200.pool.agents.memory import InMemoryAgent
from lake_b200.pool.pool_iface import PoolIface
from lake_b200.pool.types import (FinishRequest, ForwardMode, PoolError, PoolErrorCode, PreparePlan, ReadyHandle,
                                  ReqIoSet)


def plan(step, reads=(), writes=(("a", 0, 16),), budget=0, partial=False):
    rs = [ReqIoSet(r, s, e) for r, s, e in reads]
    ws = [ReqIoSet(r, s, e) for r, s, e in writes]
    return PreparePlan(step, ForwardMode.EXTEND, rs, ws, {io.req_id: io.token_end - io.token_start for io in ws},
                       budget, partial)


def test_ready_done_fences_are_strictly_paired():
    ag = InMemoryAgent()
    h = ag.prepare_step(plan(1))
    assert h.step_id == 1 and h.block_table_by_req["a"] == [0]
    with pytest.raises(PoolError) as e:
        ag.prepare_step(plan(2))
    assert e.value.code == PoolErrorCode.PROTOCOL_ERROR
    with pytest.raises(PoolError):
        ag.done(7)
    ag.done(1)
    ag.prepare_step(plan(2))


def test_pull_budget_timeout_or_partial_hit():
    ag = InMemoryAgent()
    ag.force_pull_reqs = {"a"}
    ag.pull_cost_ms = 50
    with pytest.raises(PoolError) as e:
        ag.prepare_step(plan(1, reads=[("a", 0, 32)], writes=[("a", 32, 33)], budget=20))
    assert e.value.code == PoolErrorCode.TIMEOUT
    # with partial hits allowed the request is dropped from the step instead
    h = ag.prepare_step(plan(2, reads=[("a", 0, 32)], writes=[("a", 32, 33), ("b", 0, 16)], budget=20,
                             partial=True))
    assert [io.req_id for io in h.effective_write_set] == ["b"]
    ag.done(2)


def test_finish_between_fences_is_deferred_until_done():
    ag = InMemoryAgent()
    ag.prepare_step(plan(1))
    ag.on_request_finished(FinishRequest("a", "n0"))
    assert ag.finished == []  # the step still reads/writes "a"
    ag.done(1)
    assert ag.finished == ["a"]


def test_commit_keeps_a_reservation_a_newer_prepare_raised():
    ag = InMemoryAgent()
    ag.prepare_step(plan(1, writes=[("a", 0, 16)]))
    ag.done(1)
    ag.prepare_step(plan(2, writes=[("a", 16, 32)]))
    ag.done(2)
    ag.commit_write_extent("a", 16)  # stale commit from step 1: step 2 raised the extent
    assert ag.l0_token_end["a"] == 32
    ag.commit_write_extent("a", 20)
    assert ag.l0_token_end["a"] == 20


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


def test_engine_steps_through_the_pool_and_done_survives_a_failed_step():
    from lake_b200.engine.llm_engine import LLMEngine

    ag = InMemoryAgent()
    pool = PoolIface(ag)
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=64, max_model_len=256, num_blocks=64)
    eng.attach_pool(pool)
    outs = eng.generate([[1, 2, 3, 4, 5] * 7, [9] * 20], max_new_tokens=5)
    assert all(len(o) == 5 for o in outs)
    assert ag.prepare_calls == ag.done_calls == eng.step_count
    assert sorted(ag.finished) == sorted(eng.requests)  # every finished request reached the agent
    # a forward that raises still closes the step's compute fence
    eng.add_request([7] * 10, max_new_tokens=3)

    def fail(*a, **k):
        raise RuntimeError("device lost")

    eng.runner.execute = fail
    with pytest.raises(RuntimeError, match="device lost"):
        eng.step()
    assert ag.prepare_calls == ag.done_calls
