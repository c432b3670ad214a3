"""Scheduler policy under the scenarios the reference's scheduler budget tests pin
(python/lake/runtime/tests/test_scheduler_budget.py:45-165): a long prompt advances in chunks
capped by the long-prefill threshold, the token budget caps a step's batch, decodes take their
tokens first and the rest of the budget goes to a prefill chunk (a mixed step), and admission
rejects a request whose prompt plus output exceeds the model length. Pure host logic on the
block pool, no model."""
import pytest

from lake_b200.engine.block_pool import BlockPool
from lake_b200.engine.request import Request, SamplingParams
from lake_b200.engine.scheduler import Scheduler, SchedulerConfig


def _req(rid, prompt, out=2):
    return Request(rid=rid, prompt=list(prompt), params=SamplingParams(max_new_tokens=out))


def _sched(**kw):
    args = dict(max_running=4, max_batched_tokens=64, max_model_len=256)
    args.update(kw)
    return Scheduler(BlockPool(64, 16), SchedulerConfig(**args))


def _run(s, token=7):
    """Steps the scheduler to idle; returns each step's prefill chunk sizes."""
    sizes = []
    for _ in range(100):
        if not s.has_work():
            break
        o = s.schedule()
        sizes.append([c.n for c in o.prefill])
        s.update(o, [token] * sum(c.n_samples for c in o.chunks), 0.0)
    return sizes


def test_a_long_prompt_advances_in_threshold_sized_chunks():
    s = _sched(long_prefill_threshold=4)
    r = _req("c1", range(10), out=2)
    s.add(r)
    sizes = _run(s)
    assert [n for step in sizes for n in step] == [4, 4, 2]  # 10 tokens: 4 + 4 + 2
    assert r.finished and len(r.output) == 2


def test_the_token_budget_caps_a_steps_batch():
    s = _sched(max_batched_tokens=8, long_prefill_threshold=0)
    a, b = _req("a", range(8), out=1), _req("b", range(8, 16), out=1)
    s.add(a)
    s.add(b)
    o = s.schedule()
    assert [(c.req.rid, c.n) for c in o.prefill] == [("a", 8)]  # room for one whole prompt
    s.update(o, [7] * sum(c.n_samples for c in o.chunks), 0.0)
    _run(s)
    assert a.finished and b.finished


def test_decodes_come_first_and_the_rest_of_the_budget_prefills():
    s = _sched(max_batched_tokens=8, long_prefill_threshold=0)
    a = _req("a", range(7), out=3)
    s.add(a)
    o = s.schedule()
    s.update(o, [7] * sum(c.n_samples for c in o.chunks), 0.0)  # a is now decoding
    s.add(_req("b", range(100, 108), out=1))
    o = s.schedule()
    assert [c.req.rid for c in o.decode] == ["a"]
    assert [(c.req.rid, c.n) for c in o.prefill] == [("b", 7)]  # 8 - 1 decode token
    assert sum(c.n for c in o.decode) + sum(c.n for c in o.prefill) == 8


def test_admission_rejects_a_request_longer_than_the_model():
    s = _sched(max_model_len=10)
    with pytest.raises(ValueError, match="max_model_len"):
        s.add(_req("x", range(8), out=5))
    s.add(_req("y", range(5), out=5))  # exactly at the limit: admitted
