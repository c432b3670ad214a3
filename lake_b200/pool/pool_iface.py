"""The engine's interface to the storage pool.

PoolIface turns one scheduled step into a PreparePlan, calls the agent's ready
fence, validates the returned ReadyHandle (same step id; effective sets only
shrink the plan, and only when partial hits are allowed), forwards the compute
fence and the request-finish call (idempotent), and wraps unexpected agent
failures as DOWNSTREAM errors. Counters are kept per call kind.

Reference parity: python/lake/engine/pool_iface.py:52-211 and the StorageAgent
protocol in python/lake/engine/agent.py:15-41.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Protocol, runtime_checkable

from .types import (FinishRequest, PoolError, PoolErrorCode, PreparePlan, PrefixHint, ReadyHandle, ReqIoSet,
                    forward_mode_of)

LOG = logging.getLogger("lake_b200.pool")


@runtime_checkable
class StorageAgent(Protocol):
    def prepare_step(self, plan: PreparePlan) -> ReadyHandle: ...

    def done(self, step_id: int) -> None: ...

    def on_request_finished(self, finish: FinishRequest) -> None: ...

    def commit_write_extent(self, req_id: str, token_end: int) -> None: ...


@dataclass
class PoolIfaceStats:
    prepare_calls: int = 0
    done_calls: int = 0
    finish_calls: int = 0
    duplicate_finish_calls: int = 0
    commit_calls: int = 0
    errors: int = 0


class PoolIface:
    def __init__(self, agent, *, pull_budget_ms: int = 0, allow_partial_hit: bool = False, node_id: str = "node-0"):
        self.agent = agent
        self.pull_budget_ms = pull_budget_ms
        self.allow_partial_hit = allow_partial_hit
        self.node_id = node_id
        self.stats = PoolIfaceStats()
        self._last_ready: ReadyHandle | None = None
        self._finished: set[str] = set()

    # ------------------------------------------------------------ plan construction
    @staticmethod
    def plan_from_step(out, pull_budget_ms: int = 0, allow_partial_hit: bool = False) -> PreparePlan:
        """PreparePlan of an engine SchedulerOutput: each chunk reads its context [0, start)
        and writes [start, start+n)."""
        read, write, nsched = [], [], {}
        for ch in out.chunks:
            rid = ch.req.rid
            if ch.start:
                read.append(ReqIoSet(rid, 0, ch.start))
            write.append(ReqIoSet(rid, ch.start, ch.start + ch.n))
            nsched[rid] = ch.n
        return PreparePlan(out.step_id, forward_mode_of(len(out.decode), len(out.prefill)), read, write, nsched,
                           pull_budget_ms, allow_partial_hit)

    # ------------------------------------------------------------ calls
    def _call(self, what: str, fn):
        try:
            return fn()
        except PoolError:
            self.stats.errors += 1
            raise
        except Exception as e:  # unexpected agent failure -> downstream error
            self.stats.errors += 1
            raise PoolError(PoolErrorCode.DOWNSTREAM, f"{what}: {type(e).__name__}: {e}") from e

    def probe_prefix(self, req) -> PrefixHint:
        probe = getattr(self.agent, "probe_prefix", None)
        if callable(probe):
            return self._call("probe_prefix", lambda: probe(req))
        return PrefixHint()

    def prepare_step(self, out) -> ReadyHandle:
        plan = self.plan_from_step(out, self.pull_budget_ms, self.allow_partial_hit)
        self.stats.prepare_calls += 1
        handle = self._call("prepare_step", lambda: self.agent.prepare_step(plan))
        self._validate(plan, handle)
        self._last_ready = handle
        return handle

    def done(self, step_id: int) -> None:
        self.stats.done_calls += 1
        self._call("done", lambda: self.agent.done(step_id))
        self._last_ready = None

    def on_request_finished(self, req, model_id: str = "") -> None:
        if req.rid in self._finished:
            self.stats.duplicate_finish_calls += 1
            return
        self.stats.finish_calls += 1
        self._call("on_request_finished",
                   lambda: self.agent.on_request_finished(FinishRequest(req.rid, self.node_id, model_id)))
        self._finished.add(req.rid)

    def commit_write_extent(self, req_id: str, token_end: int) -> None:
        if token_end < 0:
            raise PoolError(PoolErrorCode.INVALID_ARG, f"token_end must be >= 0: {token_end}")
        commit = getattr(self.agent, "commit_write_extent", None)
        if not callable(commit):
            return
        self.stats.commit_calls += 1
        self._call("commit_write_extent", lambda: commit(req_id, token_end))

    # ------------------------------------------------------------ validation
    def _validate(self, plan: PreparePlan, h: ReadyHandle) -> None:
        if h.step_id != plan.step_id:
            raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"ready step={h.step_id} != plan step={plan.step_id}")
        planned = {(io.req_id): io for io in plan.write_set}
        for ios, name in ((h.effective_read_set, "read"), (h.effective_write_set, "write")):
            if ios is None:
                continue
            for io in ios:
                if io.token_end < io.token_start:
                    raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"invalid {name} range for {io.req_id}")
                if io.req_id not in plan.num_scheduled_tokens:
                    raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"effective {name} set has unplanned {io.req_id}")
        if h.effective_write_set is not None:
            eff = {io.req_id: io for io in h.effective_write_set}
            shrunk = set(planned) - set(eff) or any(
                eff[r].token_end < planned[r].token_end for r in eff if r in planned)
            if shrunk and not plan.allow_partial_hit:
                raise PoolError(PoolErrorCode.PROTOCOL_ERROR, "agent shrank the batch without allow_partial_hit")
