"""In-memory storage agent for unit tests of the pool contract.

It simulates per-request L0 token extents (no bytes), lets tests force pulls
with an injected cost to exercise the pull budget (TIMEOUT, or dropping the
request from the step when partial hits are allowed), defers request finishes
that arrive while a step is between its ready and done fences, and guards
commit_write_extent against shrinking a reservation a newer prepare raised.

Reference parity: python/lake/engine/agents/memory.py:23-162 (same contract;
block tables here use the engine's 16-token pages).
"""
from __future__ import annotations

import logging

from ..types import FinishRequest, PoolError, PoolErrorCode, PreparePlan, ReadyHandle, StepStats

LOG = logging.getLogger("lake_b200.pool.memory")


class InMemoryAgent:
    def __init__(self, block_size: int = 16):
        self.block_size = block_size
        self.l0_token_end: dict[str, int] = {}
        self.force_pull_reqs: set[str] = set()
        self.pull_cost_ms = 0
        self.finished: list[str] = []
        self.prepare_calls = 0
        self.done_calls = 0
        self._ready_step: int | None = None
        self._frozen: set[str] = set()
        self._deferred: list[FinishRequest] = []
        self._prepares_since_commit: dict[str, int] = {}

    def seed_local_prefix(self, req_id: str, token_end: int) -> None:
        self.l0_token_end[req_id] = max(self.l0_token_end.get(req_id, 0), token_end)

    def probe_local(self, req_id: str, prompt_len: int) -> tuple[int, bool]:
        have = self.l0_token_end.get(req_id, 0)
        return min(have, prompt_len), prompt_len > 0 and have >= prompt_len

    def prepare_step(self, plan: PreparePlan) -> ReadyHandle:
        self.prepare_calls += 1
        if self._ready_step is not None:
            raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"prepare while step {self._ready_step} is ready")
        self._flush_deferred()
        stats: dict[str, StepStats] = {}
        eff_read, eff_write = list(plan.read_set), list(plan.write_set)
        spent = 0
        for io in plan.read_set:
            have = self.l0_token_end.get(io.req_id, 0)
            if io.req_id in self.force_pull_reqs or have < io.token_end:
                spent += self.pull_cost_ms
                if plan.pull_budget_ms > 0 and spent > plan.pull_budget_ms:
                    if plan.allow_partial_hit:
                        eff_read = [x for x in eff_read if x.req_id != io.req_id]
                        eff_write = [x for x in eff_write if x.req_id != io.req_id]
                        continue
                    raise PoolError(PoolErrorCode.TIMEOUT, f"pull budget {plan.pull_budget_ms}ms exceeded "
                                                           f"for {io.req_id}")
                self.l0_token_end[io.req_id] = max(have, io.token_end)
                stats.setdefault(io.req_id, StepStats()).pulled_blocks += 1
            self._frozen.add(io.req_id)
            stats.setdefault(io.req_id, StepStats())
        live_write = {x.req_id for x in eff_write}
        for io in plan.write_set:
            if io.req_id not in live_write:
                continue
            self.l0_token_end[io.req_id] = max(self.l0_token_end.get(io.req_id, 0), io.token_end)
            self._prepares_since_commit[io.req_id] = self._prepares_since_commit.get(io.req_id, 0) + 1
            self._frozen.add(io.req_id)
            st = stats.setdefault(io.req_id, StepStats())
            if io.token_start == 0 and io.token_end > 0:
                st.prefill_blocks = max(st.prefill_blocks, 1)
        self._ready_step = plan.step_id
        bs = self.block_size
        live = {x.req_id for x in eff_read} | live_write
        tables = {r: list(range((self.l0_token_end.get(r, 0) + bs - 1) // bs)) for r in live}
        slots = {io.req_id: list(range(io.token_start, io.token_end)) for io in eff_write}
        return ReadyHandle(plan.step_id, stats, eff_read, eff_write, tables, slots)

    def done(self, step_id: int) -> None:
        self.done_calls += 1
        if self._ready_step != step_id:
            raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"done step={step_id} ready={self._ready_step}")
        self._ready_step = None
        self._frozen.clear()
        self._flush_deferred()

    def on_request_finished(self, finish: FinishRequest) -> None:
        if finish.req_id in self._frozen or self._ready_step is not None:
            self._deferred.append(finish)
            return
        self._apply_finish(finish)

    def commit_write_extent(self, req_id: str, token_end: int) -> None:
        n = self._prepares_since_commit.get(req_id, 0)
        if n > 1:  # a newer prepare raised the reservation: keep it
            self._prepares_since_commit[req_id] = n - 1
            return
        if req_id in self.l0_token_end:
            self.l0_token_end[req_id] = min(self.l0_token_end[req_id], max(0, token_end))
        self._prepares_since_commit[req_id] = 0

    def _flush_deferred(self) -> None:
        if self._ready_step is not None or self._frozen:
            return
        pending, self._deferred = self._deferred, []
        for f in pending:
            self._apply_finish(f)

    def _apply_finish(self, f: FinishRequest) -> None:
        self.l0_token_end.pop(f.req_id, None)
        self._prepares_since_commit.pop(f.req_id, None)
        self.finished.append(f.req_id)
