"""Step fences of the storage-agent contract, shared by this package's agents.

The engine brackets every step with the agent's ready fence (prepare_step, after
which the step's block tables are valid) and its compute fence (done, after which
the step's KV writes are complete). Exactly one step may sit between the two. A
request that finishes while a step is open may still be read or written by that
step, so its finish is held and run when the step closes.

Reference parity: the fence contract of python/lake/engine/agent.py:15-41 and
pool_iface.py:52-211 (protocol errors on unpaired fences, deferred finishes).
"""
from __future__ import annotations

from ..types import FinishRequest, PoolError, PoolErrorCode


class StepFences:
    """Mixin: subclasses implement ``_finish(FinishRequest)``; the fence calls are
    ``_open(step_id)`` (at the end of a successful prepare_step), ``done(step_id)``
    and ``on_request_finished(finish)``."""

    def __init__(self) -> None:
        self._open_step: int | None = None
        self._held: list[FinishRequest] = []
        self.fence_stats = {"steps": 0, "held_finishes": 0}

    def _check_closed(self) -> None:
        if self._open_step is not None:
            raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"prepare while step {self._open_step} is ready")

    def _open(self, step_id: int) -> None:
        self._check_closed()
        self._open_step = step_id

    def done(self, step_id: int) -> None:
        if self._open_step is None or self._open_step != step_id:
            raise PoolError(PoolErrorCode.PROTOCOL_ERROR, f"done for step {step_id}, open step {self._open_step}")
        self._open_step = None
        self.fence_stats["steps"] += 1
        held, self._held = self._held, []
        for f in held:
            self._finish(f)

    def on_request_finished(self, finish: FinishRequest) -> None:
        if self._open_step is not None:
            self._held.append(finish)
            self.fence_stats["held_finishes"] += 1
            return
        self._finish(finish)

    def commit_write_extent(self, req_id: str, token_end: int) -> None:
        """The engine's scheduler owns every L0 page and its extent, so there is no pool-side
        reservation to trim here."""
        return None

    def _finish(self, finish: FinishRequest) -> None:  # pragma: no cover - abstract
        raise NotImplementedError
