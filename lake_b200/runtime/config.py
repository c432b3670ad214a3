"""Worker role configuration, lifecycle state machine and execution modes.

Environment variables keep the reference's names (python/lake/runtime/role.py:70-108)
so deployment scripts carry over; defaults fit the B200 engine.
Lifecycle: Idle -> Boot -> Warm -> Ready -> Serving -> Drain -> Terminate
(python/lake/runtime/lifecycle.py:16-96). Execution modes and the node-side
mode selection twin the router's (python/lake/runtime/mode_select.py:22-41,
exec_mode.py:8-11).
"""
from __future__ import annotations

import enum
import os
from dataclasses import dataclass

from ..pool.types import PrefixHint


class WorkerRole(str, enum.Enum):
    PREFILL = "prefill"
    DECODE = "decode"
    HYBRID = "hybrid"


class ExecMode(str, enum.Enum):
    COLOCATED = "COLOCATED"
    PD_DISAGG = "PD_DISAGG"
    D_DIRECT = "D_DIRECT"


TRANSFER_BW_THRESHOLD_GBPS = 1.0


def select_exec_mode(hint: PrefixHint, prompt_len: int, role: WorkerRole, bw_gbps: float = 0.0) -> ExecMode:
    """Local full hit -> D_DIRECT; pool hit over a slow link -> COLOCATED; prefill/decode
    roles -> PD_DISAGG; else COLOCATED (same rule as the router core)."""
    if prompt_len > 0 and hint.local_hit and hint.computed_tokens > 0:
        return ExecMode.D_DIRECT
    if hint.reused_blocks > 0 and 0 < bw_gbps < TRANSFER_BW_THRESHOLD_GBPS:
        return ExecMode.COLOCATED
    if role in (WorkerRole.PREFILL, WorkerRole.DECODE):
        return ExecMode.PD_DISAGG
    return ExecMode.COLOCATED


def full_local_hit(hint: PrefixHint, prompt_len: int) -> bool:
    return prompt_len > 0 and hint.local_hit and hint.computed_tokens >= prompt_len


def _env_bool(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    if v is None or not v.strip():
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    try:
        return int(v) if v is not None and v.strip() else default
    except ValueError:
        return default


@dataclass
class RoleConfig:
    role: WorkerRole = WorkerRole.HYBRID
    enable_drafter: bool = False
    num_draft_tokens: int = 2
    enable_overlap: bool = True
    max_running_reqs: int = 256
    max_num_scheduled_tokens: int = 8192
    long_prefill_token_threshold: int = 0
    max_model_length: int = 8192
    pull_budget_ms: int = 0
    allow_partial_hit: bool = False
    model_backend: str = "llama3-8b"  # a preset name, a config.json path, a checkpoint directory, or "mock"
    model_path: str = ""
    served_model_name: str = "model"
    model_revision: str = ""
    warmup_num_reqs: int = 1
    warmup_tokens_per_req: int = 1
    device: str = "cuda"
    num_blocks: int = 0

    def __post_init__(self):
        if self.max_num_scheduled_tokens <= 0:
            raise ValueError(f"max_num_scheduled_tokens must be > 0, got {self.max_num_scheduled_tokens}")
        if self.max_running_reqs <= 0:
            raise ValueError(f"max_running_reqs must be > 0, got {self.max_running_reqs}")
        if self.warmup_num_reqs <= 0 or self.warmup_tokens_per_req <= 0:
            raise ValueError("warmup sizes must be > 0")

    @classmethod
    def from_env(cls) -> "RoleConfig":
        role_raw = os.environ.get("LAKE_WORKER_ROLE", "hybrid").strip().lower()
        try:
            role = WorkerRole(role_raw)
        except ValueError:
            role = WorkerRole.HYBRID
        return cls(
            role=role,
            model_backend=(os.environ.get("LAKE_MODEL_BACKEND", "llama3-8b").strip() or "llama3-8b"),
            model_path=os.environ.get("LAKE_MODEL_PATH", "").strip(),
            served_model_name=os.environ.get("LAKE_SERVED_MODEL_NAME", "model").strip() or "model",
            model_revision=os.environ.get("LAKE_MODEL_REVISION", "").strip(),
            enable_drafter=_env_bool("LAKE_ENABLE_DRAFTER", False),
            enable_overlap=_env_bool("LAKE_ENABLE_OVERLAP", True),
            allow_partial_hit=_env_bool("LAKE_ALLOW_PARTIAL_HIT", False),
            num_draft_tokens=_env_int("LAKE_NUM_DRAFT_TOKENS", 2),
            max_running_reqs=_env_int("LAKE_MAX_RUNNING_REQS", 256),
            max_num_scheduled_tokens=_env_int("LAKE_MAX_NUM_SCHEDULED_TOKENS", 8192),
            long_prefill_token_threshold=_env_int("LAKE_LONG_PREFILL_TOKEN_THRESHOLD", 0),
            max_model_length=_env_int("LAKE_MAX_MODEL_LENGTH", 8192),
            pull_budget_ms=_env_int("LAKE_PULL_BUDGET_MS", 0),
            warmup_num_reqs=_env_int("LAKE_WARMUP_NUM_REQS", 1),
            warmup_tokens_per_req=_env_int("LAKE_WARMUP_TOKENS_PER_REQ", 1),
            device=os.environ.get("LAKE_DEVICE", "cuda").strip() or "cuda",
            num_blocks=_env_int("LAKE_NUM_BLOCKS", 0),
        )


class WorkerState(str, enum.Enum):
    IDLE = "idle"
    BOOT = "boot"
    WARM = "warm"
    READY = "ready"
    SERVING = "serving"
    DRAIN = "drain"
    TERMINATE = "terminate"


_ORDER = [WorkerState.IDLE, WorkerState.BOOT, WorkerState.WARM, WorkerState.READY, WorkerState.SERVING,
          WorkerState.DRAIN, WorkerState.TERMINATE]


@dataclass(frozen=True)
class CapacitySignal:
    """Load reported upward (the worker reports, it does not throttle by itself)."""

    waiting: int
    running: int
    inflight_reqs: int
    max_running_reqs: int
    state: WorkerState
    role: str
    model_backend: str
    served_model_name: str = "model"
    model_loaded: bool = False
    model_warmed: bool = False

    @property
    def remaining_slots(self) -> int:
        return max(0, self.max_running_reqs - self.running)


class WorkerLifecycle:
    def __init__(self, initial: WorkerState = WorkerState.IDLE):
        self._state = initial

    @property
    def state(self) -> WorkerState:
        return self._state

    def advance(self, to: WorkerState) -> None:
        if to == self._state or self._state == WorkerState.TERMINATE:  # terminal: nothing follows it
            return
        if to in (WorkerState.DRAIN, WorkerState.TERMINATE):
            self._state = to
            return
        if _ORDER.index(to) < _ORDER.index(self._state):
            raise ValueError(f"cannot regress {self._state.value} -> {to.value}")
        self._state = to

    def warm(self) -> None:
        if self._state == WorkerState.IDLE:
            self.advance(WorkerState.BOOT)
        self.advance(WorkerState.WARM)

    def ready(self) -> None:
        self.advance(WorkerState.READY)

    def serve(self) -> None:
        self.advance(WorkerState.SERVING)

    def drain(self) -> None:
        self.advance(WorkerState.DRAIN)

    def terminate(self) -> None:
        self.advance(WorkerState.TERMINATE)

    @property
    def accepting(self) -> bool:
        return self._state in (WorkerState.READY, WorkerState.SERVING)
