"""Types shared by the engine's pool interface and the storage agents.

Names and fields follow the reference's pool contract
(python/lake/engine/pool_types.py:12-72, runtime/scheduler_output.py:15-103) so
agents written against it keep working: a per-step PreparePlan goes to the
agent, a ReadyHandle (ready fence) comes back, done() is the compute fence, and
on_request_finished() closes a request's KV.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field


class PoolErrorCode(str, enum.Enum):
    OK = "OK"
    TIMEOUT = "TIMEOUT"  # pull exceeded its budget
    CAPACITY = "CAPACITY"  # hard quota / no free L0 page
    PROTOCOL_ERROR = "PROTOCOL_ERROR"  # ready/done fence mismatch
    DOWNSTREAM = "DOWNSTREAM"  # control plane / KV backend failure
    INVALID_ARG = "INVALID_ARG"


class PoolError(Exception):
    def __init__(self, code: PoolErrorCode, message: str = "") -> None:
        self.code = code
        super().__init__(message or code.value)

    def __str__(self) -> str:
        return f"{self.code.value}: {super().__str__()}"


class ForwardMode(str, enum.Enum):
    EXTEND = "EXTEND"
    DECODE = "DECODE"
    MIXED = "MIXED"
    IDLE = "IDLE"
    TARGET_VERIFY = "TARGET_VERIFY"
    DRAFT_EXTEND = "DRAFT_EXTEND"
    PREBUILT = "PREBUILT"


@dataclass
class ReqIoSet:
    """Token range [token_start, token_end) of one request read or written this step."""

    req_id: str
    token_start: int
    token_end: int
    pool_kind: str = "TARGET"


@dataclass
class StepStats:
    reused_blocks: int = 0
    prefill_blocks: int = 0
    pulled_blocks: int = 0


@dataclass
class ReadyHandle:
    step_id: int
    stats_by_req: dict[str, StepStats] = field(default_factory=dict)
    effective_read_set: list[ReqIoSet] | None = None
    effective_write_set: list[ReqIoSet] | None = None
    block_table_by_req: dict[str, list[int]] = field(default_factory=dict)
    slot_mapping_by_req: dict[str, list[int]] = field(default_factory=dict)


@dataclass
class PreparePlan:
    step_id: int
    forward_mode: ForwardMode
    read_set: list[ReqIoSet]
    write_set: list[ReqIoSet]
    num_scheduled_tokens: dict[str, int]
    pull_budget_ms: int = 0
    allow_partial_hit: bool = False


@dataclass
class FinishRequest:
    req_id: str
    node_id: str
    model_id: str = ""


@dataclass
class PrefixHint:
    """Router-provided (or probed) reuse hint for one request (reference: runtime/prefix_hint.py:8-13)."""

    computed_tokens: int = 0
    reused_blocks: int = 0
    local_hit: bool = False
    prebuilt: bool = False


def forward_mode_of(n_decode: int, n_prefill: int) -> ForwardMode:
    if n_decode and n_prefill:
        return ForwardMode.MIXED
    if n_decode:
        return ForwardMode.DECODE
    if n_prefill:
        return ForwardMode.EXTEND
    return ForwardMode.IDLE
