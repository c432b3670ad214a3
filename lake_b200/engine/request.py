"""Host request state for the engine (reference: python/lake/runtime/req.py:13-39)."""
from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field


# Placeholder for a token an in-flight step is still sampling (overlapped scheduling); the
# engine replaces it when the step completes. Real token ids are >= 0.
PENDING = -1


class RequestStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"
    ABORTED = "aborted"


@dataclass
class SamplingParams:
    max_new_tokens: int = 16
    temperature: float = 0.0  # greedy only on the fused path
    eos_token_id: int | None = None
    ignore_eos: bool = True


@dataclass(eq=False)
class Request:
    rid: str
    prompt: list[int]
    params: SamplingParams = field(default_factory=SamplingParams)
    output: list[int] = field(default_factory=list)
    status: RequestStatus = RequestStatus.WAITING
    num_computed: int = 0  # tokens whose KV is resident
    num_cached: int = 0  # prefix tokens served from the prefix cache at admission
    block_ids: list[int] = field(default_factory=list)
    block_hashes: list[bytes] = field(default_factory=list)
    registered_blocks: int = 0
    bitmask: object | None = None  # optional [ceil(V/32)] int32 allowed-token mask for the next token
    arrival: float = field(default_factory=time.perf_counter)
    admit_time: float | None = None  # when the scheduler gave it pages (end of its queue wait)
    first_token_time: float | None = None
    finish_time: float | None = None
    token_times: list[float] = field(default_factory=list)
    # disaggregation hooks
    exec_mode: str = "colocated"
    # pages of this request's KV in a decode instance's arena (prefill side of PD-split)
    remote_blocks: list[int] | None = None
    # page index -> host tier slot the QKV epilogue also writes this page's K/V into (the kernel
    # side of the D -> pool write-behind; set by the storage agent)
    mirror_blocks: dict | None = None
    meta: dict = field(default_factory=dict)

    @property
    def all_tokens(self) -> list[int]:
        return self.prompt + self.output

    def tokens_slice(self, a: int, b: int) -> list[int]:
        lp = len(self.prompt)
        if a >= lp:
            return self.output[a - lp:b - lp]
        if b <= lp:
            return self.prompt[a:b]
        return self.prompt[a:] + self.output[: b - lp]

    @property
    def num_tokens(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def is_prefill(self) -> bool:
        return self.num_computed < len(self.prompt)

    @property
    def finished(self) -> bool:
        return self.status in (RequestStatus.FINISHED, RequestStatus.ABORTED)

    def should_stop(self) -> bool:
        if len(self.output) >= self.params.max_new_tokens:
            return True
        if (not self.params.ignore_eos and self.params.eos_token_id is not None and self.output
                and self.output[-1] == self.params.eos_token_id):
            return True
        return False

    def ttft(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.arrival

    def tpot(self) -> float | None:
        if len(self.token_times) < 2:
            return None
        return (self.token_times[-1] - self.token_times[0]) / (len(self.token_times) - 1)
