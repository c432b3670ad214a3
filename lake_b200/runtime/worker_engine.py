"""Long-lived engine loop of one worker process.

One step thread owns the LLMEngine. gRPC handler threads submit requests into
an inbound queue (coalesced for up to 5 ms when the engine is idle, so a burst
lands in one batch) and block on a per-request event. The loop admits the
inbound requests, runs engine steps while work exists, and completes each
request's event when it finishes. A step failure fails every in-flight request
with the error, rejects new submissions and stops the loop (the router then
re-dispatches: a PoolError surfaces as UNAVAILABLE at the gRPC layer).

Lifecycle: Boot -> Warm (build the model, one warm-up generation) -> Ready ->
Serving; stop() drains or aborts.

Reference parity: python/lake/runtime/worker_engine.py:36-270 and
node_scheduler.py:151-228 (run loop with overlap; here the engine step itself
is the overlap unit: host scheduling of step n+1 follows the device sync of
step n).
"""
from __future__ import annotations

import logging
import queue
import threading
import time
from dataclasses import dataclass, field

from ..engine.request import PENDING, RequestStatus
from ..pool.types import PoolError, PoolErrorCode, PrefixHint
from .config import CapacitySignal, ExecMode, RoleConfig, WorkerLifecycle, WorkerState, select_exec_mode

LOG = logging.getLogger("lake_b200.worker")
COALESCE_S = 0.005


def _step_error_code(e: Exception) -> PoolErrorCode:
    """A kernel's bounded wait that ran out (a peer GPU stopped answering) is a TIMEOUT; any other
    step failure is DOWNSTREAM. Both reach the router as UNAVAILABLE and trigger re-dispatch."""
    from ..ops.core import KernelError

    return PoolErrorCode.TIMEOUT if isinstance(e, KernelError) and e.timeout else PoolErrorCode.DOWNSTREAM


@dataclass
class GenerateResult:
    request_id: str
    output_tokens: list[int] = field(default_factory=list)
    reused_blocks: int = 0
    prefill_blocks: int = 0
    mode: str = ExecMode.COLOCATED.value
    error: Exception | None = None


@dataclass
class _Inbound:
    rid: str
    prompt: list[int]
    max_new_tokens: int
    mode: ExecMode
    hint: PrefixHint
    event: threading.Event = field(default_factory=threading.Event)
    result: GenerateResult | None = None


def build_engine(cfg: RoleConfig, **kw):
    from ..engine.llm_engine import LLMEngine

    model = cfg.model_backend
    device = cfg.device
    if model == "mock":  # small CPU model for plumbing tests
        model, device = "tiny", "cpu"
    elif cfg.model_path:
        model = cfg.model_path
    return LLMEngine(model, device=device, max_running=cfg.max_running_reqs,
                     max_batched_tokens=cfg.max_num_scheduled_tokens,
                     long_prefill_threshold=cfg.long_prefill_token_threshold,
                     max_model_len=cfg.max_model_length or 8192, num_blocks=cfg.num_blocks,
                     use_cuda_graphs=device != "cpu",
                     **{"overlap": cfg.enable_overlap,
                        "spec_tokens": cfg.num_draft_tokens if cfg.enable_drafter else 0, **kw})


class WorkerEngine:
    def __init__(self, cfg: RoleConfig, pool=None, engine=None, node_id: str = "worker-0", pool_factory=None):
        self.cfg = cfg
        self.pool = pool
        # pool_factory(engine) -> PoolIface: a pool interface that needs the built engine (the
        # remote storage agent); attached after the warm-up generation, which stays local
        self.pool_factory = pool_factory
        self.node_id = node_id
        self.engine = engine
        self.lifecycle = WorkerLifecycle()
        self._inbox: "queue.Queue[_Inbound]" = queue.Queue()
        self._inflight: dict[str, _Inbound] = {}
        self._thread: threading.Thread | None = None
        self._stop = threading.Event()
        # intake: submit() enqueues under this lock and only while open; stop() and a step
        # failure close it before they reject what is queued, so no submitter is left waiting
        self._intake = threading.Lock()
        self._intake_open = True
        self._failed: Exception | None = None
        self.steps = 0
        self.on_finished = None  # optional callback(request) after a request completes
        # PD-split: a decode worker's link to its prefill instance(s) (parallel.pd.DecodeSide);
        # PD_DISAGG requests are granted pages here and prefilled there
        self.pd_side = None
        self._engine_rid: dict[str, str] = {}  # request id -> the engine's id for it
        from .metrics import WorkerMetrics

        self.metrics = WorkerMetrics(node_id)

    # ------------------------------------------------------------ lifecycle
    def start(self, timeout_s: float = 600.0) -> None:
        self.lifecycle.warm()
        if self.engine is None:
            self.engine = build_engine(self.cfg)
        self.metrics.engine = self.engine
        if self.pool is not None:
            self.engine.attach_pool(self.pool)
        self._warmup()
        if self.pool is None and self.pool_factory is not None:
            self.pool = self.pool_factory(self.engine)
            self.engine.attach_pool(self.pool)
        self.lifecycle.ready()
        self._thread = threading.Thread(target=self._loop, name="lakeb-step", daemon=True)
        self._thread.start()
        self.lifecycle.serve()

    def _warmup(self) -> None:
        n = self.cfg.warmup_num_reqs
        toks = [[1] * max(1, self.cfg.warmup_tokens_per_req) for _ in range(n)]
        self.engine.generate(toks, max_new_tokens=1)

    def stop(self, drain: bool = True, timeout_s: float = 60.0) -> None:
        """Stop the step loop. With `drain`, requests already accepted finish first (up to
        timeout_s). Every request still queued or in flight then fails with "worker stopped". If
        the loop does not exit within timeout_s (a step is still running), the worker stays in
        DRAIN and its in-flight requests are left to the loop, which fails them when it exits:
        they are not touched here while a step may still use them. Calling stop again, or on a
        worker that never started, is harmless."""
        if self.state == WorkerState.TERMINATE:
            return
        self.lifecycle.drain()
        if drain:
            t0 = time.monotonic()
            while (self._inflight or not self._inbox.empty()) and time.monotonic() - t0 < timeout_s:
                if self._thread is None or not self._thread.is_alive():
                    break
                time.sleep(0.01)
        self._close_intake()
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=timeout_s)
            if self._thread.is_alive():
                LOG.warning("step loop still running after %.1fs; it fails its requests when it exits", timeout_s)
                return
        self._fail_all(PoolError(PoolErrorCode.DOWNSTREAM, "worker stopped"))
        self.lifecycle.terminate()

    def _close_intake(self) -> None:
        with self._intake:
            self._intake_open = False

    def _fail_all(self, err: Exception) -> None:
        self._fail_inflight(err)
        self._reject_inbound(err)

    @property
    def state(self) -> WorkerState:
        return self.lifecycle.state

    def capacity_signal(self) -> CapacitySignal:
        eng = self.engine
        waiting = len(eng.scheduler.waiting) if eng else 0
        running = len(eng.scheduler.running) if eng else 0
        return CapacitySignal(waiting=waiting + self._inbox.qsize(), running=running,
                              inflight_reqs=len(self._inflight),
                              max_running_reqs=eng.ec.max_running if eng else self.cfg.max_running_reqs,
                              state=self.state, role=self.cfg.role.value, model_backend=self.cfg.model_backend,
                              served_model_name=self.cfg.served_model_name, model_loaded=eng is not None,
                              model_warmed=self.state in (WorkerState.READY, WorkerState.SERVING))

    # ------------------------------------------------------------ requests
    def submit(self, rid: str, prompt: list[int], max_new_tokens: int, exec_mode: str = "",
               hint: PrefixHint | None = None, timeout_s: float | None = None) -> GenerateResult:
        if self._failed is not None:
            raise PoolError(PoolErrorCode.DOWNSTREAM, f"worker failed: {self._failed}")
        if not self.lifecycle.accepting:
            raise PoolError(PoolErrorCode.CAPACITY, f"worker not accepting requests ({self.state.value})")
        if not prompt:
            raise PoolError(PoolErrorCode.INVALID_ARG, "empty prompt")
        hint = hint or PrefixHint()
        mode = ExecMode(exec_mode) if exec_mode else select_exec_mode(hint, len(prompt), self.cfg.role)
        job = _Inbound(rid, list(prompt), int(max_new_tokens), mode, hint)
        with self._intake:
            if not self._intake_open:
                raise PoolError(PoolErrorCode.CAPACITY, f"worker not running ({self.state.value})")
            self._inbox.put(job)
        if not job.event.wait(timeout_s):
            raise PoolError(PoolErrorCode.TIMEOUT, f"request {rid} did not finish in {timeout_s}s")
        res = job.result
        if res.error is not None:
            raise res.error
        return res

    # ------------------------------------------------------------ loop
    def _drain_inbound(self, block: bool) -> None:
        first = True
        while True:
            try:
                job = self._inbox.get(timeout=COALESCE_S if (block and first) else 0.0) if block else \
                    self._inbox.get_nowait()
            except queue.Empty:
                return
            first = False
            try:
                if job.mode == ExecMode.PD_DISAGG and self.pd_side is not None:
                    local = self.pd_side.submit(job.prompt, job.max_new_tokens)
                    if local is None:
                        job.result = GenerateResult(job.rid, error=PoolError(
                            PoolErrorCode.CAPACITY, "no free KV pages for a prefill grant"))
                        job.event.set()
                        continue
                    if local.startswith("dd-"):  # the prefix is held here: prefilled locally
                        job.mode = ExecMode.D_DIRECT
                    self._engine_rid[job.rid] = local
                else:
                    self.engine.add_request(job.prompt, max_new_tokens=job.max_new_tokens, rid=job.rid)
                self._inflight[job.rid] = job
            except Exception as e:  # invalid request: fail just this one
                job.result = GenerateResult(job.rid, error=PoolError(PoolErrorCode.INVALID_ARG, str(e)))
                job.event.set()

    def _busy(self) -> bool:
        return self.engine.has_unfinished() or bool(self.pd_side is not None and self.pd_side.pending)

    def _loop(self) -> None:
        eng = self.engine
        try:
            self._run_steps(eng)
        finally:
            if self._stop.is_set():  # a stop that may have given up waiting: the loop cleans up
                self._close_intake()
                self._fail_all(PoolError(PoolErrorCode.DOWNSTREAM, "worker stopped"))
                self.lifecycle.terminate()

    def _run_steps(self, eng) -> None:
        while not self._stop.is_set():
            try:
                self._drain_inbound(block=not self._busy())
                if self.pd_side is not None:
                    self.pd_side.poll()  # prefilled requests join the decode batch
                if not eng.has_unfinished():
                    if self._busy():
                        time.sleep(0.0005)  # waiting on a prefill instance
                    continue
                eng.step()
                self.steps += 1
                self.metrics.steps.inc()
                self._complete_finished()
            except Exception as e:  # step failure: fail in-flight work and stop accepting
                LOG.exception("engine step failed")
                self.metrics.step_failures.inc()
                self._failed = e
                err = e if isinstance(e, PoolError) else PoolError(_step_error_code(e), str(e))
                self._close_intake()
                self._fail_all(err)
                self.lifecycle.drain()
                return

    def _complete_finished(self) -> None:
        bs = self.engine.ec.block_size
        for rid in list(self._inflight):
            req = self.engine.requests.get(self._engine_rid.get(rid, rid))
            if req is None or req.status not in (RequestStatus.FINISHED, RequestStatus.ABORTED):
                continue
            if req.output and req.output[-1] == PENDING:
                continue  # overlapped steps: its last token is still being sampled
            job = self._inflight.pop(rid)
            self._engine_rid.pop(rid, None)
            prefill_tokens = len(req.prompt) - req.num_cached
            job.result = GenerateResult(rid, list(req.output), req.num_cached // bs, (prefill_tokens + bs - 1) // bs,
                                        job.mode.value)
            self.metrics.observe_finished(req, job.mode.value)
            if self.on_finished is not None:
                self.on_finished(req)
            job.event.set()

    def _fail_inflight(self, err: Exception) -> None:
        for rid, job in list(self._inflight.items()):
            job.result = GenerateResult(rid, error=err)
            job.event.set()
        self._inflight.clear()

    def _reject_inbound(self, err: Exception) -> None:
        while True:
            try:
                job = self._inbox.get_nowait()
            except queue.Empty:
                return
            job.result = GenerateResult(job.rid, error=err)
            job.event.set()
