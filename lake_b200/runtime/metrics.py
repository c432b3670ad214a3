"""Worker-side observability: Prometheus metrics and a per-request trace.

Metrics (one registry per worker, served over HTTP by ``serve_metrics`` on
``LAKE_WORKER_METRICS_ADDR``, e.g. ``0.0.0.0:9101``):

* histograms ``lake_worker_ttft_seconds`` (arrival -> first token),
  ``lake_worker_tpot_seconds`` (mean gap between a request's output tokens),
  ``lake_worker_queue_seconds`` (arrival -> pages granted) and
  ``lake_worker_e2e_seconds`` (arrival -> finish), labelled by execution mode;
* counters of finished requests (by mode), output tokens, prompt tokens prefilled and
  reused from the prefix cache, engine steps and failed steps;
* gauges of running / waiting requests, sampled at scrape time.

Trace: with ``LAKE_TRACE_OUT`` set, every finished request appends one JSON line with its
stage timestamps (seconds, perf_counter clock of the worker: arrival, admitted, first token,
finish), token counts, execution mode and reused / prefilled blocks.

Reference parity: the router-side histogram of go/router/metrics.go; the reference worker
exposes no metrics of its own.
"""
from __future__ import annotations

import json
import os
import threading

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, start_http_server

LATENCY_BUCKETS = (0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0)
TPOT_BUCKETS = (0.001, 0.0025, 0.005, 0.01, 0.02, 0.035, 0.05, 0.075, 0.1, 0.2, 0.5)


class WorkerMetrics:
    def __init__(self, node_id: str = "worker-0", engine=None, trace_path: str | None = None):
        self.node_id = node_id
        self.registry = CollectorRegistry()
        r = self.registry
        self.ttft = Histogram("lake_worker_ttft_seconds", "arrival to first output token", ["mode"],
                              buckets=LATENCY_BUCKETS, registry=r)
        self.tpot = Histogram("lake_worker_tpot_seconds", "mean time per output token after the first", ["mode"],
                              buckets=TPOT_BUCKETS, registry=r)
        self.queue = Histogram("lake_worker_queue_seconds", "arrival to KV pages granted", ["mode"],
                               buckets=LATENCY_BUCKETS, registry=r)
        self.e2e = Histogram("lake_worker_e2e_seconds", "arrival to the last output token", ["mode"],
                             buckets=LATENCY_BUCKETS, registry=r)
        self.finished = Counter("lake_worker_requests_finished", "finished requests", ["mode"], registry=r)
        self.out_tokens = Counter("lake_worker_output_tokens", "output tokens of finished requests", registry=r)
        self.prefill_tokens = Counter("lake_worker_prefill_tokens", "prompt tokens computed", registry=r)
        self.reused_tokens = Counter("lake_worker_reused_tokens", "prompt tokens served from the prefix cache",
                                     registry=r)
        self.steps = Counter("lake_worker_steps", "engine steps", registry=r)
        self.step_failures = Counter("lake_worker_step_failures", "engine steps that raised", registry=r)
        self.engine = engine
        running = Gauge("lake_worker_running_requests", "requests in the running batch", registry=r)
        waiting = Gauge("lake_worker_waiting_requests", "requests waiting for admission", registry=r)
        running.set_function(lambda: len(self.engine.scheduler.running) if self.engine else 0)
        waiting.set_function(lambda: len(self.engine.scheduler.waiting) if self.engine else 0)
        self.trace_path = trace_path if trace_path is not None else os.environ.get("LAKE_TRACE_OUT", "")
        self._lock = threading.Lock()

    def observe_finished(self, req, mode: str) -> None:
        ttft, tpot = req.ttft(), req.tpot()
        if ttft is not None:
            self.ttft.labels(mode).observe(ttft)
        if tpot is not None:
            self.tpot.labels(mode).observe(tpot)
        if req.admit_time is not None:
            self.queue.labels(mode).observe(max(0.0, req.admit_time - req.arrival))
        end = req.finish_time or (req.token_times[-1] if req.token_times else None)
        if end is not None:
            self.e2e.labels(mode).observe(max(0.0, end - req.arrival))
        self.finished.labels(mode).inc()
        self.out_tokens.inc(len(req.output))
        self.prefill_tokens.inc(max(0, len(req.prompt) - req.num_cached))
        self.reused_tokens.inc(req.num_cached)
        if self.trace_path:
            self._trace(req, mode, end)

    def _trace(self, req, mode: str, end) -> None:
        bs = self.engine.ec.block_size if self.engine is not None else 16
        rec = {"request_id": req.rid, "node": self.node_id, "mode": mode, "prompt_tokens": len(req.prompt),
               "output_tokens": len(req.output), "reused_blocks": req.num_cached // bs,
               "prefill_blocks": (len(req.prompt) - req.num_cached + bs - 1) // bs,
               "t_arrival": req.arrival, "t_admitted": req.admit_time, "t_first_token": req.first_token_time,
               "t_finish": end, "ttft_s": req.ttft(), "tpot_s": req.tpot()}
        with self._lock, open(self.trace_path, "a") as f:
            f.write(json.dumps(rec) + "\n")


def serve_metrics(metrics: WorkerMetrics, addr: str):
    """Serve the registry at http://addr/metrics; returns (server, thread)."""
    host, _, port = addr.rpartition(":")
    return start_http_server(int(port), addr=host or "0.0.0.0", registry=metrics.registry)
