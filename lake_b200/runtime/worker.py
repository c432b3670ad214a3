"""WorkerService gRPC facade of a compute worker.

Generate builds a request from the proto, consumes the router's execution
mode and reuse hint when present (empty exec_mode = a caller that did not go
through the router: COLOCATED, no reuse hint), submits it to the WorkerEngine
and maps pool errors onto gRPC status codes: TIMEOUT / DOWNSTREAM /
PROTOCOL_ERROR -> UNAVAILABLE (the router's signal to re-dispatch elsewhere),
CAPACITY -> RESOURCE_EXHAUSTED, INVALID_ARG -> INVALID_ARGUMENT.

Reference parity: python/lake/runtime/worker.py:42-162, __main__.py:18-23.
"""
from __future__ import annotations

import logging
import os
from concurrent import futures

import grpc

from ..api import proto
from ..pool.types import PoolError, PoolErrorCode, PrefixHint
from .config import RoleConfig
from .worker_engine import WorkerEngine

LOG = logging.getLogger("lake_b200.worker")

POOL_ERROR_STATUS = {
    PoolErrorCode.TIMEOUT: grpc.StatusCode.UNAVAILABLE,
    PoolErrorCode.DOWNSTREAM: grpc.StatusCode.UNAVAILABLE,
    PoolErrorCode.PROTOCOL_ERROR: grpc.StatusCode.UNAVAILABLE,
    PoolErrorCode.CAPACITY: grpc.StatusCode.RESOURCE_EXHAUSTED,
    PoolErrorCode.INVALID_ARG: grpc.StatusCode.INVALID_ARGUMENT,
}


class WorkerServicer:
    def __init__(self, engine: WorkerEngine):
        self.engine = engine
        self.pb = proto.messages()

    def Generate(self, request, context):
        hint = PrefixHint(computed_tokens=request.computed_tokens, reused_blocks=request.reused_blocks,
                          local_hit=request.local_hit)
        try:
            res = self.engine.submit(request.request_id, list(request.prompt_tokens),
                                     request.max_new_tokens or 16, request.exec_mode, hint)
        except PoolError as e:
            context.abort(POOL_ERROR_STATUS.get(e.code, grpc.StatusCode.INTERNAL), str(e))
        return self.pb.GenerateResponse(request_id=res.request_id, output_tokens=res.output_tokens,
                                        reused_blocks=res.reused_blocks, prefill_blocks=res.prefill_blocks,
                                        mode=res.mode)


def serve(bind: str = "0.0.0.0:50053", cfg: RoleConfig | None = None, pool=None, engine=None,
          max_workers: int = 8, block: bool = True, pool_factory=None, node_id: str = "worker-0"):
    cfg = cfg or RoleConfig.from_env()
    eng = WorkerEngine(cfg, pool=pool, engine=engine, node_id=node_id, pool_factory=pool_factory)
    eng.start()
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers))
    proto.add_service(server, "WorkerService", WorkerServicer(eng))
    port = server.add_insecure_port(bind)
    server.start()
    LOG.info("worker serving on %s (port %d)", bind, port)
    if block:
        try:
            server.wait_for_termination()
        finally:
            eng.stop(drain=False)
    return server, eng, port


def remote_pool_factory(cp_addr: str, kv_addr: str, node_id: str, model_id: str, pool_node_id: str = "kv-pool",
                        pull_budget_ms: float = 0.0, revision: str = ""):
    """pool_factory for a worker whose KV pool is the control plane at `cp_addr` plus the kv-pool
    byte service at `kv_addr`: prefix pages are pulled from the pool at admission and finished
    requests' pages are written back to it."""
    def make(engine):
        from ..pool.agents.remote import connect
        from ..pool.pool_iface import PoolIface

        agent = connect(engine, cp_addr, kv_addr, node_id=node_id, model_id=model_id, revision=revision,
                        pool_node_id=pool_node_id, pull_budget_ms=pull_budget_ms)
        return PoolIface(agent, node_id=node_id)
    return make


def main() -> None:
    """Environment: LAKE_WORKER_BIND, LAKE_NODE_ID, LAKE_WORKER_METRICS_ADDR (Prometheus endpoint),
    LAKE_TRACE_OUT (per-request JSONL trace), LAKE_CP_ADDR (control plane), LAKE_KV_ADDR
    (kv-pool byte service), LAKE_KV_NODE_ID (the pool node's id in the view, default kv-pool),
    LAKE_PULL_BUDGET_MS (0 = unbounded). With both addresses the worker's storage agent is the
    remote pool agent; with only LAKE_CP_ADDR it publishes its resident prefix blocks."""
    logging.basicConfig(level=os.environ.get("LAKE_LOG", "INFO"))
    cfg = RoleConfig.from_env()
    node_id = os.environ.get("LAKE_NODE_ID", "worker-0")
    cp_addr = os.environ.get("LAKE_CP_ADDR", "")
    kv_addr = os.environ.get("LAKE_KV_ADDR", "")
    factory = None
    if cp_addr and kv_addr:
        factory = remote_pool_factory(cp_addr, kv_addr, node_id, cfg.served_model_name,
                                      os.environ.get("LAKE_KV_NODE_ID", "kv-pool"), cfg.pull_budget_ms,
                                      cfg.model_revision)
    server, eng, port = serve(os.environ.get("LAKE_WORKER_BIND", "0.0.0.0:50053"), cfg, block=False,
                              pool_factory=factory, node_id=node_id)
    metrics_addr = os.environ.get("LAKE_WORKER_METRICS_ADDR", "")
    if metrics_addr:  # Prometheus: TTFT/TPOT/queue/e2e histograms, token and step counters
        from .metrics import serve_metrics

        serve_metrics(eng.metrics, metrics_addr)
    if cp_addr and factory is None:  # publish resident prefix blocks to the control plane's view
        from ..engine.llm_engine import page_bytes
        from .cp_reporter import ControlPlaneReporter

        e = eng.engine
        ch = grpc.insecure_channel(cp_addr)
        eng.on_finished = ControlPlaneReporter(
            proto.Stub(ch, "ControlPlaneService"), node_id,
            cfg.served_model_name, page_bytes(e.cfg, e.ec.block_size, e.arena.element_size()), e.ec.block_size,
            e.cfg.n_layers)
    try:
        server.wait_for_termination()
    finally:
        eng.stop(drain=False)


if __name__ == "__main__":
    main()
