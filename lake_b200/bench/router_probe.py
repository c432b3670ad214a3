"""Router latency probe: the real HTTP handler, admission queue and mode selection in front of a
stand-in worker that answers Generate after a fixed delay, driven by concurrent chat requests.

    python -m lake_b200.bench.router_probe [--requests 96] [--max-inflight 4] [--worker-delay-ms 2]

JSON lines on stdout (and appended to LAKE_BENCH_OUT when set):

* ``router_e2e_latency``: p50/p99 ms from POST to the complete response (the stand-in worker
  answers at once after its delay, so this is not a time to first token);
* ``router_queue_wait``: p50/p99 ms the admission queue held requests (PQScheduler samples);
* ``router_mode_distribution``: requests per execution mode, and the achieved request rate.

The control plane is the real service over loopback gRPC; the agent is the real AgentService.

Reference parity: go/router/bench_p71_test.go:72-166 (bufconn fake worker/agent, 96 requests,
4 in flight, 2 ms generate).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import time
from concurrent import futures

import grpc

from ..api import proto
from ..utils.trace import emit

pb = proto.messages()


class DelayWorker:
    """WorkerService stand-in: sleeps `delay_s`, echoes the request's execution mode."""

    def __init__(self, delay_s: float):
        self.delay_s = delay_s

    def Generate(self, request, context):
        time.sleep(self.delay_s)
        return pb.GenerateResponse(request_id=request.request_id, output_tokens=[1, 2, 3, 4],
                                   mode=request.exec_mode)


def _pct(xs, q):
    if not xs:
        return 0.0
    xs = sorted(xs)
    return xs[int(q * (len(xs) - 1))]


def run(requests: int = 96, max_inflight: int = 4, delay_ms: float = 2.0) -> list[dict]:
    from aiohttp.test_utils import TestClient, TestServer

    from ..router.http import make_app
    from ..router.server import Router, RouterConfig
    from ..services.agent_service import AgentServer
    from ..services.controlplane import ControlPlane

    cp = ControlPlane()
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max(16, 2 * max_inflight)))
    proto.add_service(server, "ControlPlaneService", cp)
    proto.add_service(server, "AgentService", AgentServer("worker-0"))
    proto.add_service(server, "WorkerService", DelayWorker(delay_ms / 1000.0))
    port = server.add_insecure_port("127.0.0.1:0")
    server.start()
    addr = f"127.0.0.1:{port}"
    cfg = RouterConfig(worker_addr=addr, agent_addr=addr, cp_addr=addr, max_inflight=max_inflight,
                       request_timeout_s=60)
    lat: list[float] = []

    async def drive():
        router = Router(cfg)
        async with TestClient(TestServer(make_app(router))) as client:
            async def one(i):
                t0 = time.perf_counter()
                body = {"model": "m", "messages": [{"role": "u", "content": f"{i} hello world prefix tokens here"}],
                        "max_tokens": 4}
                r = await client.post("/v1/chat/completions", json=body)
                await r.read()
                if r.status != 200:
                    raise RuntimeError(f"request {i}: HTTP {r.status}")
                lat.append((time.perf_counter() - t0) * 1000)

            t0 = time.perf_counter()
            await asyncio.gather(*(one(i) for i in range(requests)))
            wall = time.perf_counter() - t0
            waits = [w * 1000 for w in router.pq.wait_samples()]
            modes = dict(router.mode_counts)
        return wall, waits, modes

    try:
        wall, waits, modes = asyncio.run(drive())
    finally:
        cp.stop()
        server.stop(0)
    env = {"transport": "loopback gRPC", "compute": f"stand-in worker, {delay_ms:g} ms per Generate",
           "max_inflight": max_inflight}
    return [
        {"name": "router_e2e_latency", "env": env, "latency_ms": {"p50": _pct(lat, .5), "p99": _pct(lat, .99)},
         "counters": {"requests": requests}},
        {"name": "router_queue_wait", "env": env, "latency_ms": {"p50": _pct(waits, .5), "p99": _pct(waits, .99)},
         "counters": {"samples": len(waits)}},
        {"name": "router_mode_distribution", "env": env,
         "counters": {"requests": requests, **{f"mode_{k}": v for k, v in modes.items()}},
         "req_per_s": requests / wall},
    ]


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=96)
    ap.add_argument("--max-inflight", type=int, default=4)
    ap.add_argument("--worker-delay-ms", type=float, default=2.0)
    args = ap.parse_args(argv)
    for rec in run(args.requests, args.max_inflight, args.worker_delay_ms):
        print(json.dumps(rec))
        emit(rec)


if __name__ == "__main__":
    main()
