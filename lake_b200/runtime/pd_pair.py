"""A PD-split serving pair on one machine: a prefill instance and a decode worker that serves
WorkerService.

The decode worker runs PD_DISAGG requests through parallel.pd: it reserves pages in its own KV
arena, grants them to the prefill instance, whose QKV epilogue writes the prompt's K/V into
them (GPU peer memory; a shared-memory arena file on the CPU), and adopts the request into its
decode batch with the first token the prefill instance sampled. D_DIRECT requests (or a prompt
whose prefix the decode worker already holds) and COLOCATED ones run on the decode worker.

    python -m lake_b200.runtime.pd_pair --bind 0.0.0.0:50053            # LAKE_* role settings
    LAKE_MODEL_BACKEND=mock python -m lake_b200.runtime.pd_pair --bind 127.0.0.1:50053   # CPU

The two processes meet through torch.distributed (gloo, 127.0.0.1) only to exchange the arena
handle; control messages use shared-memory rings. SIGTERM / SIGINT stops both.
"""
from __future__ import annotations

import argparse
import logging
import os
import signal
import socket
import threading

import torch.multiprocessing as mp

LOG = logging.getLogger("lake_b200.pd_pair")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank: int, port: int, bind: str, job: str, device_base: int) -> None:
    import grpc
    import torch
    import torch.distributed as dist
    from concurrent import futures

    from ..api import proto
    from ..parallel import pd
    from .config import RoleConfig
    from .worker import WorkerServicer
    from .worker_engine import WorkerEngine, build_engine

    logging.basicConfig(level=os.environ.get("LAKE_LOG", "INFO"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    cfg = RoleConfig.from_env()
    if cfg.device.startswith("cuda"):
        cfg.device = f"cuda:{device_base + rank}"
        torch.cuda.set_device(device_base + rank)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    role = "prefill" if rank == 0 else "decode"
    # the prefill instance reports each first token as soon as its step completes (no overlap)
    eng = build_engine(cfg, shared_arena=role == "decode", **({} if role == "decode" else {"overlap": False}))
    side = pd.connect_pair(eng, role, rank, 1 if role == "prefill" else [0], None, job=job,
                           shm_path=getattr(eng, "arena_path", None))
    if role == "prefill":
        pd.serve_prefill(side)
        side.close()
        dist.destroy_process_group()
        return
    we = WorkerEngine(cfg, engine=eng)
    we.pd_side = side
    we.start()
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=8))
    proto.add_service(server, "WorkerService", WorkerServicer(we))
    bound = server.add_insecure_port(bind)
    server.start()
    LOG.info("PD decode worker serving on %s (port %d)", bind, bound)
    stop = threading.Event()
    for sig in (signal.SIGTERM, signal.SIGINT):
        signal.signal(sig, lambda *_: stop.set())
    stop.wait()
    server.stop(1)
    we.stop(drain=False)
    side.shutdown()
    side.close()
    dist.destroy_process_group()
    if getattr(eng, "arena_path", None):
        from ..parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--bind", default=os.environ.get("LAKE_WORKER_BIND", "0.0.0.0:50053"))
    ap.add_argument("--device-base", type=int, default=0, help="GPU of the prefill instance; decode uses the next")
    a = ap.parse_args(argv)
    job = f"pair{os.getpid()}"
    ctx = mp.get_context("spawn")
    port = _free_port()
    prefill = ctx.Process(target=_run, args=(0, port, a.bind, job, a.device_base), daemon=True)
    prefill.start()
    _run(1, port, a.bind, job, a.device_base)  # returns after SIGTERM / SIGINT, having stopped the prefill side
    prefill.join(timeout=30)


if __name__ == "__main__":
    main()
