"""Stand-alone kv-pool byte service: TcpDataService (opaque block bytes keyed by model,
revision, pool kind and block hash) on LAKE_KV_ADDR (default 0.0.0.0:50052), for deployments
that run the byte store apart from the node services (which also serve it on their port).

    python -m lake_b200.services.kvpool

Reference parity: rust/kv-pool (lib.rs:34-83, main.rs:1-20).
"""
from __future__ import annotations

import logging
import os
from concurrent import futures

import grpc

from .. import _host as H
from ..api import proto
from .transfer import TcpDataServer

LOG = logging.getLogger("lake_b200.kvpool")


def serve(bind: str, max_workers: int = 16, capacity_bytes: int = 0):
    store = H.ByteStore(capacity_bytes)  # 0 = unbounded
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers), options=proto.message_options())
    proto.add_service(server, "TcpDataService", TcpDataServer(store))
    port = server.add_insecure_port(bind)
    server.start()
    return server, port


def main() -> None:
    logging.basicConfig(level=os.environ.get("LAKE_LOG", "INFO"))
    bind = os.environ.get("LAKE_KV_ADDR", "0.0.0.0:50052")
    cap = int(os.environ.get("LAKE_KV_CAPACITY_BYTES", "0") or 0)
    server, port = serve(bind, capacity_bytes=cap)
    LOG.info("kv-pool byte service on port %d", port)
    server.wait_for_termination()


if __name__ == "__main__":
    main()
