"""Node-side storage services in one process: AgentService, TransferService
and TcpDataService (the kv-pool byte store) on one gRPC port, sharing one
C++ byte store and transfer engine."""
from __future__ import annotations

import logging
import os
from concurrent import futures

import grpc

from ..api import proto
from .agent_service import AgentServer
from .transfer import TcpDataServer, TransferServer

LOG = logging.getLogger("lake_b200.node")


def serve(bind: str, node_id: str = "worker-0", max_workers: int = 16):
    ts = TransferServer()
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers), options=proto.message_options())
    proto.add_service(server, "AgentService", AgentServer(node_id))
    proto.add_service(server, "TransferService", ts)
    proto.add_service(server, "TcpDataService", TcpDataServer(ts.store))
    port = server.add_insecure_port(bind)
    server.start()
    return server, port


def main() -> None:
    logging.basicConfig(level=os.environ.get("LAKE_LOG", "INFO"))
    bind = os.environ.get("LAKE_AGENT_BIND", os.environ.get("LAKE_AGENT_ADDR", "0.0.0.0:50054"))
    server, port = serve(bind, os.environ.get("LAKE_NODE_ID", "worker-0"))
    LOG.info("node services (agent/transfer/tcp-data) on port %d", port)
    server.wait_for_termination()


if __name__ == "__main__":
    main()
