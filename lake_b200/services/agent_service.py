"""AgentService of a node's storage agent (router -> agent).

Dispatch requires a target node and is counted; ReportLoad acknowledges each
load report of the router's stream; both acks carry the most recent hard-quota
backpressure signal seen on this node's write path while it is fresh (30 s),
so the router pauses new starts of that model. PlaceBlocks hands the ids to a
placement callback (the node's warm-up path: promote those blocks toward L0).

Reference parity: rust/storage-agent/src/lib.rs:28-119.
"""
from __future__ import annotations

import threading

import grpc

from .. import _host as H
from ..api import proto
from . import convert as C

pb = proto.messages()
BACKPRESSURE_FRESH_TTL_S = 30.0


class AgentServer:
    def __init__(self, node_id: str = "node-0", place=None, backpressure: "H.BackpressureMemory | None" = None):
        self.node_id = node_id
        self.place = place  # callable(list[KVBlockID proto], target_node_id) or None
        self.bp = backpressure or H.BackpressureMemory(BACKPRESSURE_FRESH_TTL_S)
        self.dispatch_count = 0
        self.load_report_count = 0
        self.last_loads: dict[str, tuple[int, int, int]] = {}
        self._lock = threading.Lock()

    def _ack(self):
        return pb.Ack(ok=True, backpressure=C.bp_out(self.bp.fresh()))

    def Dispatch(self, request, context):
        if not request.target_node_id:
            context.abort(grpc.StatusCode.INVALID_ARGUMENT, "target_node_id required")
        with self._lock:
            self.dispatch_count += 1
        return self._ack()

    def ReportLoad(self, request_iterator, context):
        for rep in request_iterator:
            with self._lock:
                self.load_report_count += 1
                self.last_loads[rep.node_id] = (rep.queue_len, rep.in_flight, rep.remaining_cap)
            yield self._ack()

    def PlaceBlocks(self, request, context):
        if self.place is not None and request.ids:
            try:
                self.place(list(request.ids), request.target_node_id or self.node_id)
            except Exception as e:
                return pb.Ack(ok=False, err=str(e))
        return pb.Ack(ok=True)
