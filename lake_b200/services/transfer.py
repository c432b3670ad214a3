"""TransferService (batch / pull / publish) and TcpDataService (opaque byte
store) over the C++ TransferEngine and ByteStore.

SubmitTransfer validates every op (source tier L0/L1/L2, known segments,
ranges) before any byte moves; ops are executed by the engine (memcpy for
host-host, one cudaMemcpyAsync each otherwise). Pull copies the requested
blocks from the byte store into a fresh segment of the requester; the policy
decides completion: BEST_EFFORT skips missing blocks and completes,
WAIT_COMPLETE fails NOT_FOUND on a missing block, TIMEOUT caps the number of
pulled blocks at budget_ms (coarse stand-in for a latency budget) and reports
completed only when nothing was cut. Publish accumulates layer-wise slice
lengths per (request, block, layer) with a per-request sequence fence: a seq
below the last one is rejected, an equal seq is a resend and is deduplicated
slice by slice. FreePull / FreePublish release the session state.

Reference parity: rust/transfer/src/service.rs:113-337, bytes.rs,
kv-pool/src/lib.rs:28-82.
"""
from __future__ import annotations

import itertools
import threading

import grpc

from .. import _host as H
from ..api import proto

pb = proto.messages()
PULL_BEST_EFFORT, PULL_WAIT_COMPLETE, PULL_TIMEOUT = 0, 1, 2
STATE = {0: 0, 1: 1, 2: 2, 3: 3}  # TaskState -> TransferStatusResponse.State (same numbering)


def block_key(kid) -> bytes:
    return H.ByteStore.key(kid.model_id, kid.revision, int(kid.pool_kind), bytes(kid.block_hash))


class TransferServer:
    def __init__(self, engine: "H.TransferEngine | None" = None, store: "H.ByteStore | None" = None):
        self.engine = H.TransferEngine() if engine is None else engine
        self.store = H.ByteStore() if store is None else store
        self._pulls: dict[int, int] = {}  # handle -> dest segment
        self._pull_ids = itertools.count(1)
        self._publish: dict[str, dict] = {}
        self._lock = threading.Lock()

    # ---------------------------------------------------------------- batch API
    def SubmitTransfer(self, request, context):
        if not request.reqs:
            context.abort(grpc.StatusCode.INVALID_ARGUMENT, "empty transfer batch")
        ops = []
        for r in request.reqs:
            if not r.HasField("source"):
                context.abort(grpc.StatusCode.INVALID_ARGUMENT, "TransferRequest.source required")
            s = r.source
            if s.tier not in (1, 2, 3):
                context.abort(grpc.StatusCode.INVALID_ARGUMENT, f"invalid source tier {s.tier} (L0/L1/L2 only)")
            ops.append(H.TransferOp(s.tier, s.node_id, s.segment_id, s.offset, r.target_segment_id,
                                    r.target_offset, r.length))
        bid = self.engine.allocate_batch_id(len(ops))
        try:
            self.engine.submit_transfer(bid, ops)
        except Exception as e:
            self.engine.free_batch_id(bid)
            context.abort(grpc.StatusCode.INVALID_ARGUMENT, str(e))
        return pb.TransferBatchAck(batch_id=bid)

    def GetTransferStatus(self, request, context):
        try:
            st = self.engine.get_transfer_status(request.batch_id, request.task_id)
        except Exception as e:
            context.abort(grpc.StatusCode.NOT_FOUND, str(e))
        return pb.TransferStatusResponse(state=STATE[st.state], bytes_done=st.bytes_done)

    def FreeBatch(self, request, context):
        try:
            self.engine.free_batch_id(request.batch_id)
        except Exception:
            return pb.Ack(ok=False, err=f"unknown batch_id={request.batch_id}")
        return pb.Ack(ok=True)

    # ---------------------------------------------------------------- pull
    def Pull(self, request, context):
        policy = int(request.policy)
        cap = request.budget_ms if policy == PULL_TIMEOUT and request.budget_ms > 0 else None
        payloads = []
        for kid in request.ids:
            if cap is not None and len(payloads) >= cap:
                break
            data = self.store.get(block_key(kid))
            if data is None:
                if policy == PULL_WAIT_COMPLETE:
                    context.abort(grpc.StatusCode.NOT_FOUND,
                                  f"Pull WAIT_COMPLETE missing block hash_len={len(kid.block_hash)}")
                continue
            payloads.append(data)
        total = sum(len(d) for d in payloads)
        seg = self.engine.open_segment(f"pull-{request.requester_node_id}", max(1, total))
        off = 0
        for d in payloads:
            self.engine.write_segment(seg, off, d)
            off += len(d)
        pulled = len(payloads)
        if policy == PULL_WAIT_COMPLETE:
            completed = pulled == len(request.ids)
        elif policy == PULL_TIMEOUT:
            completed = pulled >= len(request.ids)
        else:
            completed = True
        with self._lock:
            handle = next(self._pull_ids)
            self._pulls[handle] = seg
        return pb.PullResponse(handle=handle, pulled_length=pulled, completed=completed)

    def pull_segment(self, handle: int) -> int:
        with self._lock:
            return self._pulls[handle]

    def FreePull(self, request, context):
        with self._lock:
            seg = self._pulls.pop(request.handle, None)
        if seg is None:
            return pb.Ack(ok=False, err=f"unknown pull handle={request.handle}")
        try:
            self.engine.free_segment(seg)
        except Exception:
            return pb.Ack(ok=True, err=f"pull handle={request.handle} freed; dest segment {seg} already gone")
        return pb.Ack(ok=True)

    # ---------------------------------------------------------------- publish
    def Publish(self, request, context):
        scope = request.request_id or "_"
        with self._lock:
            st = self._publish.setdefault(scope, {"last_seq": 0, "layers": {}, "seen": set()})
            if 0 < request.seq < st["last_seq"]:
                return pb.Ack(ok=False, err=f"Publish seq={request.seq} < last_seq={st['last_seq']} "
                                            f"(overlap fence, request_id={scope!r})")
            st["last_seq"] = max(st["last_seq"], request.seq)
            for sl in request.slices:
                if not sl.HasField("id"):
                    continue
                h = bytes(sl.id.block_hash)
                k = (h, sl.layer_idx, sl.offset)
                if k in st["seen"]:
                    continue
                st["seen"].add(k)
                st["layers"][(h, sl.layer_idx)] = st["layers"].get((h, sl.layer_idx), 0) + sl.length
        return pb.Ack(ok=True)

    def published_layer_bytes(self, request_id: str, block_hash: bytes, layer: int) -> int | None:
        with self._lock:
            st = self._publish.get(request_id or "_")
            return None if st is None else st["layers"].get((block_hash, layer))

    def FreePublish(self, request, context):
        scope = request.request_id or "_"
        with self._lock:
            removed = self._publish.pop(scope, None) is not None
        return pb.Ack(ok=removed, err="" if removed else f"unknown publish request_id={scope!r}")

    @property
    def publish_stream_count(self) -> int:
        return len(self._publish)

    @property
    def pull_handle_count(self) -> int:
        return len(self._pulls)


class TcpDataServer:
    """Opaque byte Put/Get keyed by (model_id, revision, pool_kind, block_hash)."""

    def __init__(self, store: "H.ByteStore | None" = None):
        self.store = H.ByteStore() if store is None else store

    def PutBlocks(self, request, context):
        skipped = 0
        for b in request.blocks:
            if not b.HasField("id"):
                skipped += 1
                continue
            self.store.put(block_key(b.id), bytes(b.data))
        return pb.Ack(ok=skipped == 0, err=f"skipped {skipped} block(s) without id" if skipped else "")

    def GetBlocks(self, request, context):
        out = []
        for kid in request.ids:
            d = self.store.get(block_key(kid))
            if d is not None:
                out.append(pb.OpaqueBlock(id=kid, data=d))
        return pb.GetBlocksResponse(blocks=out)
