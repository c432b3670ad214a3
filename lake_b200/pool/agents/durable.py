"""Durable tier behind a host-cache agent: L1 pages committed to L2 with PutEnd, off the engine
thread.

When a request finishes, its full pages are in the agent's pinned L1 slab (written there by the
QKV epilogue, or by the write-behind copy). The agent hands the request's page chain to
``commit``: the chain's already-durable blocks and the new ones with their L1 slots. A
background thread then runs one PutEnd session per request (``csrc/host/agent``): it copies
each new block's bytes out of its L1 slot, writes them as checksummed, fdatasync'd L2 records
of the tier engine, registers them with the location authority (L1 on this node and L2), cycles
their references and completes the request barrier. A slot stays pinned (not evictable from L1)
until its bytes have been copied into the session, and a copy still in flight on the
write-behind stream is waited for first.

``read_into`` brings an L2 block back into host memory for the agent's promotion path when L1
no longer holds it (the record is validated on read; a failed read counts as a miss).

Reference parity: the PutEnd protocol of rust/storage-agent/src/putend.rs:193-382 and the
storage agent's durable write-back (python/lake/engine/agents/grpc_skeleton.py:177-253), with
real segment files instead of in-memory maps.
"""
from __future__ import annotations

import os
import queue
import tempfile
import threading
import time

from ... import _host as H


class DurableTier:
    def __init__(self, model_id: str, page_bytes: int, num_layers: int, block_size: int, l2_blocks: int = 4096,
                 storage_dir: str | None = None, node_id: str = "node-0", authority: "H.Authority | None" = None,
                 revision: str = ""):
        self.model_id, self.revision, self.node_id = model_id, revision, node_id
        self.page_bytes = page_bytes
        self.authority = authority or H.Authority()
        if not self.authority.has_namespace(model_id, revision):
            self.authority.register_model(H.ModelDescriptor(model_id, revision, num_layers, block_size, page_bytes))
        self.port = H.AuthorityPort(self.authority)
        root = storage_dir or tempfile.mkdtemp(prefix="lakeb_durable_")
        # L2/L3 only: the agent's slab is the L1 tier, so the tier engine keeps no slots of its own
        self.tiers = H.TierEngine(H.TierCaps(1, 0, l2_blocks), page_bytes, 0, os.path.join(root, "l2"),
                                  os.path.join(root, "l3"), model_id)
        self.lock = threading.Lock()  # the tier engine and the authority are used from two threads
        self.durable: set[bytes] = set()
        self.stats = {"durable_blocks": 0, "durable_ms": 0.0, "sessions": 0, "l2_reads": 0, "failed_sessions": 0}
        self._q: "queue.Queue" = queue.Queue()
        self._thread = threading.Thread(target=self._run, name="lakeb-durable", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------ engine thread
    def commit(self, rid: str, chain: list[tuple[bytes, int, int, bool]], ready, unpin) -> None:
        """Queue one request's page chain, in order: (hash, pinned L1 slot, its host address,
        already durable). `ready` (a CUDA event or None) orders the reads after the write-behind
        copy; `unpin(slot)` runs for every slot of the chain once its bytes are no longer needed."""
        self._q.put((rid, chain, ready, unpin))

    def is_durable(self, h: bytes) -> bool:
        return h in self.durable

    def read_into(self, h: bytes, dst_addr: int) -> bool:
        with self.lock:
            ok = self.tiers.read_host(h, dst_addr)
        if ok:
            self.stats["l2_reads"] += 1
        return ok

    def flush(self, timeout_s: float = 60.0) -> None:
        """Wait until every queued session has been committed."""
        done = threading.Event()
        self._q.put(done)
        done.wait(timeout_s)

    def close(self) -> None:
        self._q.put(None)
        self._thread.join(timeout=60)

    # ------------------------------------------------------------ background thread
    def _run(self) -> None:
        while True:
            item = self._q.get()
            if item is None:
                return
            if isinstance(item, threading.Event):
                item.set()
                continue
            rid, chain, ready, unpin = item
            t0 = time.perf_counter()
            if ready is not None:
                ready.synchronize()
            sess = H.PutEndSession(rid, self.node_id, self.model_id, self.revision)
            new = []
            for h, slot, addr, dur in chain:
                if dur and not new:
                    sess.add_prefix(h)  # durable already: only its place in the chain
                else:  # new, or durable after a new block (the session needs a contiguous chain)
                    sess.put_start_ptr(h, addr, self.page_bytes)
                    new.append(h)
                unpin(slot)
            if not new:
                continue
            try:
                with self.lock:
                    sess.commit_through(self.port, self.tiers)
                self.durable.update(new)
                self.stats["durable_blocks"] += len(new)
                self.stats["sessions"] += 1
            except Exception:  # quota / capacity refusals leave the blocks in L1 only
                self.stats["failed_sessions"] += 1
            self.stats["durable_ms"] += (time.perf_counter() - t0) * 1000
