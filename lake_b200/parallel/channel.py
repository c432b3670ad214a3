"""Single-producer / single-consumer message ring in shared host memory.

Used for the control messages between a decode instance and its prefill
partner (page grants one way, "prefill done" the other). Messages are int64
arrays; the ring stores [length, payload...] records and publishes them by
advancing the head index after the payload is written (x86 stores are not
reordered with other stores, and Python executes them in program order).
"""
from __future__ import annotations

import time
from multiprocessing import shared_memory

import numpy as np

HDR = 8  # head, tail, ... (int64 slots)


def _untrack(shm) -> None:
    """An attaching process must not unlink the segment at exit (its own resource tracker
    would). A process spawned by the creator shares the creator's tracker instead (it inherited
    the tracker's pipe and did not start one: `_fd` set, `_pid` unset); unregistering there would
    drop the creator's entry, and the creator's unlink would then fail inside the tracker."""
    try:
        from multiprocessing import resource_tracker

        rt = resource_tracker._resource_tracker
        if getattr(rt, "_fd", None) is not None and getattr(rt, "_pid", None) is None:
            return
        resource_tracker.unregister(shm._name, "shared_memory")
    except Exception:  # pragma: no cover - tracker layout differs across Python versions
        pass


class ShmRing:
    def __init__(self, name: str, capacity_words: int = 1 << 20, create: bool = False):
        self.name = name
        self.cap = capacity_words
        size = (HDR + capacity_words) * 8
        if create:
            try:
                old = shared_memory.SharedMemory(name=name)
                old.close()
                old.unlink()
            except FileNotFoundError:
                pass
            self.shm = shared_memory.SharedMemory(name=name, create=True, size=size)
            self.buf = np.ndarray((HDR + capacity_words,), dtype=np.int64, buffer=self.shm.buf)
            self.buf[:] = 0
        else:
            self.shm = shared_memory.SharedMemory(name=name)
            self.buf = np.ndarray((HDR + capacity_words,), dtype=np.int64, buffer=self.shm.buf)
            _untrack(self.shm)  # the creating process owns the name and unlinks it
        self.owner = create

    # head: total words written; tail: total words consumed
    def put(self, payload) -> bool:
        p = np.asarray(payload, dtype=np.int64)
        n = int(p.shape[0]) + 1
        head, tail = int(self.buf[0]), int(self.buf[1])
        if head + n - tail > self.cap:
            return False
        rec = np.empty(n, dtype=np.int64)
        rec[0] = n - 1
        rec[1:] = p
        self._write(head, rec)
        self.buf[0] = head + n
        return True

    def _write(self, pos: int, rec: np.ndarray) -> None:
        start = pos % self.cap
        first = min(rec.shape[0], self.cap - start)
        self.buf[HDR + start:HDR + start + first] = rec[:first]
        if first < rec.shape[0]:
            self.buf[HDR:HDR + rec.shape[0] - first] = rec[first:]

    def _read(self, pos: int, n: int) -> np.ndarray:
        start = pos % self.cap
        first = min(n, self.cap - start)
        out = np.empty(n, dtype=np.int64)
        out[:first] = self.buf[HDR + start:HDR + start + first]
        if first < n:
            out[first:] = self.buf[HDR:HDR + n - first]
        return out

    def put_wait(self, payload, timeout_s: float = 30.0) -> None:
        t0 = time.monotonic()
        while not self.put(payload):
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"ring {self.name} full for {timeout_s}s (consumer stalled?)")
            time.sleep(0.0001)

    def get(self):
        head, tail = int(self.buf[0]), int(self.buf[1])
        if head == tail:
            return None
        n = int(self.buf[HDR + tail % self.cap])
        out = self._read(tail + 1, n)
        self.buf[1] = tail + 1 + n
        return out

    def close(self):
        if self.buf is None:
            return
        self.buf = None
        self.shm.close()
        if self.owner:
            try:
                self.shm.unlink()
            except FileNotFoundError:
                pass
