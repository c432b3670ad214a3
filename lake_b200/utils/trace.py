"""Tracing and probe output.

* ``nvtx(name)`` - an NVTX range around a region (engine step, layer, collective)
  when ``LAKEB_NVTX=1``; a no-op context otherwise, so the hot loop pays nothing.
* ``emit(record)`` - append one JSON line to the file named by ``LAKE_BENCH_OUT``
  (the reference's bench probe sink), when set.
"""
from __future__ import annotations

import contextlib
import json
import os

ENABLED = os.environ.get("LAKEB_NVTX", "") in ("1", "true")


@contextlib.contextmanager
def _range(name: str):
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx(name: str):
    return _range(name) if ENABLED else contextlib.nullcontext()


def emit(record: dict) -> None:
    path = os.environ.get("LAKE_BENCH_OUT")
    if not path:
        return
    with open(path, "a") as f:
        f.write(json.dumps(record) + "\n")
