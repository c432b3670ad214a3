"""Peer-memory fabric: share one process's KV arena with the other processes of
the box so their kernels can store into it directly.

On the GPU the arena's allocation is exported as a CUDA IPC handle and mapped
into the peer's context (NVLink 5 / NVSwitch P2P): a kernel on the prefill GPU
then writes K/V rows into the decode GPU's pages with ordinary global stores.
On the CPU path the arena lives in a /dev/shm file both processes map.

Reference parity: replaces the Transport/segment registration of the reference's
transfer engine (rust/transfer/src/transport.rs:47-68, tcp.rs:185-301), which
copies bytes between in-process segments.
"""
from __future__ import annotations

import os
import uuid

import torch


def alloc_shared_cpu_arena(shape, dtype, name: str | None = None) -> tuple[torch.Tensor, str]:
    """Zero-filled CPU tensor backed by a /dev/shm file (mappable by other processes)."""
    n = 1
    for d in shape:
        n *= d
    path = f"/dev/shm/lakeb_{name or uuid.uuid4().hex}"
    t = torch.from_file(path, shared=True, size=n, dtype=dtype)
    t.zero_()
    return t.view(*shape), path


def alloc_ipc_arena(shape, dtype, device) -> torch.Tensor:
    """Zero-filled device tensor in its own cudaMalloc allocation, exportable with export_tensor."""
    from ..ops._ext import native

    with torch.cuda.device(device):
        return native().alloc_ipc_tensor(list(shape), dtype)


def export_tensor(t: torch.Tensor, shm_path: str | None = None):
    """Picklable handle from which another process can map `t` (CUDA tensors must come from
    alloc_ipc_arena so the IPC handle covers exactly the tensor)."""
    if t.is_cuda:
        from ..ops._ext import native

        return ("cuda", native().ipc_export(t), tuple(t.shape), t.dtype, t.device.index)
    if shm_path is None:
        raise ValueError("CPU tensors are shared through their /dev/shm path")
    return ("cpu", shm_path, tuple(t.shape), t.dtype)


def import_tensor(handle) -> torch.Tensor:
    kind = handle[0]
    if kind == "cuda":
        # Opened with this process's current device current: its kernels address the
        # peer GPU's memory through the mapping (P2P over NVLink).
        from ..ops._ext import native

        _, h, shape, dtype, _owner = handle
        return native().ipc_import(h, list(shape), dtype)
    _, path, shape, dtype = handle
    n = 1
    for d in shape:
        n *= d
    return torch.from_file(path, shared=True, size=n, dtype=dtype).view(*shape)


def unlink_shared(path: str) -> None:
    try:
        os.unlink(path)
    except OSError:
        pass


def enable_peer_access(dev_a: int, dev_b: int) -> bool:
    """True if device dev_a can address dev_b's memory directly."""
    if not torch.cuda.is_available():
        return False
    return bool(torch.cuda.can_device_access_peer(dev_a, dev_b))
