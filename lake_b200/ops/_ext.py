"""Loader for the native kernel module ``lake_b200._C``.

CUDA tensors always go to the native kernels; if the extension is missing the
call raises instead of falling back, so a GPU run can never silently use a
PyTorch path. CPU tensors use the fp32 reference implementations in
:mod:`lake_b200.oracle.ops_ref` (the correctness oracle).
"""
from __future__ import annotations

import importlib
import os

_C = None
_ERR: Exception | None = None


def native():
    """Return the compiled module or raise with the build instruction."""
    global _C, _ERR
    if _C is None:
        try:
            # LAKEB_DEBUG_CHECKS=1: the bounds-checked build (python -m lake_b200._build --debug)
            debug = os.environ.get("LAKEB_DEBUG_CHECKS", "0") not in ("", "0")
            _C = importlib.import_module("lake_b200._C_debug" if debug else "lake_b200._C")
            # two-SM tcgen05 GEMM for large plain projections (LAKEB_GEMM_PAIR=0 turns it off)
            _C.set_gemm_pair_mode(int(os.environ.get("LAKEB_GEMM_PAIR", "1") or 0))
            _C.set_gemm_streamk_mode(int(os.environ.get("LAKEB_GEMM_STREAMK", "1") or 0))
            _C.set_decode_split_mode(int(os.environ.get("LAKEB_DECODE_SPLITS", "0") or 0))
            _C.set_prefill_kernel(int(os.environ.get("LAKEB_PREFILL_KERNEL", "1") or 0))
        except ImportError as e:  # pragma: no cover - depends on the build
            _ERR = e
            raise RuntimeError(
                "lake_b200._C is not built (python -m lake_b200._build); CUDA ops have no fallback"
            ) from e
    return _C


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False
