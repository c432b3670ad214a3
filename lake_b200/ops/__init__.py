"""Kernel-level ops. CUDA tensors run the sm_100a kernels in ``lake_b200._C``;
CPU tensors run the fp32 oracle (:mod:`lake_b200.oracle.ops_ref`)."""
from .core import (  # noqa: F401
    apply_token_bitmask,
    build_prefill_tiles,
    chain_reject_sample,
    decode_splits,
    embedding,
    greedy_from_keys,
    greedy_sample,
    linear,
    linear_argmax,
    linear_qkv,
    linear_residual,
    linear_swiglu,
    page_copy,
    paged_decode_attention,
    paged_prefill_attention,
    resolve_tokens,
    rms_norm,
)
from ..oracle.ops_ref import interleave_gate_up, rope_cache  # noqa: F401
from ._ext import available as native_available  # noqa: F401
