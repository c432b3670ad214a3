"""Tensor-parallel fused ops (GPU only): column-parallel GEMMs that wait for
all-gathered row shards, row-parallel GEMMs whose epilogue performs the
reduce-scatter, and the reduce + residual + RMSNorm + all-gather kernel.
The ``tp`` dicts come from lake_b200.parallel.tp.TPGroup."""
from __future__ import annotations

from ._ext import native
from .core import LAUNCHES, status_word
from .fp8 import unpack


def linear_qkv_ag(a, w_qkv, q_out, rope_cs, positions, slots, arena, layer, n_q_heads, n_kv_heads, tp: dict,
                  peer_arena=None, peer_slots=None):
    wq, ws = unpack(w_qkv)
    native().linear_qkv(a, wq, q_out, rope_cs, positions, slots, arena, layer, n_q_heads, n_kv_heads,
                        peer_arena, peer_slots, status_word(a.device), tp, None, None, 1e-6, ws)
    LAUNCHES[0] += 1
    return q_out


def linear_swiglu_ag(a, w_gate_up, out, tp: dict):
    wq, ws = unpack(w_gate_up)
    native().linear_swiglu(a, wq, out, status_word(a.device), tp, ws)
    LAUNCHES[0] += 1
    return out


def linear_rs(a, w, tp: dict):
    wq, ws = unpack(w)
    native().linear_rs(a, wq, tp, status_word(a.device), ws)
    LAUNCHES[0] += 1


def norm_push(h, w, eps, tp: dict):
    native().tp_norm_push(h, w, eps, tp, status_word(h.device))
    LAUNCHES[0] += 1


def linear_argmax_tp(a, w, keys, tp: dict):
    wq, ws = unpack(w)
    native().linear_argmax(a, wq, keys, None, status_word(a.device), tp, ws)
    LAUNCHES[0] += 2  # memset of the keys + GEMM
