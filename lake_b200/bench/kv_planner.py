"""KV planning calculator: prefix-hit load bandwidth, pool capacity and hit-rate economics
for this framework's model families (CPU arithmetic, no GPU).

Three questions, each answered for a model configuration and a paged-KV block size:

  prefill   How many KV bytes must a prefill instance load per request (and per second)
            when a fraction `hit` of each request's context is a prefix held in the pool,
            `remote` of it on another node? Request rate comes either from a measured
            unique-token throughput per GPU (compute-bound prefill) or is given.
  capacity  How much pool capacity do `users` retained sessions plus the KV the prefill
            GPUs generate over 5 / 30 / 60 minutes take, logical and raw (copies and the
            usable fraction of raw media)?
  compare   Two hit rates side by side: compute-bound request rate, load bandwidth and
            capacity, with relative increases.

Bytes are counted two ways: logical (layers x 2 x kv_heads x head_dim x element bytes per
token) and page-allocated (whole blocks of `block` tokens, the arena's unit).

Reference parity: the analytical pages of tools/cmx-sim (sim.js prefillScenario :445,
capacityScenario :621, hitComparisonScenario :745, matchedTokens :427), which cover other
model representations; the browser front end is not reproduced.

    python -m lake_b200.bench.kv_planner prefill --model llama3-8b --context 8192 --hit 0.9 --tps-gpu 70000
"""
from __future__ import annotations

import argparse
import json
import math

from ..models.config import ModelConfig, get_config

WINDOWS_S = (300, 1800, 3600)


def kv_bytes_per_token(cfg: ModelConfig, elem_bytes: int = 2) -> int:
    return cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * elem_bytes


def kv_bytes(cfg: ModelConfig, tokens: int, block: int = 16, elem_bytes: int = 2) -> dict:
    """Logical and page-allocated KV bytes of `tokens` tokens."""
    per = kv_bytes_per_token(cfg, elem_bytes)
    pages = math.ceil(max(0, tokens) / block)
    return {"tokens": tokens, "logical": tokens * per, "pages": pages, "allocated": pages * block * per}


def matched_tokens(context: int, hit: float, block: int) -> int:
    """Prefix tokens a hit rate can reuse: whole blocks only (a partial block is recomputed)."""
    context = max(0, int(context))
    hit = min(1.0, max(0.0, hit))
    blocks = math.floor(context * hit / block + 1e-9)
    return min(context, blocks * block)


def prefill(cfg: ModelConfig, context: int, hit: float, block: int = 16, extra: int = 0, remote: float = 1.0,
            gpus: int = 1, tps_gpu: float | None = None, req_s: float | None = None, elem_bytes: int = 2) -> dict:
    """Per-request and aggregate KV load of prefill instances."""
    matched = matched_tokens(context, hit, block)
    unique = context - matched + extra
    if req_s is None and tps_gpu is not None:
        req_s = (gpus * tps_gpu / unique) if unique > 0 else None
    load = kv_bytes(cfg, matched, block, elem_bytes)
    remote = min(1.0, max(0.0, remote))
    per_req = load["allocated"] * remote  # pages moved into the prefill instance's arena
    written = kv_bytes(cfg, context + extra, block, elem_bytes)["allocated"] - load["allocated"]
    return {
        "model": cfg.name, "context": context, "extra": extra, "matched_tokens": matched, "unique_tokens": unique,
        "req_s": req_s, "load_bytes_per_req": per_req, "new_kv_bytes_per_req": written,
        "load_gbs": None if req_s is None else req_s * per_req / 1e9,
        "new_kv_gbs": None if req_s is None else req_s * written / 1e9,
    }


def capacity(cfg: ModelConfig, context: int, hit: float, users: int, gpus: int, tps_gpu: float, block: int = 16,
             extra: int = 0, copies: int = 1, usable: float = 1.0, elem_bytes: int = 2) -> dict:
    """Pool capacity for `users` retained sessions plus the KV generated while the prefill
    GPUs run flat out. A session's requests extend one prefix lineage: each user holds the
    shared (matched) part once; every request adds its unique part."""
    matched = matched_tokens(context, hit, block)
    unique = context - matched + extra
    req_s = gpus * tps_gpu / unique if unique > 0 else None
    anchor = kv_bytes(cfg, matched, block, elem_bytes)["allocated"]
    new_per_req = kv_bytes(cfg, context + extra, block, elem_bytes)["allocated"] - anchor
    users = max(1, int(users))
    usable = min(1.0, max(0.0, usable))

    def raw(x):
        return None if x is None or usable == 0 else x * max(1, copies) / usable

    windows = []
    for s in WINDOWS_S:
        new = None if req_s is None else req_s * s * new_per_req
        logical = users * anchor + (new or 0)
        windows.append({"seconds": s, "requests": None if req_s is None else req_s * s,
                        "new_kv_bytes": new, "logical_bytes": logical, "raw_bytes": raw(logical)})
    return {"model": cfg.name, "req_s": req_s, "anchor_bytes_per_user": anchor, "anchor_bytes": users * anchor,
            "raw_anchor_bytes": raw(users * anchor), "new_kv_bytes_per_req": new_per_req,
            "new_kv_gbs": None if req_s is None else req_s * new_per_req / 1e9, "windows": windows}


def compare(cfg: ModelConfig, hit_a: float, hit_b: float, context: int, users: int, gpus: int, tps_gpu: float,
            block: int = 16, copies: int = 1, usable: float = 1.0) -> dict:
    """Two hit rates at the same compute budget: how much faster, how much more load and capacity."""
    out = {}
    for tag, h in (("a", hit_a), ("b", hit_b)):
        p = prefill(cfg, context, h, block, gpus=gpus, tps_gpu=tps_gpu)
        c = capacity(cfg, context, h, users, gpus, tps_gpu, block, copies=copies, usable=usable)
        out[tag] = {"hit": h, "req_s": p["req_s"], "load_gbs": p["load_gbs"],
                    "raw_bytes_1h": c["windows"][-1]["raw_bytes"]}

    def rel(x, y):
        return None if not x or y is None else y / x - 1.0

    out["increase"] = {k: rel(out["a"][k], out["b"][k]) for k in ("req_s", "load_gbs", "raw_bytes_1h")}
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("scenario", choices=["prefill", "capacity", "compare"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--extra", type=int, default=0, help="fresh tokens appended after the context")
    ap.add_argument("--hit", type=float, default=0.9)
    ap.add_argument("--hit-b", type=float, default=0.95)
    ap.add_argument("--remote", type=float, default=1.0)
    ap.add_argument("--block", type=int, default=16)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--tps-gpu", type=float, default=70000.0, help="unique prefill tokens/s per GPU")
    ap.add_argument("--req-s", type=float, default=None)
    ap.add_argument("--users", type=int, default=64)
    ap.add_argument("--copies", type=int, default=1)
    ap.add_argument("--usable", type=float, default=1.0)
    a = ap.parse_args(argv)
    cfg = get_config(a.model)
    if a.scenario == "prefill":
        r = prefill(cfg, a.context, a.hit, a.block, a.extra, a.remote, a.gpus,
                    None if a.req_s else a.tps_gpu, a.req_s)
    elif a.scenario == "capacity":
        r = capacity(cfg, a.context, a.hit, a.users, a.gpus, a.tps_gpu, a.block, a.extra, a.copies, a.usable)
    else:
        r = compare(cfg, a.hit, a.hit_b, a.context, a.users, a.gpus, a.tps_gpu, a.block, a.copies, a.usable)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
