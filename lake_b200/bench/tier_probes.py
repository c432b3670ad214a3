"""Tier-engine probes on the real L2/L3 media of this host: latency distributions of the
durable write and the promotion into L0, and the hit-rate / cost curves of a synthetic
prefix-sharing workload.

    python -m lake_b200.bench.tier_probes [--only latency,curves] [--requests 3000] [--dir DIR]

Every record is one JSON line on stdout (and appended to LAKE_BENCH_OUT when set):

* ``tier_put_durable`` / ``tier_promote_l0``: p50/p99 milliseconds of put_durable (an
  fdatasync'd L2 record, with the L2 -> L3 demotion it may trigger) and promote_to_l0 (from
  L1, L2 or L3, through an L1 slot), and ``tier_hit_stats`` (probe outcome counts).
* ``hit_curve``: L0 capacity (L1 = 4x, L2 = 16x) -> L0/L1/L2/L3 hits and cold misses of a
  workload where 70 % of requests share one of 256 prefixes (zipf 1.2 popularity) and the
  rest are unique; bytes written and bytes moved between tiers.
* ``promote_calibration``: measured promotion time per source tier against the engine's
  modelled cost (block bytes x hops), and the L3/L1 time ratio.
* ``block_granularity``: reusable share of a fully shared prompt (256..2048 tokens) at block
  sizes 16 (this engine), 64, 128 and 256.
* ``writeback_scan``: decode write-back batching N in {1, 2, 4}: bytes do not change, write
  operations fall as 1/N (the WritebackBatcher's flushes counted).
* ``admission_experiment``: the same workload with promotion admitted as hot only from the
  second hit (one-shot blocks are evicted first) against admitting every promotion.
* ``gc_proxy``: bytes moved between tiers per byte read or written on the data path.

Reference parity: rust/tiered-store/src/bin/p71_probe.rs:1-124 and p73_curves.rs:1-411
(there the tiers are in-memory maps; here L2 is fdatasync'd segment files and L3 an object
directory, so the latencies are this host's).
"""
from __future__ import annotations

import argparse
import bisect
import json
import os
import tempfile
import time

import torch

from .. import _host as H
from ..utils.trace import emit

BLOCK_BYTES = 4096
HOT_PREFIXES = 256
UNIQUE_PREFIXES = 4096
BLOCKS_PER_REQ = 16
SHARE_PCT = 70


class XorShift:
    def __init__(self, seed: int):
        self.s = (seed | 1) & 0xFFFFFFFFFFFFFFFF

    def next(self) -> int:
        x = self.s
        x ^= (x << 13) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 7
        x ^= (x << 17) & 0xFFFFFFFFFFFFFFFF
        self.s = x
        return x

    def below(self, n: int) -> int:
        return self.next() % n


class Zipf:
    def __init__(self, n: int, alpha: float):
        acc, self.cum = 0.0, []
        for i in range(1, n + 1):
            acc += 1.0 / i ** alpha
            self.cum.append(acc)

    def sample(self, rng: XorShift) -> int:
        return bisect.bisect_left(self.cum, rng.next() / 2 ** 64 * self.cum[-1])


def request_blocks(rng: XorShift, zipf: Zipf, share_pct: int) -> list[bytes]:
    prefix = zipf.sample(rng) if rng.below(100) < share_pct else HOT_PREFIXES + rng.below(UNIQUE_PREFIXES)
    return [((prefix << 32) | i).to_bytes(8, "little") for i in range(BLOCKS_PER_REQ)]


class Engine:
    """A TierEngine over a fresh directory, its pinned-host L1 slab and an L0 page counter."""

    def __init__(self, root: str, l0: int, l1: int, l2: int, admit_after: int = 0):
        self.l1 = torch.zeros(l1 * BLOCK_BYTES, dtype=torch.uint8)
        d = tempfile.mkdtemp(dir=root)
        self.e = H.TierEngine(H.TierCaps(l0, l1, l2), BLOCK_BYTES, self.l1.data_ptr(), os.path.join(d, "l2"),
                              os.path.join(d, "l3"), "probe")
        if admit_after:
            self.e.set_promote_admit_after(admit_after)
        self.next_page = 0

    def alloc(self) -> int:
        self.next_page += 1
        return self.next_page


def _pct(xs: list[float], q: float) -> float:
    if not xs:
        return 0.0
    xs = sorted(xs)
    return xs[int(q * (len(xs) - 1))]


def _out(rec: dict) -> None:
    print(json.dumps(rec))
    emit(rec)


# ------------------------------------------------------------------ latency
def latency(root: str, n: int = 512) -> None:
    eng = Engine(root, 64, 256, 1024)
    e = eng.e
    block = bytes(BLOCK_BYTES)
    for i in range(n):
        e.put_durable_bytes(i.to_bytes(4, "little"), block)
    promote = []
    for i in range(n):
        t = time.perf_counter()
        c, _, _ = e.promote_to_l0(i.to_bytes(4, "little"), eng.alloc)
        if c is not None:
            promote.append((time.perf_counter() - t) * 1000)
    put = []
    for i in range(n, 2 * n):
        t = time.perf_counter()
        e.put_durable_bytes(i.to_bytes(4, "little"), block)
        put.append((time.perf_counter() - t) * 1000)
    for i in range(2 * n):
        e.probe(i.to_bytes(4, "little"))
    c = e.stats.counts
    _out({"name": "tier_promote_l0", "latency_ms": {"p50": _pct(promote, .5), "p99": _pct(promote, .99)},
          "counters": {"samples": len(promote)}})
    _out({"name": "tier_put_durable", "latency_ms": {"p50": _pct(put, .5), "p99": _pct(put, .99)},
          "counters": {"samples": len(put)}, "note": "fdatasync'd L2 record"})
    _out({"name": "tier_hit_stats", "counters": {"l0": c[0], "l1": c[1], "l2": c[2], "l3": c[3], "miss": c[4],
                                                  "modelled_cost_us": e.stats.modelled_cost_us()}})


# ------------------------------------------------------------------ curves
def drive(root: str, l0: int, requests: int, share_pct: int, seed: int, admit_after: int = 0) -> dict:
    eng = Engine(root, l0, 4 * l0, 16 * l0, admit_after)
    e = eng.e
    rng, zipf = XorShift(seed), Zipf(HOT_PREFIXES, 1.2)
    block = bytes(BLOCK_BYTES)
    written = moved = promotes = 0
    for _ in range(requests):
        for h in request_blocks(rng, zipf, share_pct):
            kind = e.probe(h)
            if kind == H.AccessKind.L0_HIT:
                continue
            if kind == H.AccessKind.MISS:
                _, fx = e.put_durable_bytes(h, block)
                written += BLOCK_BYTES
                moved += (len(fx.l0_demoted) + len(fx.l2_demoted_to_l3)) * BLOCK_BYTES
                continue
            try:
                c, evict, fx = e.promote_to_l0(h, eng.alloc)
            except ValueError:
                continue
            promotes += 1
            moved += BLOCK_BYTES + (len(evict) + len(fx.l0_demoted) + len(fx.l2_demoted_to_l3)) * BLOCK_BYTES
    c = e.stats.counts
    return {"l0_hit": c[0], "l1_hit": c[1], "l2_hit": c[2], "l3_hit": c[3], "cold_miss": c[4],
            "write_bytes": written, "moved_bytes": moved, "promotes": promotes}


def curves(root: str, requests: int) -> None:
    for l0 in (32, 64, 128, 256, 512):
        r = drive(root, l0, requests, SHARE_PCT, 42, admit_after=1)
        total = sum(r[k] for k in ("l0_hit", "l1_hit", "l2_hit", "l3_hit", "cold_miss"))
        _out({"name": "hit_curve", "counters": {"l0_cap": l0, **r},
              "hit_rate": (r["l0_hit"] + r["l1_hit"] + r["l2_hit"]) / total,
              "hit_rate_with_l3": (total - r["cold_miss"]) / total})

    # promotion time per source tier vs the modelled cost (bytes x hops)
    eng = Engine(root, 8, 64, 512)
    e = eng.e
    block = bytes(BLOCK_BYTES)
    key = lambda tag, i: ((tag << 32) | i).to_bytes(8, "little")  # noqa: E731
    for i in range(8):
        e.put_durable_bytes(key(1, i), block)
        e.put_durable_bytes(key(2, i), block)
    for i in range(16):
        e.put_durable_bytes(key(3, i), block)
        e.put_durable_bytes(key(4, i), block)
    for tag in (1, 2):  # group 1 fills L0, group 2 pushes it down to L1
        for i in range(8):
            e.promote_to_l0(key(tag, i), eng.alloc)
    per_hops: dict[int, list[float]] = {}

    def measure(tag, i):
        h = key(tag, i)
        hops = e.estimate_promote_cost(h) // BLOCK_BYTES
        t = time.perf_counter()
        c, _, _ = e.promote_to_l0(h, eng.alloc)
        if c is not None:
            per_hops.setdefault(hops, []).append((time.perf_counter() - t) * 1e6)

    for i in range(8):
        measure(1, i)  # L1
    for i in range(16):
        measure(3, i)  # L2
    for i in range(600):  # overflow L2: group 4 goes to L3
        e.put_durable_bytes(key(5, i), block)
    for i in range(16):
        measure(4, i)  # L3
    avg = {h: sum(v) / len(v) for h, v in per_hops.items()}
    for h, v in sorted(per_hops.items()):
        _out({"name": "promote_calibration", "counters": {"hops": h, "samples": len(v)}, "avg_us": avg[h]})
    if 1 in avg and 3 in avg:
        _out({"name": "promote_calibration_ratio", "hops3_over_hops1": avg[3] / avg[1]})

    rng = XorShift(7)
    prompts = [256 + rng.below(1793) for _ in range(10000)]
    for blk in (16, 64, 128, 256):
        reused = sum(p // blk * blk for p in prompts)
        _out({"name": "block_granularity", "counters": {"block_tokens": blk}, "reuse_ratio": reused / sum(prompts)})

    decode_blocks = 8
    for n in (1, 2, 4):
        w = H.WritebackBatcher(n)
        ops = 0
        for r in range(requests):
            for b in range(decode_blocks):
                if w.push(((r << 8) | b).to_bytes(8, "little")):
                    ops += 1
            if w.drain():
                ops += 1
        _out({"name": "writeback_scan", "counters": {"batch_n": n, "ops": ops,
                                                     "bytes": decode_blocks * BLOCK_BYTES * requests}})

    for l0 in (64, 128, 512):
        for tag, admit in (("baseline", 1), ("admit>=2", 2)):
            r = drive(root, l0, requests, SHARE_PCT, 42, admit_after=admit)
            reads = (r["l0_hit"] + r["l1_hit"] + r["l2_hit"] + r["l3_hit"]) * BLOCK_BYTES
            _out({"name": "admission_experiment", "counters": {"l0_cap": l0, "admitted": int(admit > 1), **r},
                  "moved_per_read_write": r["moved_bytes"] / max(1, reads + r["write_bytes"])})

    r = drive(root, 256, requests, SHARE_PCT, 99, admit_after=1)
    reads = (r["l0_hit"] + r["l1_hit"] + r["l2_hit"] + r["l3_hit"]) * BLOCK_BYTES
    _out({"name": "gc_proxy", "counters": {"moved_bytes": r["moved_bytes"], "read_bytes": reads,
                                           "write_bytes": r["write_bytes"]},
          "share": r["moved_bytes"] / max(1, reads + r["write_bytes"])})


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="latency,curves")
    ap.add_argument("--requests", type=int, default=3000)
    ap.add_argument("--dir", default=None, help="where the L2/L3 files go (default: a temporary directory)")
    args = ap.parse_args(argv)
    root = args.dir or tempfile.mkdtemp(prefix="lakeb_tier_probe_")
    os.makedirs(root, exist_ok=True)
    if "latency" in args.only:
        latency(root)
    if "curves" in args.only:
        curves(root, args.requests)


if __name__ == "__main__":
    main()
