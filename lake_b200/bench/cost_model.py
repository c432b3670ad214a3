"""Transfer-versus-recompute cost model for the three execution modes.

Moving H cached tokens of KV costs  t_move(H) = c_move + H * kv_bytes / bw
and recomputing them costs          t_comp(H) = c_comp + H / prefill_rate.
Moving wins once H exceeds the break-even H* = (c_move - c_comp) / (1/prefill_rate - kv_bytes/bw);
when kv_bytes/bw >= 1/prefill_rate moving never wins. The same comparison per
storage tier (its bandwidth and fixed cost) decides whether a pool hit is loaded
or the tail is recomputed. Mode choice: a local HBM hit of at least one block
runs D_DIRECT, a pool hit worth moving runs PD_DISAGG, everything else COLOCATED.

Defaults are this box's measurements for the Llama-3-8B architecture: 131,072 KV
bytes per token (32 layers x K,V x 8 kv heads x 128 x bf16), prefill ~70k tokens/s
per B200 (bench.py PD prefill ranks), NVLink peer copy 770 GB/s, pinned host
DRAM ~50 GB/s (PCIe Gen5), NVMe ~5 GB/s, object store ~1 GB/s.

    python -m lake_b200.bench.cost_model

Reference parity: bench/cost_model.py (same linear transfer/recompute form,
parameters from mock measurements and SLO drafts there).
"""
from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass, field

GB = 1e9
LLAMA3_8B_KV_BYTES = 32 * 2 * 8 * 128 * 2


@dataclass
class CostParams:
    kv_bytes_per_token: int = LLAMA3_8B_KV_BYTES
    block_tokens: int = 16
    link_gbs: float = 770.0  # NVLink 5 peer copy, measured
    move_fixed_s: float = 20e-6  # one fused-epilogue store stream / one batched copy launch
    prefill_tok_s: float = 70_000.0
    prefill_fixed_s: float = 1e-3
    tiers: dict = field(default_factory=lambda: {  # tier: (GB/s, fixed cost s)
        "L1": (50.0, 50e-6), "L2": (5.0, 1e-3), "L3": (1.0, 20e-3)})


def t_move(hit: float, p: CostParams, gbs: float | None = None, fixed: float | None = None) -> float:
    return (p.move_fixed_s if fixed is None else fixed) + hit * p.kv_bytes_per_token / ((gbs or p.link_gbs) * GB)


def t_recompute(tokens: float, p: CostParams) -> float:
    return p.prefill_fixed_s + tokens / p.prefill_tok_s


def breakeven(p: CostParams, gbs: float | None = None, fixed: float | None = None) -> float | None:
    per_tok_move = p.kv_bytes_per_token / ((gbs or p.link_gbs) * GB)
    gain = 1.0 / p.prefill_tok_s - per_tok_move
    if gain <= 0:
        return None
    return ((p.move_fixed_s if fixed is None else fixed) - p.prefill_fixed_s) / gain


def load_or_recompute(tier: str, hit: float, p: CostParams) -> str:
    gbs, fixed = p.tiers[tier]
    h = breakeven(p, gbs, fixed)
    return "load" if h is not None and hit >= max(h, 0.0) else "recompute"


def mode(hit: float, p: CostParams, local_hit: bool, gbs: float | None = None) -> str:
    blocks = int(hit // p.block_tokens)
    if local_hit and blocks > 0:
        return "D_DIRECT"
    h = breakeven(p, gbs)
    return "PD_DISAGG" if h is not None and blocks > 0 and hit >= max(h, p.block_tokens) else "COLOCATED"


def crossover_gbs(p: CostParams) -> float:
    """Link bandwidth below which moving KV never beats recomputing it."""
    return p.kv_bytes_per_token * p.prefill_tok_s / GB


def report(p: CostParams) -> dict:
    sweep = []
    for gbs in (0.5, 1, 5, 10, 50, 100, 770):
        h = breakeven(p, gbs)
        sweep.append({"gbs": gbs, "breakeven_tokens": None if h is None else round(max(h, 0.0), 1),
                      "move_2048_ms": round(t_move(2048, p, gbs) * 1e3, 3)})
    tiers = {t: {"breakeven_tokens": (lambda h: None if h is None else round(max(h, 0.0), 1))(breakeven(p, *v)),
                 "load_2048_ms": round(t_move(2048, p, *v) * 1e3, 3)} for t, v in p.tiers.items()}
    return {"params": asdict(p), "crossover_gbs": round(crossover_gbs(p), 3),
            "recompute_2048_ms": round(t_recompute(2048, p) * 1e3, 3), "link_sweep": sweep, "tiers": tiers}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--prefill-tok-s", type=float, default=70_000.0)
    ap.add_argument("--kv-bytes", type=int, default=LLAMA3_8B_KV_BYTES)
    a = ap.parse_args(argv)
    print(json.dumps(report(CostParams(kv_bytes_per_token=a.kv_bytes, prefill_tok_s=a.prefill_tok_s)), indent=1))


if __name__ == "__main__":
    main()
