"""Transfer-vs-recompute cost model (reference behaviour: bench/test_cost_model.py)."""
from lake_b200.bench.cost_model import CostParams, breakeven, crossover_gbs, load_or_recompute, mode, report


def test_breakeven_and_crossover():
    p = CostParams()
    # moving 128 KB/token over NVLink beats recomputing at 70k tok/s for any non-trivial hit
    h = breakeven(p)
    assert h is not None and h < 0  # fixed recompute cost exceeds the fixed move cost
    assert abs(crossover_gbs(p) - 131072 * 70000 / 1e9) < 1e-9
    assert breakeven(p, gbs=5.0) is None  # below ~9.2 GB/s recomputing always wins
    slow = CostParams(prefill_tok_s=5000.0, kv_bytes_per_token=114688, move_fixed_s=2e-3)
    assert 10 < breakeven(slow, gbs=1.0) < 13  # the reference's 1 GB/s anchor (~11.7 tokens)


def test_modes_and_tiers():
    p = CostParams()
    assert mode(64, p, local_hit=True) == "D_DIRECT"
    assert mode(8, p, local_hit=True) == "COLOCATED"  # below one block
    assert mode(2048, p, local_hit=False) == "PD_DISAGG"
    assert mode(2048, p, local_hit=False, gbs=1.0) == "COLOCATED"
    assert load_or_recompute("L1", 2048, p) == "load"
    assert load_or_recompute("L3", 2048, p) == "recompute"
    r = report(p)
    assert r["link_sweep"][-1]["gbs"] == 770 and r["tiers"]["L1"]["breakeven_tokens"] is not None
