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


def test_kv_planner_arithmetic():
    from lake_b200.bench import kv_planner as kp
    from lake_b200.models.config import get_config

    cfg = get_config("llama3-8b")
    per = 32 * 2 * 8 * 128 * 2  # 131072 bytes per token
    assert kp.kv_bytes_per_token(cfg) == per
    assert kp.matched_tokens(8192, 0.9, 16) == 7360  # whole blocks of the 7372.8-token hit
    assert kp.matched_tokens(100, 1.0, 16) == 96
    p = kp.prefill(cfg, 8192, 0.9, 16, gpus=2, tps_gpu=1000.0, remote=0.5)
    assert p["unique_tokens"] == 832
    assert abs(p["req_s"] - 2000.0 / 832) < 1e-9
    assert p["load_bytes_per_req"] == 7360 * per * 0.5
    c = kp.capacity(cfg, 4096, 0.5, users=10, gpus=1, tps_gpu=2048.0, copies=2, usable=0.5)
    assert c["anchor_bytes_per_user"] == 2048 * per and c["req_s"] == 1.0
    w = c["windows"][0]
    assert w["seconds"] == 300 and w["logical_bytes"] == 10 * 2048 * per + 300 * 2048 * per
    assert w["raw_bytes"] == w["logical_bytes"] * 4
    cmp = kp.compare(cfg, 0.5, 0.75, 4096, 10, 1, 2048.0)
    assert abs(cmp["increase"]["req_s"] - 1.0) < 1e-9  # half the unique tokens: twice the requests
