"""Host-side pieces of bench.py that need no GPU."""
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_poisson_arrivals_rate_and_closed_loop():
    b = _bench()
    t = [0.0]
    src = b.Arrivals(50.0, seed=3, clock=lambda: t[0])
    t[0] = 100.0
    n = src.due()
    assert 4500 < n < 5500  # ~50/s over 100 s
    for _ in range(n):
        src.take()
    assert src.due() == 0
    closed = b.Arrivals(0.0, seed=3, clock=lambda: t[0])
    assert closed.due() > 1000 and (closed.take() or closed.due() > 1000)


def test_pd_layouts():
    b = _bench()
    assert b.pd_split(2) == (1, 1) and b.pd_split(4) == (2, 2) and b.pd_split(8) == (4, 4)
    assert b.pd_split(8, prefill_ranks=5) == (5, 3)
    assert b.pd_layout(8, 4) == (1, 1) and b.pd_layout(4, 2) == (1, 1)
    assert b.pd_layout(8, 1, n_experts=8) == (4, 4)  # expert-parallel decode ranks divide the experts
    assert [b.pd_layout(n, 1, mesh=True) for n in (2, 4, 8)] == [(1, 1), (2, 2), (5, 3)]


def test_prefill_window_clipping():
    """A prefill rank's device time and first tokens are cut to the decode ranks' window: steps
    inside count fully, a straddling step by its share of the window, steps after it not at all."""
    b = _bench()
    w = b.Window()
    w.role, w.t0 = "prefill", 10.0
    # (host start, host end, device ms, first tokens)
    w.steps_log = [(10.0, 10.1, 90.0, 4), (10.1, 10.2, 95.0, 4), (10.2, 10.4, 180.0, 4), (10.4, 10.5, 90.0, 4)]
    w.clip_to(10.0, 10.3)
    assert abs(w.dev_ms - (90.0 + 95.0 + 90.0)) < 1e-6  # half of the 180 ms straddling step
    assert w.tokens == 8  # the straddling step ended after the window
    assert abs(w.wall_s - 0.3) < 1e-9


def test_sweep_commands():
    from lake_b200.bench import sweep

    one = sweep.command(1, 12.5, ["--steps", "10"])
    assert one[1].endswith("bench.py") and "--arrival-rate" in one and "12.5" in one and one[-1] == "10"
    many = sweep.command(8, 0.0, [], port=29611)
    assert "torch.distributed.run" in many and "--nproc-per-node=8" in many and "127.0.0.1" in many
    assert "29611" in many and many[many.index("--arrival-rate") + 1] == "0"


def test_tier_probes_curves_and_latency(tmp_path, capsys):
    """The tier-engine probes on this host's files: latency records, capacity curve that does
    not fall as L0 grows, write-back ops falling as 1/N at constant bytes, block granularity."""
    import json

    from lake_b200.bench import tier_probes

    tier_probes.main(["--requests", "120", "--dir", str(tmp_path)])
    recs = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    by = {}
    for r in recs:
        by.setdefault(r["name"], []).append(r)
    for name in ("tier_put_durable", "tier_promote_l0", "tier_hit_stats", "hit_curve", "promote_calibration",
                 "block_granularity", "writeback_scan", "admission_experiment", "gc_proxy"):
        assert name in by, name
    rates = [r["hit_rate"] for r in by["hit_curve"]]
    assert rates == sorted(rates)
    wb = {r["counters"]["batch_n"]: r["counters"] for r in by["writeback_scan"]}
    assert wb[1]["bytes"] == wb[4]["bytes"] and wb[1]["ops"] == 4 * wb[4]["ops"]
    reuse = [r["reuse_ratio"] for r in by["block_granularity"]]
    assert reuse == sorted(reuse, reverse=True) and reuse[0] > 0.99


def test_router_probe_reports_latency_queue_and_modes():
    from lake_b200.bench import router_probe

    recs = {r["name"]: r for r in router_probe.run(requests=24, max_inflight=2, delay_ms=1.0)}
    assert recs["router_e2e_latency"]["latency_ms"]["p99"] >= recs["router_e2e_latency"]["latency_ms"]["p50"] > 0
    assert recs["router_queue_wait"]["counters"]["samples"] == 24
    assert sum(v for k, v in recs["router_mode_distribution"]["counters"].items() if k.startswith("mode_")) == 24
