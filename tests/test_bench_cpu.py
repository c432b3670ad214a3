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
    assert b.pd_split(2) == (1, 1) and b.pd_split(4) == (2, 2) and b.pd_split(8) == (5, 3)
    assert b.pd_layout(8, 4) == (1, 1) and b.pd_layout(4, 2) == (1, 1)
    assert b.pd_layout(8, 1, n_experts=8) == (4, 4)  # expert-parallel decode ranks divide the experts


def test_sweep_commands():
    from lake_b200.bench import sweep

    one = sweep.command(1, 12.5, ["--steps", "10"])
    assert one[1].endswith("bench.py") and "--arrival-rate" in one and "12.5" in one and one[-1] == "10"
    many = sweep.command(8, 0.0, [], port=29611)
    assert "torch.distributed.run" in many and "--nproc-per-node=8" in many and "127.0.0.1" in many
    assert "29611" in many and many[many.index("--arrival-rate") + 1] == "0"
