"""Arrival-rate sweep of the serving benchmark: bench.py once per Poisson rate (plus the
saturated closed loop), one JSON line per point with output tok/s and p50 TTFT / TPOT.

    python -m lake_b200.bench.sweep --gpus 8 --rates 10,20,40 -- --steps 60 --warmup 5

Arguments after `--` go to bench.py unchanged. For more than one GPU each point is launched
with torch.distributed.run on 127.0.0.1 (one rank per GPU), as the serving bench expects.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def command(gpus: int, rate: float, extra: list[str], port: int = 29600) -> list[str]:
    bench = [os.path.join(ROOT, "bench.py"), "--gpus", str(gpus), "--arrival-rate", f"{rate:g}"] + list(extra)
    if gpus == 1:
        return [sys.executable] + bench
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr", "127.0.0.1", "--master-port", str(port)] + bench


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    extra = []
    if "--" in argv:
        i = argv.index("--")
        argv, extra = argv[:i], argv[i + 1:]
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--rates", default="", help="comma-separated requests/s per request source")
    ap.add_argument("--no-saturated", action="store_true", help="skip the closed-loop point")
    a = ap.parse_args(argv)
    rates = [float(x) for x in a.rates.split(",") if x]
    if not a.no_saturated:
        rates.append(0.0)
    for k, rate in enumerate(rates):
        r = subprocess.run(command(a.gpus, rate, extra, 29600 + k), cwd=ROOT, capture_output=True, text=True)
        line = next((ln for ln in r.stdout.splitlines() if ln.startswith("{")), None)
        if r.returncode or line is None:
            print(json.dumps({"rate": rate, "error": (r.stderr or r.stdout)[-400:]}))
            continue
        d = json.loads(line)
        print(json.dumps({"rate": rate or "saturated", "value": d["value"], "e2e": d["e2e"]["value"],
                          "ttft_p50_ms": d.get("ttft_p50_ms"), "tpot_p50_ms": d.get("tpot_p50_ms"),
                          "n_gpus": d["n_gpus"], "parallelism": d["config"]["parallelism"]}))


if __name__ == "__main__":
    main()
