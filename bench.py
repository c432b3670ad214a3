"""Serving benchmark: output tokens/s of the Llama-3-8B engine (bf16, random
init, synthetic uniform-random token ids) under a saturated 2048-in / 256-out
request stream.

    python bench.py --gpus N --steps K --warmup W
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1, one rank per GPU)
    python bench.py --impl reference                        (reference arm)

One step = one engine iteration: every running request decodes one token and
newly arrived requests are prefilled (chunked, decode-first). Before timing,
`--running` requests are brought into flight with staggered progress (request j
has already produced j*256/running tokens, its prompt covers them), and the
closed-loop source submits a fresh 2048/256 request whenever one finishes, so
the timed steps run the steady state of the serving loop.

`value` = output tokens / summed device time of the K steps (CUDA events around
each step's kernels, max over ranks); `e2e.value` = the same tokens / wall time
of the K public-API `LLMEngine.step()` calls, which include scheduling, the
pinned host->device copy of each step's metadata and the device->host read of
the sampled tokens.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "output tok/s per box (Llama-3-8B PD-split); p50 TTFT/TPOT; P→D KV GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="lakeb", choices=["lakeb", "reference"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--input-len", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--running", type=int, default=256)
    ap.add_argument("--budget", type=int, default=8192)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, indices):
        self.indices = indices
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.indices:
            cmd += ["-i", ",".join(str(i) for i in self.indices)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        threading.Thread(target=self._read, daemon=True).start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        time.sleep(0.1)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def visible_gpu_indices(n, local_rank=None):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            ids = [int(x) for x in vis.split(",")]
        except ValueError:
            return None
        return ids[:n] if local_rank is None else [ids[local_rank]]
    return list(range(n)) if local_rank is None else [local_rank]


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    why = ("reference has no GPU compute path (its Qwen3 modules are identity shells on the meta device, "
           "logits are a dummy, no Llama architecture is registered) and its generated gRPC stubs fail to import "
           "with the installed protobuf 6.33 (gencode 7.35)")
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": why, "metric": METRIC, "n_gpus": args.gpus}))
    return 0


# ---------------------------------------------------------------- our arm
def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.ops import core as opscore

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))

    import numpy as np

    nprng = np.random.default_rng(args.seed * 1000 + rank)
    eng = LLMEngine(args.model, device=f"cuda:{local}", max_running=args.running, max_batched_tokens=args.budget,
                    max_model_len=args.input_len + args.output_len + 16, use_cuda_graphs=not args.no_graphs,
                    seed=args.seed)
    vocab = eng.cfg.vocab

    def new_prompt(n):
        return nprng.integers(0, vocab, n).tolist()

    # bring `running` requests into flight with staggered progress
    initial = []
    for j in range(args.running):
        done = (j * args.output_len) // args.running
        initial.append(eng.add_request(new_prompt(args.input_len + done), max_new_tokens=args.output_len - done))

    def top_up():
        live = len(eng.scheduler.running) + len(eng.scheduler.waiting)
        while live < args.running:
            eng.add_request(new_prompt(args.input_len), max_new_tokens=args.output_len)
            live += 1

    eng.runner.capture_graphs()
    # populate: step until every initial request has produced its first token (arrivals replace finishers)
    guard = 0
    while any(eng.requests[r].first_token_time is None for r in initial):
        eng.step()
        top_up()
        guard += 1
        if guard > 100000:
            raise RuntimeError("populate did not converge")

    for _ in range(args.warmup):
        eng.step()
        top_up()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    clocks = ClockSampler(visible_gpu_indices(world) if rank == 0 else [])
    if rank == 0:
        clocks.start()
    eng.runner.time_device = True
    opscore.LAUNCHES[0] = 0
    h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
    tokens = 0
    dev_ms = 0.0
    ttft, tpot = [], []
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        outs = eng.step()
        tokens += len(outs)
        dev_ms += eng.runner.last_device_ms
        top_up()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    launches = opscore.LAUNCHES[0]
    eng.runner.time_device = False
    ck = clocks.stop() if rank == 0 else {}
    t1 = t0 + wall
    for r in eng.requests.values():
        if r.first_token_time is not None and t0 <= r.arrival and r.first_token_time <= t1:
            ttft.append(r.ttft())
        tt = [x for x in r.token_times if t0 <= x <= t1]
        if len(tt) >= 2:
            tpot.append((tt[-1] - tt[0]) / (len(tt) - 1))
    h2d = (eng.runner.h2d_bytes - h2d0) / args.steps
    d2h = (eng.runner.d2h_bytes - d2h0) / args.steps

    stats = torch.tensor([dev_ms, wall * 1000.0, float(tokens), h2d, d2h, float(launches)], dtype=torch.float64,
                         device=dev)
    if world > 1:
        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        dev_ms_max, wall_ms_max = mx[0].item(), mx[1].item()
        tok_total, h2d_t, d2h_t, launches_t = sm[2].item(), sm[3].item(), sm[4].item(), sm[5].item()
    else:
        dev_ms_max, wall_ms_max, tok_total, h2d_t, d2h_t, launches_t = (stats[0].item(), stats[1].item(),
                                                                         stats[2].item(), stats[3].item(),
                                                                         stats[4].item(), stats[5].item())
    value = tok_total / (dev_ms_max / 1000.0)
    e2e = tok_total / (wall_ms_max / 1000.0)
    if rank == 0:
        p50 = (lambda xs: sorted(xs)[len(xs) // 2] if xs else None)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "output tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms_max / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform random token ids, random-init weights)",
            "config": {"model": "Llama-3-8B architecture (32 layers, hidden 4096, 32q/8kv heads, FFN 14336, "
                                "vocab 128256)", "global_batch": args.running * world,
                       "seq_len": args.input_len + args.output_len, "input_len": args.input_len,
                       "output_len": args.output_len, "parallelism": f"dp{world}" if world > 1 else "single",
                       "mode": "colocated engine per GPU (prefill+decode on the same GPU)",
                       "l2": "inputs larger than L2 (16 GB weights, >60 GB KV read per step)",
                       "step": "one engine iteration: decode all running + chunked prefill of arrivals"},
            "e2e": {"value": round(e2e, 1), "unit": "output tok/s", "h2d_bytes_per_step": int(h2d_t),
                    "d2h_bytes_per_step": int(d2h_t), "api": "LLMEngine.step()"},
            "gpu_launches": int(launches_t),
            "ttft_p50_ms": round(p50(ttft) * 1000, 2) if ttft else None,
            "tpot_p50_ms": round(p50(tpot) * 1000, 2) if tpot else None,
            "clocks": ck, "impl": "lakeb",
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
