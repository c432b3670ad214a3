"""Serving benchmark: output tokens/s of the Llama-3-8B engine (bf16, random
init, synthetic uniform-random token ids) under a saturated 2048-in / 256-out
request stream.

    python bench.py --gpus N --steps K --warmup W
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1, one rank per GPU)
    python bench.py --impl reference                        (reference arm)
    python bench.py --impl torch ...                        (library arm: same engine and
                                                             workload, cuBLAS / SDPA / NCCL ops)

One step = one engine iteration: every running request decodes one token and
newly arrived requests are prefilled (chunked, decode-first). Before timing,
`--running` requests are brought into flight with staggered progress (request j
has already produced j*256/running tokens, its prompt covers them), and the
closed-loop source submits a fresh 2048/256 request whenever one finishes, so
the timed steps run the steady state of the serving loop.

`value` = output tokens / device time of the window, the MAX over every rank of
its summed per-step device time (CUDA events around each step's kernels): the
colocated ranks, or under PD-split both the decode ranks (K steps) and the
prefill ranks (their device time inside the decode ranks' window: a prefill step
that straddles an edge of the window counts in proportion to the share of its
host interval inside it); `e2e.value` = the same tokens / the max over ranks of
the wall time of the window's public-API `LLMEngine.step()` calls, which include
scheduling, the pinned host->device copy of each step's metadata and the
device->host read of the sampled tokens.

PD-split (the default from 2 GPUs): single-GPU prefill and decode instances in
pairs (2 GPUs: 1 + 1; 4: 2 + 2; 8: 4 + 4). A prefill instance's QKV epilogue
writes K/V straight into its decode instance's paged arena over NVLink; a decode
instance whose prefill partner is saturated prefills further requests itself in
mixed steps held near a 20 ms step period (--local-prefill, --decode-itl-ms). `--tp T` runs
tensor-parallel instances of T GPUs instead (one prefill and one decode instance
of T GPUs each at N = 2T, the TP groups running the fused NVLink collectives; TP
rank i stores into TP rank i); measured on 8 B200s, TP4 + TP4 moves fewer tokens
per GPU than single-GPU instances (a TP4 prefill instance prefills at about half
the per-GPU rate of a single-GPU one).
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
    ap.add_argument("--config", default=None, help="run configuration file (configs/*.yaml) supplying defaults")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="lakeb", choices=["lakeb", "torch", "reference"],
                    help="lakeb: this framework; torch: the same engine and workload with library ops "
                         "(cuBLAS, torch SDPA, NCCL all_reduce, peer page copies); reference: the "
                         "reference's own code")
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--input-len", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--running", type=int, default=256)
    ap.add_argument("--budget", type=int, default=8192)
    ap.add_argument("--itl-ms", type=float, default=0.0,
                    help="inter-token latency target of single-rank engines: the prefill share of mixed "
                         "steps is capped to keep the step period under it (0 = off; under a closed loop "
                         "at fixed concurrency the cap moves requests from the batch to the queue, so "
                         "TTFT grows by what TPOT gains)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="synchronous steps (default: schedule and launch step n+1 before finishing step n)")
    ap.add_argument("--mode", choices=["colocated", "pd"], default=None,
                    help="default: pd for an even number of GPUs >= 2, else colocated")
    ap.add_argument("--tp", type=int, default=0,
                    help="tensor-parallel instance size (pd: prefill and decode instances of this many GPUs; "
                         "0 = 1, single-GPU instances)")
    ap.add_argument("--ep", action="store_true",
                    help="expert parallel (MoE models): over the decode ranks in pd mode, over all ranks colocated")
    ap.add_argument("--weights", choices=["bf16", "fp8"], default="bf16",
                    help="projection weight format (fp8 = block-scaled e4m3, W8A16 GEMMs)")
    ap.add_argument("--prefill-running", type=int, default=16, help="max concurrent prefills per prefill rank")
    ap.add_argument("--prefill-ranks", type=int, default=0, help="pd mode: prefill instance count (0 = ~60%%)")
    ap.add_argument("--spec-tokens", type=int, default=0,
                    help="speculative decoding: prompt-lookup draft tokens per decode request (0 = off)")
    ap.add_argument("--arrival-rate", type=float, default=0.0,
                    help="open loop: Poisson arrivals at this many requests/s per request source "
                         "(colocated engine or decode instance); 0 = closed loop (saturated)")
    ap.add_argument("--prefill-queue", type=int, default=8,
                    help="pd mode: grants outstanding at a prefill rank (bounds queueing delay)")
    ap.add_argument("--pd-mesh", action="store_true",
                    help="pd mode, single-GPU instances: every prefill instance serves every decode instance "
                         "(a prefill step holds one destination's prompts), ~60%% of the GPUs prefilling")
    ap.add_argument("--local-prefill", type=int, default=1,
                    help="pd mode: a single-GPU decode instance whose prefill partners are saturated "
                         "prefills new requests itself (1, default) or only queues them (0)")
    ap.add_argument("--decode-itl-ms", type=float, default=20.0,
                    help="pd mode: step-period target of single-GPU decode instances that prefill "
                         "locally (caps the prefill share of their mixed steps)")
    pre, _ = ap.parse_known_args()
    if pre.config:
        from lake_b200.utils.config_files import apply_env, bench_defaults, load_run_config

        cfg = load_run_config(pre.config)
        apply_env(cfg)
        known = {a.dest for a in ap._actions}
        ap.set_defaults(**{k: v for k, v in bench_defaults(cfg).items() if k in known})
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
class Window:
    """Per-rank accounting of the timed steps."""

    def __init__(self):
        self.tokens = 0
        self.dev_ms = 0.0
        self.wall_s = 0.0
        self.h2d = 0
        self.d2h = 0
        self.launches = 0
        self.ttft: list[float] = []
        self.tpot: list[float] = []
        self.kv_bytes = 0
        self.decode_rows = 0
        self.prefill_rows = 0
        self.role = "colocated"
        self.gap_ms = 0.0  # device idle between consecutive timed steps
        self.t0 = 0.0      # host clock (time.perf_counter, system-wide monotonic) at the window start
        self.local_prefills = 0  # PD decode leader: requests it prefilled itself in the window
        self.steps_log: list[tuple] = []  # prefill ranks: (start, end, device ms, first tokens) per step

    def clip_to(self, w0: float, w1: float) -> None:
        """Prefill rank under PD-split: keep the part of its work inside the decode ranks' timed
        window [w0, w1] (host clock). A step that straddles an edge counts its device time in
        proportion to the share of its host interval inside the window; a step's first tokens
        count when the step ended inside the window."""
        busy, toks, end = 0.0, 0, w0
        for ts, te, dev, ft in self.steps_log:
            if te > ts:
                busy += dev * max(0.0, min(te, w1) - max(ts, w0)) / (te - ts)
            if w0 <= te <= w1:
                toks += ft
            end = max(end, min(te, w1))
        self.dev_ms, self.tokens = busy, toks
        self.wall_s = max(0.0, end - max(w0, self.t0))

    def count(self, eng):
        out = eng.last_step
        if out is not None:
            self.decode_rows += len(out.decode)
            self.prefill_rows += sum(c.n for c in out.prefill)

    def diag(self, steps):
        if self.steps_log:  # prefill rank: per prefill step of its own
            steps = len(self.steps_log)
        return {"role": self.role, "tokens": self.tokens, "dev_ms": round(self.dev_ms, 2),
                "wall_ms": round(self.wall_s * 1000, 2), "avg_decode_batch": round(self.decode_rows / max(1, steps), 1),
                "avg_prefill_tokens": round(self.prefill_rows / max(1, steps), 1),
                "local_prefills": self.local_prefills,
                "idle_between_steps_ms": round(self.gap_ms, 2)}


class Arrivals:
    """Open-loop request source: Poisson arrivals at `rate` requests/s (exponential gaps from a
    seeded generator). `due()` is how many requests have arrived since the last call; with
    rate 0 the source is closed-loop and always has a request ready."""

    def __init__(self, rate: float, seed: int, clock=time.perf_counter):
        import numpy as np

        self.rate, self.clock = rate, clock
        self.rng = np.random.default_rng(seed)
        self.next = clock() + (self.rng.exponential(1.0 / rate) if rate > 0 else 0.0)
        self.backlog = 0

    def due(self) -> int:
        if self.rate <= 0:
            return 1 << 30
        now = self.clock()
        while self.next <= now:
            self.backlog += 1
            self.next += self.rng.exponential(1.0 / self.rate)
        return self.backlog

    def take(self) -> None:
        if self.rate > 0:
            self.backlog -= 1


def _latency_stats(eng, t0, t1, w: Window):
    """TTFT of every request whose first token came inside the window (arrival may precede it);
    TPOT from each request's token times inside the window."""
    for r in eng.requests.values():
        if r.first_token_time is not None and t0 <= r.first_token_time <= t1:
            w.ttft.append(r.ttft())
        tt = [x for x in r.token_times if t0 <= x <= t1]
        if len(tt) >= 2:
            w.tpot.append((tt[-1] - tt[0]) / (len(tt) - 1))


def _make_engine(args, local, max_running, **kw):
    from lake_b200.engine.llm_engine import LLMEngine

    kw.setdefault("overlap", not args.no_overlap)
    kw.setdefault("spec_tokens", args.spec_tokens)
    kw.setdefault("itl_target_ms", args.itl_ms)
    return LLMEngine(args.model, device=f"cuda:{local}", max_running=max_running, max_batched_tokens=args.budget,
                     max_model_len=args.input_len + args.output_len + 16, use_cuda_graphs=not args.no_graphs,
                     seed=args.seed, weight_dtype=args.weights,
                     model_impl="library" if args.impl == "torch" else "native", **kw)


def run_colocated(args, rank, local, barrier, tp=None, ep=None):
    """One engine per GPU (or per tensor-parallel group) doing prefill and decode
    (chunked, decode-first). Ranks of a TP group submit identical requests and count
    tokens once (on the group's first rank)."""
    import numpy as np
    import torch

    from lake_b200.ops import core as opscore

    stream_id = rank if tp is None else rank // tp[1]
    nprng = np.random.default_rng(args.seed * 1000 + stream_id)
    eng = _make_engine(args, local, args.running, tp=tp, ep=ep)
    counts = tp is None or tp[0] == 0

    def everyone(flag: bool) -> bool:
        # expert parallel: ranks step in lockstep, so loop conditions are agreed on
        if ep is None:
            return flag
        import torch.distributed as dist

        t = torch.tensor([1 if flag else 0])
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ep[2])
        return bool(t.item())
    vocab = eng.cfg.vocab

    def new_prompt(n):
        return nprng.integers(0, vocab, n).tolist()

    initial = []
    for j in range(args.running):  # in flight with staggered progress
        done = (j * args.output_len) // args.running
        initial.append(eng.add_request(new_prompt(args.input_len + done), max_new_tokens=args.output_len - done))

    src = Arrivals(args.arrival_rate, args.seed * 1000 + stream_id + 7)

    def top_up():
        live = len(eng.scheduler.running) + len(eng.scheduler.waiting)
        while live < args.running and src.due() > 0:
            src.take()
            eng.add_request(new_prompt(args.input_len), max_new_tokens=args.output_len)
            live += 1

    eng.runner.capture_graphs()
    guard = 0
    while everyone(any(eng.requests[r].first_token_time is None for r in initial)):
        eng.step()
        top_up()
        guard += 1
        if guard > 100000:
            raise RuntimeError("populate did not converge")
    for _ in range(args.warmup):
        eng.step()
        top_up()
    torch.cuda.synchronize()
    barrier()
    w = Window()
    eng.runner.time_device = True
    eng.runner._prev_ev1, gap0 = None, eng.runner.gap_ms
    opscore.LAUNCHES[0] = 0
    h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    prof = os.environ.get("LAKEB_PROFILE_STEP")  # one timed step inside an NVTX range for `ncu --nvtx-include`
    for i in range(args.steps):
        if prof and i == 1:
            torch.cuda.nvtx.range_push("profile_step")
        outs = eng.step()
        if prof and i == 1:
            torch.cuda.nvtx.range_pop()
        w.tokens += len(outs) if counts else 0
        w.dev_ms += eng.runner.last_device_ms
        w.count(eng)
        top_up()
    torch.cuda.synchronize()
    w.wall_s = time.perf_counter() - t0
    w.launches = opscore.LAUNCHES[0]
    w.h2d = (eng.runner.h2d_bytes - h2d0) / args.steps
    w.d2h = (eng.runner.d2h_bytes - d2h0) / args.steps
    w.gap_ms = eng.runner.gap_ms - gap0
    eng.runner.time_device = False
    if counts:
        _latency_stats(eng, t0, t0 + w.wall_s, w)
    barrier()
    return w


def pd_split(world: int, prefill_ranks: int = 0) -> tuple[int, int]:
    """(prefill, decode) instance counts: pairs (1+1, 2+2, 4+4). Prefill of a 2048-token prompt
    costs more GPU time than its 256 decode steps at full batch, so a decode instance fed by one
    prefill instance has room left, which it fills with its own prefills of the overflow
    (--local-prefill); measured on 8 B200s, 5 prefill + 3 decode instances without that left
    two decode instances at batch 256 and their partners waiting, the third at batch 80."""
    if 0 < prefill_ranks < world:
        return prefill_ranks, world - prefill_ranks
    n_d = max(1, world // 2)
    return world - n_d, n_d


def pd_layout(world: int, tp: int, prefill_instances: int = 0, n_experts: int = 0,
              mesh: bool = False) -> tuple[int, int]:
    """(prefill, decode) instance counts for instances of `tp` GPUs each. With expert-parallel
    decode (`n_experts` > 0) the decode ranks form one EP group, so their count divides the
    expert count: the divisor nearest the ~40% share (8 GPUs: 4 + 4). With `mesh` (every
    prefill instance serves every decode instance) ~60 % of the GPUs prefill (2: 1 + 1,
    4: 2 + 2, 8: 5 + 3), the share at which one prefill GPU's prompts keep ~0.6 decode GPUs busy
    at a full batch."""
    if n_experts and not prefill_instances:
        share = world * 0.4
        n_d = min((d for d in range(1, world) if n_experts % d == 0), key=lambda d: (abs(d - share), -d))
        return world - n_d, n_d
    if mesh and not prefill_instances:
        n = world // tp
        n_d = max(1, round(n * 0.4))
        return n - n_d, n_d
    return pd_split(world // tp, prefill_instances)


def run_pd(args, rank, world, local, group, barrier, tp_groups=None, ep_group=None):
    """Prefill instances [0, P) feed decode instances [P, P + D) (prefill instance i -> decode
    instance P + i % D). An instance is `args.tp` consecutive ranks (a tensor-parallel group
    led by its first rank) or one rank. A decode instance owns its requests and reserves
    pages; its prefill partners' QKV epilogue writes K/V straight into those pages over
    NVLink. A step is one decode-instance iteration; prefill instances work continuously
    through the same window. With `--ep` (MoE) the decode ranks form one expert-parallel
    group: each is its own instance (attention data-parallel) and they step in lockstep for
    the fused expert exchange; prefill instances hold every expert."""
    import numpy as np
    import torch

    from lake_b200.ops import core as opscore
    from lake_b200.parallel import pd

    T = args.tp
    mesh = bool(args.pd_mesh) and T == 1 and not args.ep
    n_p, n_d = pd_layout(world, T, args.prefill_ranks, _n_experts(args) if args.ep else 0, mesh)
    inst = rank // T
    members = list(range(inst * T, inst * T + T))
    leader = members[0] == rank
    role = "prefill" if inst < n_p else "decode"
    if mesh:  # every prefill instance serves every decode instance
        partner = list(range(n_p, n_p + n_d)) if role == "prefill" else list(range(n_p))
    elif role == "prefill":
        d_inst = n_p + inst % n_d
        partner = list(range(d_inst * T, d_inst * T + T))  # the decode instance's ranks
    else:
        partner = [i * T for i in range(n_p) if i % n_d == inst - n_p]  # leaders of the prefill instances
    running = args.running if role == "decode" else args.prefill_running
    tp = (rank % T, T, tp_groups[inst]) if T > 1 else None
    ep = (rank - n_p, n_d, ep_group) if (ep_group is not None and role == "decode") else None
    # decode instances overlap host scheduling with the device; prefill instances report each
    # first token as soon as its step completes (overlap would hold it back one long step)
    # a single-GPU decode instance takes its saturated partners' overflow prefill in mixed steps
    # whose period the inter-token latency governor holds near --decode-itl-ms
    args.local_prefill = int(args.local_prefill and T == 1 and ep is None and role == "decode")
    eng = _make_engine(args, local, running, shared_arena=(role == "decode"), tp=tp, ep=ep,
                       overlap=role == "decode" and not args.no_overlap,
                       itl_target_ms=args.decode_itl_ms if args.local_prefill else 0.0)

    def agree(flag: bool) -> bool:
        # expert-parallel decode ranks step in lockstep: loop conditions are agreed on
        if ep is None:
            return flag
        import torch.distributed as dist

        t = torch.tensor([1 if flag else 0])
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ep_group)
        return bool(t.item())
    job = os.environ.get("TORCHELASTIC_RUN_ID", "bench").replace("-", "")[:16] + str(os.getpid() if world == 1 else 0)
    if mesh and role == "prefill":
        side = pd.connect_pair(eng, role, rank, None, group, job=job, members=members, decode_instances=partner)
    else:
        side = pd.connect_pair(eng, role, rank, partner if T > 1 or role == "decode" else partner[0], group,
                               job=job, members=members)
    w = Window()
    if role == "prefill":
        pd.serve_prefill(side, until_mark=1)          # populate + warm-up
        barrier()
        eng.runner.time_device = True
        eng.runner._prev_ev1, gap0 = None, eng.runner.gap_ms
        opscore.LAUNCHES[0] = 0
        h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        last_ft = [side.first_tokens]

        def on_step():
            # (host start, host end, device ms, first tokens) of each prefill step: the window's
            # device time and tokens are clipped to the decode ranks' window afterwards
            ft = side.first_tokens
            w.steps_log.append((side.step_t0, time.perf_counter(), eng.runner.last_device_ms,
                                ft - last_ft[0] if leader else 0))
            last_ft[0] = ft
            w.count(eng)

        pd.serve_prefill(side, until_mark=2, on_step=on_step)
        torch.cuda.synchronize()
        w.role = "prefill"
        w.t0 = t0
        w.wall_s = time.perf_counter() - t0
        w.dev_ms = sum(x[2] for x in w.steps_log)
        w.tokens = sum(x[3] for x in w.steps_log)
        w.launches = opscore.LAUNCHES[0]
        w.h2d = (eng.runner.h2d_bytes - h2d0) / max(1, args.steps)
        w.d2h = (eng.runner.d2h_bytes - d2h0) / max(1, args.steps)
        w.gap_ms = eng.runner.gap_ms - gap0
        eng.runner.time_device = False
        barrier()
        pd.serve_prefill(side)                        # until EXIT
        side.close()
        return w, role
    eng.runner.capture_graphs()
    if not leader:
        # tensor-parallel decode follower: replay the leader's decisions and steps
        side.follow()                                 # populate + warm-up (phase 1)
        torch.cuda.synchronize()
        barrier()
        eng.runner.time_device = True
        eng.runner._prev_ev1, gap0 = None, eng.runner.gap_ms
        opscore.LAUNCHES[0] = 0
        h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        w.role = "decode"

        def on_step(outs):
            w.dev_ms += eng.runner.last_device_ms
            w.count(eng)

        side.follow(on_step)                          # the timed window (phase 2)
        torch.cuda.synchronize()
        w.t0 = t0
        w.wall_s = time.perf_counter() - t0
        w.launches = opscore.LAUNCHES[0]
        w.h2d = (eng.runner.h2d_bytes - h2d0) / args.steps
        w.d2h = (eng.runner.d2h_bytes - d2h0) / args.steps
        w.gap_ms = eng.runner.gap_ms - gap0
        eng.runner.time_device = False
        barrier()
        side.follow()                                 # until EXIT
        side.close()
        return w, role
    nprng = np.random.default_rng(args.seed * 1000 + rank)
    vocab = eng.cfg.vocab

    def new_prompt(n):
        return nprng.integers(0, vocab, n).tolist()

    src = Arrivals(args.arrival_rate, args.seed * 1000 + rank + 7)

    side.queue_depth = args.prefill_queue

    def top_up():
        # keep the prefill partner's queue short (bounded TTFT) and the decode batch <= running
        while (len(side.pending) < args.prefill_queue * len(side.links) and side.inflight < args.running
               and src.due() > 0):
            if not side.submit(new_prompt(args.input_len), args.output_len):
                return
            src.take()
        # overflow: every prefill partner is saturated and the batch still has room -> prefill here
        # (colocated on this instance, chunked into its mixed steps under the step-period cap),
        # one request at a time
        while (args.local_prefill and side.saturated and side.inflight < args.running and src.due() > 0
               and not eng.scheduler.waiting and not any(r.is_prefill for r in eng.scheduler.running)):
            if not side.submit(new_prompt(args.input_len), args.output_len, local=True):
                return
            src.take()

    # populate: run the closed loop until a full request lifetime of completions has passed,
    # so the decode batch holds requests at every stage of their output
    target = max(32, args.running // 4)
    t_pop = t_note = time.perf_counter()
    pop_steps = 0
    while agree(len(eng.scheduler.finished) < target):
        side.poll()
        if eng.has_unfinished() or ep is not None:
            side.step()  # (an idle expert-parallel rank still joins the group's exchange)
            pop_steps += 1
        else:
            time.sleep(0.0005)
        top_up()
        now = time.perf_counter()
        if now - t_note > 30:  # a slow populate says where it stands (a stall shows which side waits)
            t_note = now
            print(f"rank {rank} populate {now - t_pop:.0f}s: {pop_steps} steps, finished "
                  f"{len(eng.scheduler.finished)}/{target}, running {len(eng.scheduler.running)}, "
                  f"waiting {len(eng.scheduler.waiting)}, prefill queue {len(side.pending)}, "
                  f"in flight {side.inflight}", file=sys.stderr, flush=True)
        if now - t_pop > 240:
            raise RuntimeError(f"rank {rank}: populate did not reach steady state in 240 s "
                               f"({len(eng.scheduler.finished)}/{target} requests finished)")
    for _ in range(args.warmup):
        side.poll()
        side.step()
        top_up()
    side.mark(1)
    side.phase(1)
    torch.cuda.synchronize()
    barrier()
    eng.runner.time_device = True
    eng.runner._prev_ev1, gap0 = None, eng.runner.gap_ms
    opscore.LAUNCHES[0] = 0
    h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
    kv0, local0 = side.kv_bytes, side.local
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    w.role = "decode"
    for _ in range(args.steps):
        side.poll()
        outs = side.step()
        w.tokens += len(outs)
        w.dev_ms += eng.runner.last_device_ms
        w.count(eng)
        top_up()
    torch.cuda.synchronize()
    w.t0 = t0
    w.wall_s = time.perf_counter() - t0
    w.launches = opscore.LAUNCHES[0]
    w.h2d = (eng.runner.h2d_bytes - h2d0) / args.steps
    w.d2h = (eng.runner.d2h_bytes - d2h0) / args.steps
    w.kv_bytes = side.kv_bytes - kv0
    w.local_prefills = side.local - local0
    w.gap_ms = eng.runner.gap_ms - gap0
    eng.runner.time_device = False
    _latency_stats(eng, t0, t0 + w.wall_s, w)
    side.mark(2)
    side.phase(2)
    barrier()
    side.shutdown()
    side.close()
    return w, role


def _n_experts(args) -> int:
    from lake_b200.models.config import get_config

    return get_config(args.model).n_experts or 0


def _model_desc(name):
    from lake_b200.models.config import get_config

    c = get_config(name)
    desc = {"llama3-8b": "Llama-3-8B", "llama3-70b": "Llama-3-70B", "mixtral-8x7b": "Mixtral-8x7B"}.get(name, name)
    moe = f", {c.n_experts} experts top-{c.top_k}" if c.n_experts else ""
    return (f"{desc} architecture ({c.n_layers} layers, hidden {c.hidden}, {c.n_q_heads}q/{c.n_kv_heads}kv heads, "
            f"FFN {c.intermediate}{moe}, vocab {c.vocab})")


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=900))
        group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))

    def barrier():
        if world > 1:
            dist.barrier(group=group)

    if args.tp == 0:  # auto: single-GPU instances (the highest tokens per GPU measured)
        args.tp = 1
    if world % args.tp:
        raise SystemExit("--tp must divide the GPU count")
    mode = args.mode or ("pd" if world // args.tp >= 2 else "colocated")
    ep = (rank, world, group) if args.ep and world > 1 and mode == "colocated" else None
    ep_group = None
    if args.ep and mode == "pd":
        n_p, n_d = pd_layout(world, args.tp, args.prefill_ranks, _n_experts(args))
        if n_d > 1:  # every rank creates the group (collective), decode ranks use it
            ep_group = dist.new_group(list(range(n_p, world)), backend="gloo")
    tp = None
    tp_groups = None
    if args.tp > 1:
        gid = rank // args.tp
        # the library model's all_reduce runs on NCCL; the native model's group only exchanges handles
        tp_groups = [dist.new_group(list(range(g * args.tp, (g + 1) * args.tp)),
                                    backend="nccl" if args.impl == "torch" else "gloo")
                     for g in range(world // args.tp)]
        tp = (rank % args.tp, args.tp, tp_groups[gid])
    clocks = ClockSampler(visible_gpu_indices(world) if rank == 0 else [])
    if rank == 0:
        clocks.start()
    role = "colocated"
    if mode == "pd":
        w, role = run_pd(args, rank, world, local, group, barrier, tp_groups, ep_group)
    else:
        w = run_colocated(args, rank, local, barrier, tp, ep)
    ck = clocks.stop() if rank == 0 else {}

    # aggregate over ranks (max of times, sum of counts) through the gloo group. The window's
    # device time is the busiest rank's: decode (or colocated) ranks' K steps, or a prefill rank's
    # device time inside the decode ranks' window (PD-split), whichever is larger.
    if mode == "pd" and world > 1:
        spans = [None] * world
        dist.all_gather_object(spans, (role, w.t0, w.t0 + w.wall_s), group=group)
        dec = [(a, b) for r, a, b in spans if r == "decode"]
        if role == "prefill" and dec:
            w.clip_to(min(a for a, _ in dec), max(b for _, b in dec))
    t = torch.tensor([w.dev_ms, w.wall_s * 1000.0, float(w.tokens),
                      w.h2d, w.d2h, float(w.launches), float(w.kv_bytes), w.dev_ms], dtype=torch.float64)
    lat = (w.ttft, w.tpot, w.diag(args.steps))
    if world > 1:
        mx, sm = t.clone(), t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM, group=group)
        lats = [None] * world
        dist.all_gather_object(lats, lat, group=group)
        ttft = [x for l in lats for x in l[0]]
        tpot = [x for l in lats for x in l[1]]
        ranks = [l[2] for l in lats]
    else:
        mx, sm = t, t
        ttft, tpot = lat[0], lat[1]
        ranks = [lat[2]]
    # device time of the window: the busiest rank (decode steps, or a prefill rank's busy time)
    dev_ms = mx[0].item()
    producer_ms = {}
    if world > 1:
        for l in lats:
            producer_ms[l[2]["role"]] = max(producer_ms.get(l[2]["role"], 0.0), l[2]["dev_ms"])
    wall_ms = mx[1].item()
    tokens = sm[2].item()
    value = tokens / (dev_ms / 1000.0)
    e2e = tokens / (wall_ms / 1000.0)
    if rank == 0:
        p50 = (lambda xs: sorted(xs)[len(xs) // 2] if xs else None)
        kv_gbs = sm[6].item() / (wall_ms / 1000.0) / 1e9 if sm[6].item() else None
        mesh = bool(args.pd_mesh) and args.tp == 1 and not args.ep
        n_p, n_d = pd_layout(world, args.tp, args.prefill_ranks, _n_experts(args) if args.ep else 0, mesh)
        par = (f"pd: {n_p} prefill + {n_d} decode instances (tp{args.tp} each)" +
               (", every prefill instance serving every decode instance" if mesh else "") +
               (f", decode ranks expert-parallel ep{n_d} (fused dispatch/combine)" if ep_group is not None else "")
               ) if mode == "pd" else (
            f"dp{world // args.tp} x tp{args.tp} (fused NVLink collectives)" if args.tp > 1 else
            f"ep{world} (experts split, attention data-parallel, fused dispatch/combine)" if ep else
            (f"dp{world}" if world > 1 else "single"))
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "output tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.weights == "bf16" else "bf16 activations/KV, fp8 block-scaled weights",
            "data": "synthetic (uniform random token ids, random-init weights)",
            "config": {"model": _model_desc(args.model),
                       "global_batch": args.running * (n_d if mode == "pd" else world // args.tp),
                       "seq_len": args.input_len + args.output_len, "input_len": args.input_len,
                       "output_len": args.output_len, "parallelism": par, "mode": mode,
                       "layout_note": ("single-GPU prefill/decode pairs, decode instances prefilling their saturated "
                                       "partners' overflow; the named TP4 prefill + TP4 decode layout runs with --tp 4 "
                                       "and measured fewer tokens per GPU on 8 B200s"
                                       if mode == "pd" and args.tp == 1 and not args.ep and not args.pd_mesh
                                       else None),
                       "l2": "inputs larger than L2 (16 GB weights, >60 GB KV read per step)",
                       "arrivals": (f"poisson {args.arrival_rate:g} req/s per request source" if args.arrival_rate
                                    else "closed loop: a new request whenever one finishes (saturated)"),
                       "itl_target_ms": (args.itl_ms or None) if mode != "pd" and args.tp == 1 and not args.ep else None,
                       "step": ("one decode-instance iteration (prefill instances run continuously)" if mode == "pd"
                                else "one engine iteration: decode all running + chunked prefill of arrivals")},
            "e2e": {"value": round(e2e, 1), "unit": "output tok/s", "h2d_bytes_per_step": int(sm[3].item()),
                    "d2h_bytes_per_step": int(sm[4].item()), "api": "LLMEngine.step()"},
            "gpu_launches": int(sm[5].item()),
            "ttft_p50_ms": round(p50(ttft) * 1000, 2) if ttft else None,
            "tpot_p50_ms": round(p50(tpot) * 1000, 2) if tpot else None,
            "p2d_kv_gbs": round(kv_gbs, 2) if kv_gbs else None,
            "clocks": ck, "impl": args.impl, "busiest_ms_by_role": producer_ms or None, "ranks": ranks,
        }
        print(json.dumps(line))
        from lake_b200.utils.trace import emit

        emit(line)
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
