"""Multi-turn agent workload: S sessions x T turns sharing a system prefix.

Each turn's prompt is the session's whole history (system prefix, earlier
user turns and generated answers) plus U fresh uniform-random user tokens; the
turn generates O tokens. Turn k+1 of a session is submitted when turn k
finishes. HBM for KV is capped (--hbm-blocks pages of 16 tokens), so the
engine's prefix cache alone cannot hold every session; finished requests'
pages (prompt and decode-extended) are written behind into pinned host DRAM
(D -> pool) and promoted back into HBM when the next turn arrives (pool -> P).
Per request the execution mode is chosen by the router rule from the reuse
hint: a local HBM hit runs D_DIRECT, else COLOCATED (one GPU holds both
roles here; on N GPUs sessions stick to a replica by session id).

Reported: output tok/s over the whole workload (device time of the engine
steps, and wall time of the public-API loop), TTFT p50 per turn, prompt
tokens computed vs reused, L0 hits / L1 promotions, D -> pool and pool -> P
GB/s, L1 spills, pages written into L1 by the QKV epilogue vs copied at finish,
and (with --durable-blocks) the L2 durable tier's PutEnd commits and L2
promotions; and the same workload with prefix reuse disabled as the no-reuse
baseline.

    python -m lake_b200.bench.agent                     # 1 GPU
    torchrun --nproc-per-node N -m lake_b200.bench.agent
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch


def run(args, device, rank, reuse: bool):
    from lake_b200.engine.block_pool import chain_block_hashes
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.ops import core as opscore
    from lake_b200.pool.agents.hostcache import HostCacheAgent
    from lake_b200.pool.pool_iface import PoolIface
    from lake_b200.pool.types import PrefixHint
    from lake_b200.runtime.config import WorkerRole, select_exec_mode

    max_len = args.system + args.turns * (args.user + args.output) + 16
    eng = LLMEngine(args.model, device=device, max_running=args.sessions, max_batched_tokens=args.budget,
                    max_model_len=max_len, num_blocks=args.hbm_blocks, enable_prefix_cache=reuse,
                    use_cuda_graphs=True, seed=args.seed)
    agent = tier = None
    if reuse:
        if args.durable_blocks:
            from lake_b200.pool.agents.durable import DurableTier

            page_bytes = eng.arena[0].numel() * eng.arena.element_size()
            tier = DurableTier(args.model, page_bytes, eng.cfg.n_layers, eng.ec.block_size,
                               l2_blocks=args.durable_blocks, storage_dir=args.durable_dir)
        agent = HostCacheAgent(eng, args.l1_blocks, mirror=not args.no_kernel_writeback, durable=tier)
        eng.attach_pool(PoolIface(agent))
    rng = np.random.default_rng(args.seed * 100 + rank)
    vocab = eng.cfg.vocab
    system = rng.integers(0, vocab, args.system).tolist()
    hist = {s: list(system) for s in range(args.sessions)}
    turn = {s: 0 for s in range(args.sessions)}
    rid_sess = {}
    modes = {"D_DIRECT": 0, "COLOCATED": 0, "PD_DISAGG": 0}
    prompt_tokens = 0

    def submit(s):
        nonlocal prompt_tokens
        p = hist[s] + rng.integers(0, vocab, args.user).tolist()
        hashes = chain_block_hashes(p, eng.ec.block_size, full_only=True)
        local = eng.pool.peek(hashes) if reuse else 0
        hint = PrefixHint(computed_tokens=local * eng.ec.block_size, reused_blocks=local, local_hit=local > 0)
        modes[select_exec_mode(hint, len(p), WorkerRole.HYBRID).value] += 1
        rid = eng.add_request(p, max_new_tokens=args.output)
        rid_sess[rid] = s
        prompt_tokens += len(p)
        turn[s] += 1

    eng.runner.capture_graphs()
    torch.cuda.synchronize()
    for s in range(args.sessions):
        submit(s)
    eng.runner.time_device = True
    opscore.LAUNCHES[0] = 0
    dev_ms = 0.0
    out_tokens = 0
    steps = 0
    seen_finished = 0
    t0 = time.perf_counter()
    while eng.has_unfinished():
        outs = eng.step()
        steps += 1
        out_tokens += len(outs)
        dev_ms += eng.runner.last_device_ms
        fin = eng.scheduler.finished
        while seen_finished < len(fin):
            r = fin[seen_finished]
            seen_finished += 1
            s = rid_sess.pop(r.rid, None)
            if s is None:
                continue
            hist[s] = r.prompt + r.output
            if turn[s] < args.turns:
                submit(s)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    opscore.check_status()
    reqs = [r for r in eng.requests.values() if r.first_token_time is not None]
    ttft = sorted(r.ttft() for r in reqs)
    computed = sum(len(r.prompt) - r.num_cached for r in reqs)
    res = {"output_tokens": out_tokens, "dev_ms": dev_ms, "wall_s": wall, "steps": steps,
           "ttft_p50_ms": ttft[len(ttft) // 2] * 1000 if ttft else None,
           "prompt_tokens": prompt_tokens, "prompt_tokens_computed": computed,
           "reuse_frac": 1 - computed / max(1, prompt_tokens), "modes": modes,
           "l0_evictions": eng.pool.stats["evictions"], "launches": opscore.LAUNCHES[0],
           "h2d_bytes": eng.runner.h2d_bytes, "d2h_bytes": eng.runner.d2h_bytes}
    if agent is not None:
        res.update({k: (round(v, 2) if isinstance(v, float) else v) for k, v in agent.stats.items()})
        page = eng.arena[0].numel() * eng.arena.element_size()
        res["d2pool_gbs"] = round(agent.stats["writeback_blocks"] * page / wall / 1e9, 3)  # D -> pool
        res["d2p_gbs"] = round(agent.stats["promoted_blocks"] * page / wall / 1e9, 3)  # pool -> P
        res["l1_spills"] = agent.stats["l1_evictions"]
    if tier is not None:
        tier.flush()
        res.update({f"durable_{k}": (round(v, 2) if isinstance(v, float) else v) for k, v in tier.stats.items()})
        tier.close()
    eng.runner.time_device = False
    del eng
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--turns", type=int, default=8)
    ap.add_argument("--system", type=int, default=4096)
    ap.add_argument("--user", type=int, default=512)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--budget", type=int, default=8192)
    ap.add_argument("--hbm-blocks", type=int, default=12000, help="HBM KV cap in 16-token pages")
    ap.add_argument("--l1-blocks", type=int, default=16000, help="pinned host DRAM pages")
    ap.add_argument("--durable-blocks", type=int, default=0,
                    help="L2 pages of the durable tier behind L1 (PutEnd, fdatasync'd records); 0 = off")
    ap.add_argument("--durable-dir", default=None, help="directory of the durable tier's segment files")
    ap.add_argument("--no-kernel-writeback", action="store_true",
                    help="copy decode pages to L1 at finish instead of writing them from the QKV epilogue")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-baseline", action="store_true")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("gloo")
        args.sessions = max(1, args.sessions // world)  # sessions pinned to a replica by id
    dev = f"cuda:{local}"
    res = {"reuse": run(args, dev, rank, True)}
    if not args.no_baseline:
        res["no_reuse"] = run(args, dev, rank, False)
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, res)
    else:
        allr = [res]
    if rank == 0:
        def agg(key):
            rs = [r[key] for r in allr]
            tok = sum(r["output_tokens"] for r in rs)
            dev_s = max(r["dev_ms"] for r in rs) / 1000
            wall = max(r["wall_s"] for r in rs)
            return {"tok_s": round(tok / dev_s, 1), "e2e_tok_s": round(tok / wall, 1), "output_tokens": tok,
                    "ttft_p50_ms": round(sorted(r["ttft_p50_ms"] for r in rs)[len(rs) // 2], 1),
                    "reuse_frac": round(sum(r["reuse_frac"] for r in rs) / len(rs), 4), "per_rank": rs}
        line = {"bench": "agent_multiturn", "model": args.model, "n_gpus": world,
                "workload": {"sessions": args.sessions * world, "turns": args.turns, "system": args.system,
                             "user": args.user, "output": args.output, "hbm_blocks": args.hbm_blocks,
                             "l1_blocks": args.l1_blocks},
                "reuse": agg("reuse")}
        if "no_reuse" in res:
            line["no_reuse"] = agg("no_reuse")
            line["speedup_vs_no_reuse"] = round(line["reuse"]["tok_s"] / line["no_reuse"]["tok_s"], 3)
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
