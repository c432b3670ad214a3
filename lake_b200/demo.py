"""Single-process prefix-reuse demo: two requests that share a 48-token system prompt go through
the router core (view mirror, prefix hint, mode select), two engines and one KV pool node
(tier engine, PutEnd, authority). Request A runs cold on worker-0 and writes its pages back to
the pool; request B, routed to worker-1, finds the shared prefix in the pool, promotes those
pages into its own KV arena and prefills only the rest.

    python -m lake_b200.demo [--device cuda:0]

Reference parity: src/__main__.py (the early prototype's two-request demo: B reuses A's prefix
from the KV pool instead of recomputing it).
"""
from __future__ import annotations

import argparse
import json
import tempfile


def run(device: str = "cpu", block_size: int = 16) -> dict:
    from . import _host as H
    from .engine.block_pool import chain_block_hashes
    from .engine.llm_engine import LLMEngine
    from .pool.agents.native import NativeAgent, make_pool_node
    from .pool.pool_iface import PoolIface

    model = "tiny" if device == "cpu" else "tiny-gpu"  # the GPU kernels want head_dim 128 (bf16)
    kw = dict(device=device, max_running=4, max_batched_tokens=256, max_model_len=512, num_blocks=64,
              block_size=block_size)
    authority = H.Authority()
    mirror = H.ViewMirror()
    engines = {n: LLMEngine(model, **kw) for n in ("worker-0", "worker-1")}
    page = engines["worker-0"].arena[0].numel() * engines["worker-0"].arena.element_size()
    out = {}
    with tempfile.TemporaryDirectory(prefix="lakeb_demo_") as root:
        pool_node = make_pool_node(model, page, engines["worker-0"].pool.num_blocks, l1_blocks=16, l2_blocks=64,
                                   storage_dir=root)
        for n, eng in engines.items():
            eng.attach_pool(PoolIface(NativeAgent(eng, n, authority=authority, shared_tiers=pool_node,
                                                  storage_node_id="pool-0"), node_id=n))
        system = list(range(1, 49))  # three full blocks shared by both requests
        for name, node, prompt in (("A", "worker-0", system + [100, 101]), ("B", "worker-1", system + [200, 201])):
            mirror.apply(authority.snapshot())
            hashes = chain_block_hashes(prompt, block_size, full_only=True)
            found = mirror.prefix_lookup(model, "", 1, hashes, node)
            local = 0  # leading blocks held in this node's HBM
            for blk in found:
                if not blk.local_hit:
                    break
                local += 1
            hint = H.PrefixHint(min(len(found) * block_size, len(prompt)), len(found), local, local > 0)
            mode = H.select_exec_mode(hint, len(prompt), H.Role.HYBRID, 0.0)
            eng = engines[node]
            rid = eng.add_request(prompt, max_new_tokens=4)
            while eng.has_unfinished():
                eng.step()
            req = eng.requests[rid]
            out[name] = {"node": node, "mode": mode.name, "pool_prefix_blocks": len(found),
                         "reused_blocks": req.num_cached // block_size,
                         "prefill_blocks": -(-(len(prompt) - req.num_cached) // block_size),
                         "output": list(req.output)}
        out["pool_durable_blocks"] = pool_node[0].l2_len()
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--device", default="cpu")
    r = run(ap.parse_args().device)
    for name in ("A", "B"):
        x = r[name]
        print(f"Req {name} on {x['node']} ({x['mode']}): reused={x['reused_blocks']} prefill={x['prefill_blocks']}")
    print(f"KV pool: {r['pool_durable_blocks']} durable blocks")
    print(json.dumps(r))


if __name__ == "__main__":
    main()
