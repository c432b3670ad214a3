"""CPU plumbing run (fp32, seed 0): a prefill worker and a separate decode worker joined by
the KV pool.

Model: random-init 2-layer decoder (hidden 256, 4 q / 2 kv heads, head_dim 64, SwiGLU FFN 1024,
RMSNorm, RoPE theta 10000, vocab 1024), 16-token KV blocks. Workload: 8 requests that share a
128-token prefix plus 32 unique tokens (uniform in [0, 1024)), 16 greedy decode steps each.

Flow: the prefill engine runs every prompt and writes its full pages back to the pool (PutEnd:
L2 segment files, registered in the radix/location authority). The decode engine admits the
same prompts; at admission its storage agent finds the pages through the authority and
promotes them from the pool into its own arena, so only the prompt's last block is computed
there before decoding. Checks: every request's pool prefix hit, and each decode step's logits
equal a colocated single-process run's to 1e-5 (max abs difference reported).

    python -m lake_b200.bench.cpu_plumbing
"""
from __future__ import annotations

import json
import tempfile

import numpy as np


def _step_logits(eng, prompts, output):
    """Run `prompts` through `eng` and return {(request index, position): logits row} for every
    sampled token, captured from the lm_head of each step (CPU path)."""
    from lake_b200 import ops

    rows: list = []
    real = ops.linear_argmax

    def rec(a, w, *args, **k):
        rows.append((a.float() @ w.float().t()).clone())
        return real(a, w, *args, **k)

    ops.linear_argmax = rec
    out = {}
    try:
        rids = [eng.add_request(p, max_new_tokens=output) for p in prompts]
        index = {r: i for i, r in enumerate(rids)}
        while eng.has_unfinished():
            rows.clear()
            eng.step()
            step = eng.last_step
            if step is None or not rows:
                continue
            logits = rows[-1]
            k = 0
            for ch in step.chunks:
                if ch.sample:
                    out[(index[ch.req.rid], ch.start + ch.n)] = logits[k]
                    k += 1
        tokens = [eng.requests[r].output for r in rids]
    finally:
        ops.linear_argmax = real
    return out, tokens


def run(seed: int = 0, requests: int = 8, prefix: int = 128, unique: int = 32, output: int = 16) -> dict:
    from lake_b200 import _host as H
    from lake_b200.engine.block_pool import chain_block_hashes
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.pool.agents.native import NativeAgent, make_pool_node
    from lake_b200.pool.pool_iface import PoolIface

    rng = np.random.default_rng(seed)
    shared = rng.integers(0, 1024, prefix).tolist()
    prompts = [shared + rng.integers(0, 1024, unique).tolist() for _ in range(requests)]
    kw = dict(device="cpu", max_running=8, max_batched_tokens=256, max_model_len=512, num_blocks=256, seed=seed)

    def engine():
        return LLMEngine("tiny", **kw)

    authority = H.Authority()
    p_eng, d_eng = engine(), engine()
    page = p_eng.arena[0].numel() * p_eng.arena.element_size()
    with tempfile.TemporaryDirectory(prefix="lakeb_pool_") as root:
        node = make_pool_node("tiny", page, p_eng.pool.num_blocks, l1_blocks=64, l2_blocks=512, storage_dir=root)
        p_agent = NativeAgent(p_eng, "prefill-0", authority=authority, shared_tiers=node, storage_node_id="pool-0")
        d_agent = NativeAgent(d_eng, "decode-0", authority=authority, shared_tiers=node, storage_node_id="pool-0")
        p_eng.attach_pool(PoolIface(p_agent, node_id="prefill-0"))
        d_eng.attach_pool(PoolIface(d_agent, node_id="decode-0"))

        # 1. prefill worker: every prompt (one sampled token), pages written back to the pool
        p_eng.generate(prompts, max_new_tokens=1)
        written = p_agent.stats["writeback_blocks"]
        # 2. decode worker: the same prompts; admission promotes their pages from the pool
        pool_hits = [authority.lookup_prefix("tiny", "", 1, chain_block_hashes(p, 16, full_only=True),
                                             "decode-0").hit_length for p in prompts]
        got_logits, got = _step_logits(d_eng, prompts, output)
        want_logits, want = _step_logits(engine(), prompts, output)
        promoted = d_agent.stats["promoted_blocks"]
    common = sorted(set(got_logits) & set(want_logits))
    diff = max((got_logits[k] - want_logits[k]).abs().max().item() for k in common) if common else None
    return {"bench": "cpu_plumbing", "requests": requests, "pool_written_blocks": written,
            "pool_prefix_hit_blocks": pool_hits, "promoted_blocks": promoted,
            "tokens_equal": got == want, "compared_positions": len(common), "max_abs_logit_diff": diff,
            "logits_match_1e-5": diff is not None and diff <= 1e-5}


def main():
    print(json.dumps(run()))


if __name__ == "__main__":
    main()
