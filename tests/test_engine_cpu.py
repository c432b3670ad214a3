"""CPU tests of the engine: block pool, scheduler policy, hash chain, and the
2-layer fp32 plumbing model against the dense oracle."""
import random

import numpy as np

import pytest
import torch

from lake_b200.engine.block_pool import BlockPool, NoFreeBlocks, chain_block_hashes
from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.engine.request import Request, SamplingParams
from lake_b200.engine.scheduler import Scheduler, SchedulerConfig
from lake_b200.oracle import ops_ref as ref
from lake_b200.oracle.model_ref import dense_logits, greedy_generate


# Cross-language vectors of the reference chain hash (go/router/prefixhash_test.go:13-49).
def test_chain_hash_vectors():
    got = [h.hex() for h in chain_block_hashes(list(range(16)), 8)]
    assert got == ["ff1f6ee5d67458cfac950f62e93042e21fcb867e2234dcc8721801231064ad40",
                   "db6e3872f1224a65b9d8238ba1f888935fa525fc0883a6d259369139d271ead9"]
    assert chain_block_hashes([7], 8)[0].hex() == "e8613f5a5bc9f9feeda32a8e7c80b69dd4878e47b6a91723fb15eb84236b6a2b"
    assert chain_block_hashes([], 8) == []
    assert len(chain_block_hashes(list(range(17)), 8, full_only=True)) == 2


def test_block_pool_prefix_cache_and_eviction():
    pool = BlockPool(4, 16)
    a = pool.alloc(3)
    hs = [bytes([i]) * 32 for i in range(3)]
    for b, h in zip(a, hs):
        pool.register(b, h)
    pool.release(a)
    assert pool.num_free == 4
    hit = pool.lookup(hs[:2] + [b"x" * 32])
    assert hit == a[:2]
    pool.release(hit)
    # allocating all four evicts the LRU cached blocks
    got = pool.alloc(4)
    assert sorted(got) == list(range(4))
    assert pool.lookup(hs) == []
    with pytest.raises(NoFreeBlocks):
        pool.alloc(1)


def _req(rid, n, out=4):
    return Request(rid=rid, prompt=list(range(n)), params=SamplingParams(max_new_tokens=out))


def test_scheduler_budget_decode_first_and_chunking():
    pool = BlockPool(64, 16)
    s = Scheduler(pool, SchedulerConfig(max_running=4, max_batched_tokens=40, max_model_len=256))
    s.add(_req("a", 50))
    s.add(_req("b", 10))
    o = s.schedule()
    assert [(c.req.rid, c.start, c.n, c.sample) for c in o.prefill] == [("a", 0, 40, False)]
    s.update(o, [], 0.0)
    o = s.schedule()
    # a continues (10 tokens, samples), then b is admitted with the remaining 30 budget
    assert [(c.req.rid, c.start, c.n, c.sample) for c in o.prefill] == [("a", 40, 10, True), ("b", 0, 10, True)]
    s.update(o, [1, 2], 0.0)
    o = s.schedule()
    assert [c.req.rid for c in o.decode] == ["a", "b"] and not o.prefill


def test_scheduler_preempts_when_out_of_pages():
    pool = BlockPool(5, 16)
    s = Scheduler(pool, SchedulerConfig(max_running=4, max_batched_tokens=200, max_model_len=256))
    s.add(_req("a", 32, out=40))
    s.add(_req("b", 32, out=40))
    o = s.schedule()
    s.update(o, [0, 0], 0.0)
    preempted = []
    for _ in range(40):
        o = s.schedule()
        preempted += o.preempted
        s.update(o, [0] * sum(c.sample for c in o.chunks), 0.0)
        if not s.has_work():
            break
    assert preempted, "expected a preemption when pages run out"


def test_itl_governor_caps_prefill_of_mixed_steps():
    """A simulated device whose step time is 10 ms + 0.02 ms per prefill token, under a closed
    loop (a finished request is replaced at once): with a 30 ms target the prefill share of
    mixed steps settles near 1000 tokens and steady-state periods stay under the target."""
    pool = BlockPool(8192, 16)
    s = Scheduler(pool, SchedulerConfig(max_running=64, max_batched_tokens=4096, max_model_len=4096,
                                        itl_target_ms=30.0, itl_min_prefill=128))
    def _fresh(k):  # a distinct prompt (no prefix-cache hits), staggered output lengths
        return Request(rid=f"r{k}", prompt=[(k * 4099 + t) % 100000 for t in range(2000)],
                       params=SamplingParams(max_new_tokens=20 + (7 * k) % 41))

    n = 0
    for _ in range(64):
        s.add(_fresh(n))
        n += 1
    now, periods, caps, pre = 0.0, [], [], []
    for _ in range(400):
        o = s.schedule()
        n_pre = sum(c.n for c in o.prefill)
        dt = 0.010 + 0.00002 * n_pre
        now += dt
        if o.decode:
            periods.append(dt)
            caps.append(s.itl.cap)
            pre.append(n_pre)
        for _ in s.update(o, [0] * sum(c.sample for c in o.chunks), now):
            s.add(_fresh(n))
            n += 1
    assert max(periods[-200:]) <= 0.0315, max(periods[-200:])
    assert 700 <= min(caps[-200:]) and max(caps[-200:]) <= 1100, (min(caps[-200:]), max(caps[-200:]))
    assert sum(pre[-200:]) / 200 > 600  # prefill keeps flowing at the cap


def test_itl_governor_restarts_after_idle_gap():
    from lake_b200.engine.scheduler import ItlGovernor

    g = ItlGovernor(20.0, 4096, 256)
    g.observe(0.0, 4096)
    g.observe(0.040, 4096)  # over the target: halves at most
    assert g.cap == 2048
    g.observe(10.0, 2048)  # an idle gap: no period measured
    assert g.cap == 2048
    g.observe(10.010, 2048)  # under 90 % with the cap filled: grows
    assert g.cap == int(2048 * 1.1) + 1
    g.observe(10.020, 10)  # under the target but the cap was not binding: unchanged
    assert g.cap == int(2048 * 1.1) + 1
    for k in range(50):
        g.observe(10.1 + k, 0)
    g2 = ItlGovernor(20.0, 4096, 256)
    t = 0.0
    for _ in range(20):
        t += 0.060
        g2.observe(t, 4096)
    assert g2.cap == 256


def test_rope_cache_llama3_scaling_keeps_high_freq():
    plain = ref.rope_cache(16, 500000.0)
    scaled = ref.rope_cache(16, 500000.0, scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                   "high_freq_factor": 4.0,
                                                   "original_max_position_embeddings": 8192})
    assert torch.allclose(plain[:, :8], scaled[:, :8])
    assert not torch.allclose(plain[:, -4:], scaled[:, -4:])


def test_swiglu_interleave_roundtrip():
    g = torch.randn(256, 8)
    u = torch.randn(256, 8)
    x = torch.randn(3, 8)
    w = ref.interleave_gate_up(g, u)
    out = ref.swiglu_from_interleaved(x @ w.t())
    want = torch.nn.functional.silu(x @ g.t()) * (x @ u.t())
    assert torch.allclose(out, want, atol=1e-5)


def test_plumbing_model_matches_dense_oracle():
    """2-layer fp32 model: chunked, paged, prefix-cached generation == dense recomputation."""
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=100, max_model_len=512, num_blocks=64)
    rng = random.Random(0)
    prefix = [rng.randrange(1024) for _ in range(128)]
    prompts = [prefix + [rng.randrange(1024) for _ in range(32)] for _ in range(3)]
    outs = eng.generate(prompts, max_new_tokens=6)
    assert eng.pool.stats["hits"] >= 8
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(eng.model, p, 6)


def test_library_model_matches_dense_oracle():
    """The library comparator (torch ops, standard weight layouts) run by the same engine, with
    the native model's weights: chunked, paged, prefix-cached, overlapped greedy generation ==
    dense recomputation of the native model."""
    from lake_b200.models.llama import DecoderLM

    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=100, max_model_len=512, num_blocks=64,
                    model_impl="library", overlap=True)
    native = DecoderLM(eng.cfg, "cpu", seed=0)
    eng.model._from_native(native.w)
    rng = random.Random(1)
    prefix = [rng.randrange(1024) for _ in range(128)]
    prompts = [prefix + [rng.randrange(1024) for _ in range(32)] for _ in range(3)]
    outs = eng.generate(prompts, max_new_tokens=6)
    assert eng.pool.stats["hits"] >= 8
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(native, p, 6)


def test_plumbing_logits_close():
    eng = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=64, max_model_len=256, num_blocks=32)
    prompt = list(range(40))
    eng.add_request(prompt, max_new_tokens=1)
    from lake_b200.engine.scheduler import Chunk, SchedulerOutput
    req = eng.scheduler.waiting.popleft()
    req.block_ids = eng.pool.alloc(3)
    out = SchedulerOutput(0, prefill=[Chunk(req, 0, 40, True)])
    eng.runner._pack(out)
    eng.runner._copy_cpu(0, 0, 0)
    b = eng.runner._batch_views(40, 1, 1, 1, 0, 1)
    b.want_logits = True
    logits = eng.model.forward(b, eng.arena, eng.runner.ws)
    want = dense_logits(eng.model, prompt)[-1]
    assert torch.allclose(logits[0], want, atol=1e-4, rtol=1e-4)


def test_host_cache_agent_writeback_and_promote():
    """L1 host tier: finished pages are written behind, evicted from HBM by other
    traffic, promoted back on reuse; tokens match an engine without the tier."""
    from lake_b200.pool.agents.hostcache import HostCacheAgent
    from lake_b200.pool.pool_iface import PoolIface

    rng = np.random.default_rng(3)
    sys_prompt = rng.integers(0, 1024, 96).tolist()
    first = sys_prompt + rng.integers(0, 1024, 20).tolist()
    others = [rng.integers(0, 1024, 100).tolist() for _ in range(3)]
    eng = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=128, max_model_len=512, num_blocks=20)
    agent = HostCacheAgent(eng, l1_blocks=64)
    eng.attach_pool(PoolIface(agent))
    out1 = eng.generate([first], max_new_tokens=6)[0]
    assert agent.stats["writeback_blocks"] >= 7
    for p in others:  # push the first request's pages out of the 20-page HBM pool
        eng.generate([p], max_new_tokens=2)
    assert eng.pool.stats["evictions"] > 0
    follow = first + out1 + rng.integers(0, 1024, 10).tolist()
    got = eng.generate([follow], max_new_tokens=4)[0]
    assert agent.stats["promoted_blocks"] >= 6
    ref = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    assert got == ref.generate([follow], max_new_tokens=4)[0]


def test_kernel_write_behind_of_decode_pages():
    """Decode-extended pages reach the host tier through the QKV epilogue's second KV target
    (reserved L1 slots written as the tokens are produced), not a copy at finish: a later turn
    promoted from those slots produces the same tokens as an engine that recomputes everything."""
    from lake_b200.pool.agents.hostcache import HostCacheAgent
    from lake_b200.pool.pool_iface import PoolIface

    rng = np.random.default_rng(5)
    first = rng.integers(0, 1024, 40).tolist()
    eng = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=128, max_model_len=512, num_blocks=24)
    agent = HostCacheAgent(eng, l1_blocks=64)
    eng.attach_pool(PoolIface(agent))
    assert eng.runner.mirror_arena is agent.mirror_arena
    out1 = eng.generate([first], max_new_tokens=60)[0]
    # 40 prompt + 60 generated tokens: pages 3, 4 and 5 hold generated tokens only and are full
    assert agent.stats["kernel_written_blocks"] == 3
    assert agent.stats["copied_blocks"] == 3  # prompt pages 0-2 (page 2 also holds generated tokens)
    assert not agent.reserved  # the unfinished page's slot went back
    for p in [rng.integers(0, 1024, 150).tolist() for _ in range(2)]:
        eng.generate([p], max_new_tokens=2)  # push the first request's pages out of HBM
    follow = first + out1 + rng.integers(0, 1024, 7).tolist()
    got = eng.generate([follow], max_new_tokens=5)[0]
    assert agent.stats["promoted_blocks"] >= 5
    ref = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    assert got == ref.generate([follow], max_new_tokens=5)[0]


def test_host_tier_over_durable_l2_with_putend(tmp_path):
    """The host-cache agent on the real pool tiers: finished pages are committed in the
    background with PutEnd to fdatasync'd L2 records and registered with the authority; with an
    L1 too small to keep them, a later turn promotes them from L2 and decodes the same tokens."""
    from lake_b200.engine.block_pool import chain_block_hashes
    from lake_b200.pool.agents.durable import DurableTier
    from lake_b200.pool.agents.hostcache import HostCacheAgent
    from lake_b200.pool.pool_iface import PoolIface

    rng = np.random.default_rng(13)
    first = rng.integers(0, 1024, 72).tolist()
    eng = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=128, max_model_len=512, num_blocks=24)
    page_bytes = eng.arena[0].numel() * eng.arena.element_size()
    tier = DurableTier("tiny", page_bytes, eng.cfg.n_layers, 16, l2_blocks=256, storage_dir=str(tmp_path))
    agent = HostCacheAgent(eng, l1_blocks=10, durable=tier)
    eng.attach_pool(PoolIface(agent))
    out1 = eng.generate([first], max_new_tokens=40)[0]
    tier.flush()
    hashes = chain_block_hashes((first + out1)[:6 * 16], 16, full_only=True)
    r = tier.authority.lookup_prefix("tiny", "", 1, hashes, "node-0")
    assert r.hit_length == 6 and tier.stats["durable_blocks"] == 6  # 111 tokens with KV: 6 full pages
    assert all(any(l.tier == 3 for l in b.meta.locations) for b in r.blocks)  # an L2 copy each
    for p in [rng.integers(0, 1024, 150).tolist() for _ in range(2)]:  # evict HBM and the 10-slot L1
        eng.generate([p], max_new_tokens=2)
    tier.flush()
    assert not agent.pinned
    follow = first + out1 + rng.integers(0, 1024, 5).tolist()
    got = eng.generate([follow], max_new_tokens=4)[0]
    assert agent.stats["l2_promoted_blocks"] > 0 and tier.stats["l2_reads"] > 0
    ref = LLMEngine("tiny", device="cpu", max_running=2, max_batched_tokens=128, max_model_len=512, num_blocks=64)
    assert got == ref.generate([follow], max_new_tokens=4)[0]
    tier.close()


def _overlap_run(overlap, num_blocks, eos=None, max_new=24):
    import random

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.engine.request import SamplingParams

    rng = random.Random(3)
    prompts = [[rng.randrange(1024) for _ in range(rng.randrange(1, 90))] for _ in range(12)]
    eng = LLMEngine("tiny", device="cpu", max_running=6, max_batched_tokens=64, max_model_len=512,
                    num_blocks=num_blocks, overlap=overlap)
    rids = [eng.add_request(p, params=SamplingParams(max_new_tokens=max_new, eos_token_id=eos,
                                                     ignore_eos=eos is None)) for p in prompts]
    streamed = {}
    while eng.has_unfinished():
        for o in eng.step():
            streamed.setdefault(o.rid, []).extend(o.new_tokens)
    full = [eng.requests[r].meta.get("preempted_output", []) + eng.requests[r].output for r in rids]
    pre = sum(1 for r in eng.requests.values() if r.meta.get("preempted_output"))
    return full, [streamed.get(r, []) for r in rids], pre


def test_overlapped_scheduling_matches_synchronous():
    """Overlapped steps (launch n+1 before finishing n, PENDING tokens resolved on the device
    side) generate exactly the synchronous tokens: plain, with preemption (few pages) and
    with a stop token that ends a request one step after it was scheduled again."""
    for blocks in (96, 14):
        want, _, pre_a = _overlap_run(False, blocks)
        got, streamed, pre_b = _overlap_run(True, blocks)
        assert got == want and pre_a == pre_b
        if blocks == 96:
            assert streamed == got  # every token is reported once, in order
    assert pre_a > 0  # the small arena did preempt
    eos = want[0][3]
    want, _, _ = _overlap_run(False, 96, eos=eos)
    got, streamed, _ = _overlap_run(True, 96, eos=eos)
    assert got == want and streamed == got
    assert len(want[0]) == 4


def _spec_run(spec, blocks=128, eos=None, max_new=30):
    import random

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.engine.request import SamplingParams

    rng = random.Random(1)
    base = [rng.randrange(1000) for _ in range(40)]
    prompts = [base * 3, [rng.randrange(1000) for _ in range(50)], base[:20] * 4, [5, 6, 7] * 20]
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=128, max_model_len=512,
                    num_blocks=blocks, spec_tokens=spec)
    rids = [eng.add_request(p, params=SamplingParams(max_new_tokens=max_new, eos_token_id=eos,
                                                     ignore_eos=eos is None)) for p in prompts]
    streamed = {}
    while eng.has_unfinished():
        for o in eng.step():
            streamed.setdefault(o.rid, []).extend(o.new_tokens)
    full = [eng.requests[r].meta.get("preempted_output", []) + eng.requests[r].output for r in rids]
    return full, [streamed.get(r, []) for r in rids], eng


def test_speculative_decoding_matches_greedy():
    """Prompt-lookup drafts verified in one chunk per request give exactly the greedy tokens,
    stream every verified token once, stop at the length limit and at a stop token inside an
    accepted run, and survive preemption (few pages)."""
    want, _, _ = _spec_run(0)
    got, streamed, eng = _spec_run(4)
    assert got == want and streamed == got
    st = eng.scheduler.spec_stats
    assert st["verify_chunks"] > 0 and st["accepted"] > 0 and st["accepted"] <= st["proposed"]
    assert all(len(o) == 30 for o in got)
    for blocks in (24,):
        a, _, _ = _spec_run(0, blocks=blocks)
        b, _, _ = _spec_run(4, blocks=blocks)
        assert a == b
    eos = want[0][5]
    a, _, _ = _spec_run(0, eos=eos)
    b, s, _ = _spec_run(4, eos=eos)
    assert a == b and s == b


def test_runner_packs_mixed_batch_metadata():
    """Host packing of one mixed step (decode rows first, then a prefill chunk): token ids,
    positions, KV slots from the block tables, query starts, prefill tiles, sample rows and the
    graph-bucket padding rows (the role of the reference's engine/tests/test_input_batch.py)."""
    from lake_b200 import ops

    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=512, max_model_len=512, num_blocks=64)
    a = eng.add_request(list(range(1, 21)), max_new_tokens=4)
    b = eng.add_request(list(range(30, 63)), max_new_tokens=4)
    eng.step()  # both prompts prefilled: a and b decode next
    c = eng.add_request(list(range(100, 100 + 150)), max_new_tokens=2)
    out = eng.scheduler.schedule()
    assert [ch.req.rid for ch in out.chunks] == [a, b, c] and len(out.decode) == 2
    r = eng.runner
    t, s, ntiles, nrows, nd = r._pack(out, pad_decode_to=4)
    assert (s, nd, nrows) == (5, 4, 5) and t == 2 + 2 + 150
    ids, pos = r._v(r.np_i32, "ids"), r._v(r.np_i32, "pos")
    lens, qst = r._v(r.np_i32, "lens"), r._v(r.np_i32, "qstart")
    tiles = r._v(r.np_i32, "tiles", shape=(r.max_tiles, 4))
    bt = r._v(r.np_i32, "bt", shape=(r.max_seqs, r.maxb))
    slots, rows = r.np_i64[:t], r.np_i64[r.max_tokens:r.max_tokens + nrows]
    reqs = eng.requests
    for row, rid in enumerate([a, b]):  # decode rows: the last sampled token at its position
        req = reqs[rid]
        p = len(req.prompt) + len(req.output) - 1
        assert ids[row] == req.output[-1] and pos[row] == p and lens[row] == p + 1
        assert slots[row] == req.block_ids[p // 16] * 16 + p % 16
        assert list(bt[row, :len(req.block_ids)]) == list(req.block_ids)
    # two padding rows: zero-length sequences that write no KV and are sampled but ignored
    assert list(slots[2:4]) == [-1, -1] and list(lens[2:4]) == [0, 0]
    # the prefill chunk of c: rows 4.., one sample row (its last), tiles of PREFILL_TILE rows
    rc = reqs[c]
    assert list(qst[:6]) == [0, 1, 2, 3, 4, 154] and lens[4] == 150
    assert list(ids[4:154]) == list(range(100, 250)) and list(pos[4:154]) == list(range(150))
    want_slots = [rc.block_ids[p // 16] * 16 + p % 16 for p in range(150)]
    assert list(slots[4:154]) == want_slots
    k = ops.core.PREFILL_TILE
    assert ntiles == 2 and [list(x) for x in tiles[:2]] == [[4, 4, k, 0], [4, 4 + k, 150 - k, k]]
    assert list(rows) == [0, 1, 2, 3, 153]


def test_overlap_timeline_launches_next_step_before_collecting():
    """Launch/collect order with overlapped scheduling (the reference's
    runtime/tests/test_node_scheduler_mock.py:92-134 timeline check): step n+1 is launched
    before step n is collected, every launched step is collected exactly once, in order."""
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=64, max_model_len=256, num_blocks=64,
                    overlap=True)
    timeline, handles = [], []  # handles stay referenced so their ids are never reused
    launch, collect = eng.runner.launch, eng.runner.collect

    def rec_launch(out, bitmask=None):
        h = launch(out, bitmask)
        handles.append(h)
        timeline.append(("launch", id(h)))
        return h

    def rec_collect(h):
        timeline.append(("collect", id(h)))
        return collect(h)

    eng.runner.launch, eng.runner.collect = rec_launch, rec_collect
    eng.generate([[3, 4, 5] * 10, [7] * 12], max_new_tokens=6)
    launches = [h for k, h in timeline if k == "launch"]
    collects = [h for k, h in timeline if k == "collect"]
    assert launches == collects and len(launches) >= 6  # each step collected once, in launch order
    for i in range(len(launches) - 1):  # collect(n) only after launch(n + 1)
        assert timeline.index(("collect", launches[i])) > timeline.index(("launch", launches[i + 1]))


def test_idle_expert_parallel_rank_takes_every_step():
    """An expert-parallel rank with nothing scheduled still launches one (zero-token) forward
    per engine step (expert-parallel engines step synchronously), so the group's exchange counts
    stay aligned with ranks that have work."""
    eng = LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=64, max_model_len=256, num_blocks=64)
    eng.ec.ep = (1, 2, None)  # as rank 1 of a 2-rank group (the exchange itself needs GPUs)
    calls = []
    eng.runner.execute_null = lambda: calls.append(len(calls))
    for _ in range(3):
        assert eng.step() == []
    assert len(calls) == 3
    eng.add_request([5, 6, 7], max_new_tokens=2)
    while eng.has_unfinished():
        eng.step()
    n = len(calls)
    eng.step()
    assert len(calls) == n + 1
