"""PD-split on CPU with two gloo ranks: the prefill rank writes K/V into the
decode rank's arena (shared /dev/shm mapping standing in for NVLink P2P) and the
decode rank's tokens must equal a colocated single-process run (the 2-layer
plumbing model, fp32), including a request the decode instance prefills itself
(overflow of a saturated prefill partner)."""
import json
import os
import random
import socket

import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _prompts():
    rng = random.Random(5)
    prefix = [rng.randrange(1024) for _ in range(48)]
    return [prefix + [rng.randrange(1024) for _ in range(n)] for n in (3, 20, 40, 1)]


def _worker(rank, port, out_dir):
    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.parallel import pd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    role = "prefill" if rank == 0 else "decode"
    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                    num_blocks=96, shared_arena=(role == "decode"))
    side = pd.connect_pair(eng, role, rank, 1 - rank, None, job=f"t{port}", shm_path=eng.arena_path)
    if role == "prefill":
        pd.serve_prefill(side)
    else:
        prompts = _prompts()
        # the last request is prefilled on the decode instance itself (overflow while its prefill
        # partner is saturated): same tokens, no grant
        rids = [side.submit(p, 8, local=(i == len(prompts) - 1)) for i, p in enumerate(prompts)]
        assert all(rids) and rids[-1].startswith("dd-") and side.local == 1
        while side.inflight:
            side.poll()
            eng.step()
        outs = [eng.requests[r].output for r in rids]
        ref = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512, num_blocks=96)
        want = ref.generate(prompts, max_new_tokens=8)
        side.shutdown()
        with open(os.path.join(out_dir, "res.json"), "w") as f:
            json.dump({"outs": outs, "want": want, "kv_bytes": side.kv_bytes}, f)
    dist.barrier()
    side.close()  # every rank is done with the rings: the creator unlinks them
    dist.destroy_process_group()
    if eng.arena_path:
        from lake_b200.parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def test_pd_split_matches_colocated(tmp_path):
    port = _free_port()
    mp.spawn(_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    res = json.load(open(tmp_path / "res.json"))
    assert res["outs"] == res["want"]
    assert res["kv_bytes"] > 0


def _worker_m2o(rank, port, out_dir):
    """Two prefill ranks feed one decode rank (many-to-one)."""
    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.parallel import pd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=3)
    role = "prefill" if rank < 2 else "decode"
    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                    num_blocks=96, shared_arena=(role == "decode"))
    partner = 2 if role == "prefill" else [0, 1]
    side = pd.connect_pair(eng, role, rank, partner, None, job=f"m{port}", shm_path=eng.arena_path)
    if role == "prefill":
        pd.serve_prefill(side)
    else:
        prompts = _prompts()
        for p in prompts:
            assert side.submit(p, 6)
        assert min(side.outstanding) >= 1  # both prefill instances got work
        while side.inflight:
            side.poll()
            eng.step()
        outs = [eng.requests[f"pd-{i}"].output for i in range(len(prompts))]
        want = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                         num_blocks=96).generate(prompts, max_new_tokens=6)
        side.shutdown()
        with open(os.path.join(out_dir, "m2o.json"), "w") as f:
            json.dump({"outs": outs, "want": want}, f)
    dist.barrier()
    side.close()  # every rank is done with the rings: the creator unlinks them
    dist.destroy_process_group()
    if eng.arena_path:
        from lake_b200.parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def test_pd_many_prefill_to_one_decode(tmp_path):
    port = _free_port()
    mp.spawn(_worker_m2o, args=(port, str(tmp_path)), nprocs=3, join=True)
    res = json.load(open(tmp_path / "m2o.json"))
    assert res["outs"] == res["want"]


def _worker_mesh(rank, port, out_dir):
    """Two prefill ranks [0, 1] each serve both decode ranks [2, 3] (many-to-many): a prefill
    step holds the grants of one decode instance only and stores its K/V into that instance's
    arena; every decode instance's tokens equal a colocated run."""
    import time

    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.parallel import pd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=4)
    decoders = dist.new_group([2, 3])  # collective: every rank creates it
    role = "prefill" if rank < 2 else "decode"
    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                    num_blocks=96, shared_arena=(role == "decode"))
    if role == "prefill":
        side = pd.connect_pair(eng, role, rank, None, None, job=f"x{port}", shm_path=eng.arena_path,
                               decode_instances=[2, 3])
        steps = []
        real_step = eng.step

        def step():  # record each step's destinations
            out = real_step()
            if eng.last_step is not None:
                steps.append(sorted({c.req.meta.get("pd_dest") for c in eng.last_step.prefill}))
            return out

        eng.step = step
        pd.serve_prefill(side)
        res = {"dests": steps}
    else:
        side = pd.connect_pair(eng, role, rank, [0, 1], None, job=f"x{port}", shm_path=eng.arena_path)
        prompts = _prompts() if rank == 2 else [p[::-1] for p in _prompts()]
        for p in prompts:
            assert side.submit(p, 6)
        t0 = time.perf_counter()
        while side.inflight:
            side.poll()
            if eng.has_unfinished():
                eng.step()
            else:
                time.sleep(0.001)
            assert time.perf_counter() - t0 < 120
        res = {"outs": [eng.requests[f"pd-{i}"].output for i in range(len(prompts))],
               "want": LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                                 num_blocks=96).generate(prompts, max_new_tokens=6),
               "linked": len(side.links)}
        dist.barrier(group=decoders)  # both decode instances done before either exits
        side.shutdown()
    with open(os.path.join(out_dir, f"x{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    side.close()
    dist.destroy_process_group()
    if eng.arena_path:
        from lake_b200.parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def test_pd_many_to_many_prefill_serves_several_decode_instances(tmp_path):
    port = _free_port()
    mp.spawn(_worker_mesh, args=(port, str(tmp_path)), nprocs=4, join=True)
    for r in (2, 3):
        res = json.load(open(tmp_path / f"x{r}.json"))
        assert res["outs"] == res["want"] and res["linked"] == 2
    dests = [d for r in (0, 1) for d in json.load(open(tmp_path / f"x{r}.json"))["dests"]]
    assert all(len(d) <= 1 for d in dests)  # one destination per prefill step
    assert {x for d in dests for x in d} == {0, 1}  # and both destinations were served


def _worker_groups(rank, port, out_dir):
    """Two-rank prefill instance [0, 1] feeds a two-rank decode instance [2, 3]: the leaders
    decide, the followers replay (page grants, adoptions, steps) through GroupCtl, and P's
    rank i writes into D's rank i arena. Plain engines stand in for the TP shards, so every
    rank must produce the colocated tokens."""
    import time

    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.parallel import pd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=4)
    role = "prefill" if rank < 2 else "decode"
    members = [0, 1] if role == "prefill" else [2, 3]
    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                    num_blocks=96, shared_arena=(role == "decode"))
    partner = [2, 3] if role == "prefill" else [0]
    side = pd.connect_pair(eng, role, rank, partner, None, job=f"g{port}", shm_path=eng.arena_path,
                           members=members)
    prompts = _prompts()
    res = None
    if role == "prefill":
        pd.serve_prefill(side)
        res = {"prefill_steps": side.steps}
    elif rank == 2:
        for p in prompts:
            assert side.submit(p, 8)
        t0 = time.perf_counter()
        while side.inflight:
            side.poll()
            if eng.has_unfinished():
                side.step()
            else:
                time.sleep(0.001)
            assert time.perf_counter() - t0 < 120
        side.phase(7)
        res = {"outs": [eng.requests[f"pd-{i}"].output for i in range(len(prompts))], "kv": side.kv_bytes}
        side.shutdown()
    else:
        assert side.follow() == 7
        res = {"outs": [eng.requests[f"pd-{i}"].output for i in range(len(prompts))]}
        assert side.follow() == -1
    side.close()
    if rank == 0:
        res["want"] = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                                num_blocks=96).generate(prompts, max_new_tokens=8)
    with open(os.path.join(out_dir, f"g{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()
    if eng.arena_path:
        from lake_b200.parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def test_pd_tensor_parallel_instances_replay_leader(tmp_path):
    port = _free_port()
    mp.spawn(_worker_groups, args=(port, str(tmp_path)), nprocs=4, join=True)
    r = [json.load(open(tmp_path / f"g{i}.json")) for i in range(4)]
    want = r[0]["want"]
    assert r[2]["outs"] == want
    assert r[3]["outs"] == want
    assert r[0]["prefill_steps"] == r[1]["prefill_steps"] > 0
    assert r[2]["kv"] > 0


def _worker_direct(rank, port, out_dir):
    """A session's second turn extends a prefix the decode instance already holds: it is
    prefilled there (D-direct) instead of on the prefill instance, with the same tokens."""
    import time

    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.parallel import pd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    role = "prefill" if rank == 0 else "decode"
    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512,
                    num_blocks=96, shared_arena=(role == "decode"))
    side = pd.connect_pair(eng, role, rank, 1 - rank, None, job=f"d{port}", shm_path=eng.arena_path)
    if role == "prefill":
        pd.serve_prefill(side)
        res = {"prefills": side.first_tokens}
    else:
        import random

        rng = random.Random(9)
        turn1 = [rng.randrange(1024) for _ in range(70)]

        def run_until_idle():
            t0 = time.perf_counter()
            while side.inflight:
                side.poll()
                if eng.has_unfinished():
                    eng.step()
                else:
                    time.sleep(0.001)
                assert time.perf_counter() - t0 < 60

        assert side.submit(turn1, 6)
        run_until_idle()
        out1 = eng.requests["pd-0"].output
        turn2 = turn1 + out1 + [rng.randrange(1024) for _ in range(20)]
        assert side.local_hit(turn2) >= 64
        assert side.submit(turn2, 6)
        run_until_idle()
        out2 = eng.requests["dd-1"].output
        ref = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512, num_blocks=96)
        want = ref.generate([turn1, turn2], max_new_tokens=6)
        res = {"outs": [out1, out2], "want": want, "direct": side.direct}
        side.shutdown()
    with open(os.path.join(out_dir, f"d{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()
    side.close()
    if eng.arena_path:
        from lake_b200.parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def test_pd_decode_direct_for_a_cached_prefix(tmp_path):
    port = _free_port()
    mp.spawn(_worker_direct, args=(port, str(tmp_path)), nprocs=2, join=True)
    d = json.load(open(tmp_path / "d1.json"))
    p = json.load(open(tmp_path / "d0.json"))
    assert d["outs"] == d["want"]
    assert d["direct"] == 1 and p["prefills"] == 1  # only the first turn went to the prefill instance


def test_cpu_plumbing_prefill_pool_decode():
    """The CPU plumbing configuration: a prefill worker writes every prompt's pages to the KV pool
    (radix/location authority + tier storage), a separate decode worker promotes them at admission
    and decodes 16 greedy steps; its logits equal a colocated run's to 1e-5."""
    from lake_b200.bench.cpu_plumbing import run

    r = run()
    assert r["pool_written_blocks"] == 8 + 8 * 2  # the shared 128-token prefix is stored once
    assert r["pool_prefix_hit_blocks"] == [10] * 8
    assert r["promoted_blocks"] > 0 and r["tokens_equal"]
    assert r["compared_positions"] == 8 * 16 and r["logits_match_1e-5"]
