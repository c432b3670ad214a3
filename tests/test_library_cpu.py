"""CPU tests of the library comparator model (models/library.py) under the engine's parallel
plumbing: tensor parallel over two gloo ranks (Megatron layout, all_reduce after the row-parallel
GEMMs) and prefill/decode split with the page copies into the decode rank's arena. Both must give
the tokens of a single-process native run of the same weights (2-layer plumbing model, fp32)."""
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
    rng = random.Random(7)
    prefix = [rng.randrange(1024) for _ in range(40)]
    return [prefix + [rng.randrange(1024) for _ in range(n)] for n in (5, 23, 1)]


def _engine(**kw):
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.models.llama import DecoderLM

    eng = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512, num_blocks=96,
                    model_impl="library", **kw)
    eng.model._from_native(DecoderLM(eng.cfg, "cpu", seed=0).w)
    return eng


def _want(prompts, n):
    from lake_b200.engine.llm_engine import LLMEngine

    ref = LLMEngine("tiny", device="cpu", max_running=8, max_batched_tokens=64, max_model_len=512, num_blocks=96)
    return ref.generate(prompts, max_new_tokens=n)


def _worker_tp(rank, port, out_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    eng = _engine(tp=(rank, 2, None), overlap=True)
    assert eng.model.hq == 2 and eng.model.hk == 1 and eng.arena.shape[3] == 1
    outs = eng.generate(_prompts(), max_new_tokens=6)
    if rank == 0:
        with open(os.path.join(out_dir, "tp.json"), "w") as f:
            json.dump({"outs": outs, "want": _want(_prompts(), 6)}, f)
    dist.barrier()
    dist.destroy_process_group()


def test_library_tensor_parallel_matches_native():
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker_tp, args=(_free_port(), d), nprocs=2, join=True)
        res = json.load(open(os.path.join(d, "tp.json")))
    assert res["outs"] == res["want"]


def _worker_pd(rank, port, out_dir):
    import torch.distributed as dist

    from lake_b200.parallel import pd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    role = "prefill" if rank == 0 else "decode"
    eng = _engine(shared_arena=(role == "decode"))
    side = pd.connect_pair(eng, role, rank, 1 - rank, None, job=f"l{port}", shm_path=eng.arena_path)
    if role == "prefill":
        pd.serve_prefill(side)
    else:
        prompts = _prompts()
        for p in prompts:
            assert side.submit(p, 8)
        while side.inflight:
            side.poll()
            eng.step()
        outs = [eng.requests[f"pd-{i}"].output for i in range(len(prompts))]
        side.shutdown()
        with open(os.path.join(out_dir, "pd.json"), "w") as f:
            json.dump({"outs": outs, "want": _want(prompts, 8)}, f)
    dist.barrier()
    side.close()
    dist.destroy_process_group()
    if eng.arena_path:
        from lake_b200.parallel.peer import unlink_shared

        unlink_shared(eng.arena_path)


def test_library_pd_split_matches_native(tmp_path):
    mp.spawn(_worker_pd, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    res = json.load(open(tmp_path / "pd.json"))
    assert res["outs"] == res["want"]
