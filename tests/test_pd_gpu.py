"""PD-split on two GPUs: the prefill GPU's QKV epilogue stores K/V into the decode
GPU's arena over NVLink (IPC-mapped peer memory); the decode GPU's tokens must be
identical to a colocated run of the same model on one GPU."""
import json
import os
import random
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _prompts():
    rng = random.Random(11)
    prefix = [rng.randrange(2048) for _ in range(80)]
    return [prefix + [rng.randrange(2048) for _ in range(n)] for n in (5, 60, 200, 1, 33)]


def _worker(rank, port, out_dir):
    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.ops import core
    from lake_b200.parallel import pd

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    role = "prefill" if rank == 0 else "decode"
    eng = LLMEngine("tiny-gpu", device=f"cuda:{rank}", max_running=8, max_batched_tokens=256, max_model_len=1024,
                    num_blocks=256, use_cuda_graphs=False, shared_arena=(role == "decode"))
    side = pd.connect_pair(eng, role, rank, 1 - rank, None, job=f"g{port}")
    if role == "prefill":
        pd.serve_prefill(side)
        core.check_status()
    else:
        prompts = _prompts()
        for p in prompts:
            assert side.submit(p, 8)
        while side.inflight:
            side.poll()
            if eng.has_unfinished():
                eng.step()
        outs = [eng.requests[f"pd-{i}"].output for i in range(len(prompts))]
        want = LLMEngine("tiny-gpu", device=f"cuda:{rank}", max_running=8, max_batched_tokens=256,
                         max_model_len=1024, num_blocks=256, use_cuda_graphs=False).generate(prompts, max_new_tokens=8)
        side.shutdown()
        core.check_status()
        with open(os.path.join(out_dir, "res.json"), "w") as f:
            json.dump({"outs": outs, "want": want, "kv_bytes": side.kv_bytes}, f)
    dist.barrier()
    dist.destroy_process_group()


def test_pd_split_two_gpus_matches_colocated(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    mp.spawn(_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    res = json.load(open(tmp_path / "res.json"))
    assert res["outs"] == res["want"]
    assert res["kv_bytes"] > 0
