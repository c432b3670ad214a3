"""Tensor parallel over NVLink peer memory on 2, 4 and 8 GPUs (each size runs when the box
has that many GPUs).

1. Fused collectives vs an fp32 PyTorch reference: row-parallel GEMM whose
   epilogue pushes partial rows to their owners (reduce-scatter), the owner's
   reduce + residual + RMSNorm + all-gather push, and a column-parallel SwiGLU
   GEMM that waits per row shard.
2. A TP engine generates the same greedy tokens as the TP=1 engine (bf16
   rounding of the split partial sums may flip a near-tie, after which that
   sequence diverges: >= 90% agreement at TP=2, >= 80% at TP=4 and 8, where the
   partial sums are split four and eight ways; the fused-op numerics in 1 are
   the exactness check).
   At TP=2 the model is `tiny-gpu`; at TP=4 and 8 it is widened to one KV head
   per rank (2 query heads, 256 hidden and 256 FFN columns per rank).
"""
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


def _fused_numerics(rank, world, out):
    import torch.distributed as dist

    from lake_b200.ops import core
    from lake_b200.ops import tp as tpops
    from lake_b200.oracle import ops_ref as ref
    from lake_b200.parallel.tp import TPGroup

    dev = torch.device(f"cuda:{rank}")
    H, K, I = 512, 768, 512  # hidden, K per rank (o_proj input slice), intermediate per rank
    # 300 tokens: shards straddle 128-row tiles (single-SM kernel); 1100: the two-SM kernel's
    # 256-row pair tiles straddle the shard boundary at row 550
    g = TPGroup(rank, world, dev, 1100 + world, H, 64)
    for M in (300, 1100):
        mr = g.rows_per_rank(M)
        t = mr * world
        gen = torch.Generator().manual_seed(100 + rank + M)
        a = (torch.randn(t, K, generator=gen) * 0.5).to(torch.bfloat16)
        w_o = (torch.randn(H, K, generator=gen) * 0.05).to(torch.bfloat16)
        h = torch.randn(mr, H, generator=gen).to(torch.bfloat16)
        w_n = (1.0 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(7))).to(torch.bfloat16)
        w_gu = (torch.randn(2 * I, H, generator=gen) * 0.05).to(torch.bfloat16)
        parts = [None] * world
        dist.all_gather_object(parts, (a, w_o, h))
        # fp32 reference over the whole group
        full = sum(ref.linear(p[0].float(), p[1].float()) for p in parts)  # [t, H]
        h_full = torch.cat([p[2].float() for p in parts]) + full
        h_full = h_full.to(torch.bfloat16).float()
        y = h_full * torch.rsqrt(h_full.pow(2).mean(-1, keepdim=True) + 1e-5) * w_n.float()
        act_ref = ref.swiglu_from_interleaved(ref.linear(y.to(torch.bfloat16).float(), w_gu.float()))

        a_d, w_o_d, h_d, w_n_d, w_gu_d = (x.to(dev) for x in (a, w_o, h, w_n, w_gu))
        act = torch.empty(t, I, dtype=torch.bfloat16, device=dev)
        for _ in range(3):  # repeated calls exercise the counter totals and slot rotation
            h_d.copy_(h.to(dev))
            tpops.linear_rs(a_d, w_o_d, g.gemm_rs(0, mr, H, K))
            tpops.norm_push(h_d, w_n_d, 1e-5, g.norm_push(mr, 0, 0))
            tpops.linear_swiglu_ag(g.a_full[0][:t], w_gu_d, act, g.gemm_ag(0, mr))
            g.end_step()
        torch.cuda.synchronize(dev)
        core.check_status(dev)
        r0 = rank * mr
        err_h = (h_d.float().cpu() - h_full[r0:r0 + mr]).abs().max().item()
        err_y = (g.a_full[0][:t].float().cpu() - y).abs().max().item()
        err_act = ((act.float().cpu() - act_ref).abs().max() / act_ref.abs().max()).item()
        out[f"m{M}"] = dict(err_h=err_h, err_y=err_y, err_act=err_act)


def _overrides(world):
    if world == 2:
        return {}
    return {"hidden": 256 * world, "n_q_heads": 2 * world, "n_kv_heads": world, "intermediate": 256 * world}


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.ops import core

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    _fused_numerics(rank, world, res)
    rng = random.Random(5)
    prompts = [[rng.randrange(2048) for _ in range(n)] for n in (7, 64, 150, 33, 1, 90)]
    # decode steps replay CUDA graphs (collective targets device-resident); mixed steps run eagerly
    ov = _overrides(world)
    eng = LLMEngine("tiny-gpu", device=f"cuda:{rank}", max_running=8, max_batched_tokens=256, max_model_len=1024,
                    num_blocks=256, use_cuda_graphs=True, tp=(rank, world, None), model_overrides=ov)
    eng.runner.capture_graphs()
    outs = eng.generate(prompts, max_new_tokens=8)
    core.check_status()
    res["outs"] = outs
    del eng
    # block-scaled fp8 weights under TP (the fp8 kernels' own grids size the counter waits)
    eng8 = LLMEngine("tiny-gpu", device=f"cuda:{rank}", max_running=8, max_batched_tokens=256, max_model_len=1024,
                     num_blocks=256, use_cuda_graphs=True, tp=(rank, world, None), weight_dtype="fp8",
                     model_overrides=ov)
    eng8.runner.capture_graphs()
    res["outs8"] = eng8.generate(prompts, max_new_tokens=8)
    core.check_status()
    del eng8
    if rank == 0:
        want = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=256, max_model_len=1024,
                         num_blocks=256, use_cuda_graphs=False, model_overrides=ov).generate(prompts, max_new_tokens=8)
        res["want"] = want
        res["want8"] = LLMEngine("tiny-gpu", device="cuda:0", max_running=8, max_batched_tokens=256,
                                 max_model_len=1024, num_blocks=256, use_cuda_graphs=False,
                                 weight_dtype="fp8", model_overrides=ov).generate(prompts, max_new_tokens=8)
    with open(os.path.join(out_dir, f"res{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_fused_collectives_and_engine(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    rs = [json.load(open(tmp_path / f"res{r}.json")) for r in range(world)]
    r0 = rs[0]
    for r in rs:
        for m in ("m300", "m1100"):
            assert r[m]["err_h"] < 0.1, (m, r[m])
            assert r[m]["err_y"] < 0.1, (m, r[m])
            assert r[m]["err_act"] < 3e-2, (m, r[m])
    assert all(r["outs"] == r0["outs"] for r in rs)  # every rank computes the same tokens
    flat_got = [t for o in r0["outs"] for t in o]
    flat_want = [t for o in r0["want"] for t in o]
    agree = sum(a == b for a, b in zip(flat_got, flat_want)) / len(flat_want)
    need = 0.9 if world == 2 else 0.8
    assert agree >= need, (agree, r0["outs"], r0["want"])
    assert all(r["outs8"] == r0["outs8"] for r in rs)
    got8 = [t for o in r0["outs8"] for t in o]
    want8 = [t for o in r0["want8"] for t in o]
    agree8 = sum(a == b for a, b in zip(got8, want8)) / len(want8)
    assert agree8 >= need, (agree8, r0["outs8"], r0["want8"])
