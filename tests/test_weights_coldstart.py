"""Host weight cache (C++) and layer-async cold start."""
import random

import pytest
import torch

from lake_b200 import _host as H


def test_weight_cache_put_read_evict_pin():
    c = H.WeightCache(4096, pinned=False)
    a = torch.arange(256, dtype=torch.int32)  # 1 KiB
    k = H.WeightCache.key("m", "r", "layers.0.qkv_proj")
    assert c.put(k, a.data_ptr(), a.numel() * 4)
    out = torch.zeros_like(a)
    assert c.read(k, out.data_ptr(), out.numel() * 4) and torch.equal(out, a)
    c.pin(k)
    for i in range(5):  # fill past capacity: the pinned entry survives, others are evicted
        assert c.put(H.WeightCache.key("m", "r", f"w{i}"), a.data_ptr(), 1024)
    assert c.contains(k) and c.evictions >= 1 and c.used <= 4096
    c.unpin(k)
    assert c.erase(k) and not c.contains(k)
    assert not c.put("huge", a.data_ptr(), 1 << 20)


@pytest.mark.gpu
def test_layer_async_cold_start_matches_direct_load():
    from lake_b200.engine.llm_engine import LLMEngine
    from lake_b200.runtime.coldstart import LayerAsyncLoader, load_sequential, stage_model

    kw = dict(device="cuda:0", max_running=4, max_batched_tokens=256, max_model_len=1024, num_blocks=128)
    src = LLMEngine("tiny-gpu", seed=3, **kw)
    rng = random.Random(1)
    prompts = [[rng.randrange(2048) for _ in range(n)] for n in (20, 90)]
    want = src.generate(prompts, max_new_tokens=6)
    cache = H.WeightCache(256 << 20)
    nbytes = stage_model(src.model, cache, "tiny-gpu")
    dst = LLMEngine("tiny-gpu", seed=99, **kw)  # different random weights until the load lands
    loader = LayerAsyncLoader(dst.model, cache, "tiny-gpu", serve_after_layers=1)
    loader.start()
    got = dst.generate(prompts, max_new_tokens=6)  # admitted while layers may still be streaming
    m = loader.finish()
    assert got == want
    assert m.bytes_loaded == nbytes and m.time_to_serve_gate <= m.time_to_weights_done
    seq = load_sequential(dst.model, cache, "tiny-gpu")
    assert seq.bytes_loaded == nbytes and cache.hits > 0
