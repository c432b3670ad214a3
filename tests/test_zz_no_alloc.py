"""Allocation-free decode attention entry point, called through its exported C
symbol. It must agree with the regular split-KV decode path (which takes its
scratch from caller-provided workspaces) on two calls in a row, and it must
refuse a batch whose partial results do not fit its fixed scratch array.

This file is collected last so that a run stopping at the first failure has
already run every other test."""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ETOO_LARGE = -100


def _lib():
    import lake_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.lakeb_paged_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    sz = lib.lakeb_paged_decode_noalloc_scratch_bytes
    sz.restype = ctypes.c_int64
    sz.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    return fn, sz


def _call(fn, q, out, arena, layer, hq, hkv, bt, sl, scale, splits):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), arena.data_ptr(), arena.shape[0],
              arena.shape[1], layer, hq, hkv, bt.data_ptr(), bt.stride(0), sl.data_ptr(), sl.shape[0], scale, splits,
              ctypes.c_void_p(stream))


def _case(dev, seed, nseq, hq, hkv, lens):
    g = torch.Generator(device=dev).manual_seed(seed)
    maxb = max((n + 15) // 16 for n in lens)
    nblocks = nseq * maxb + 2
    arena = (torch.randn(nblocks, 2, 2, hkv, 16, 128, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    bt = torch.randperm(nblocks, device=dev, generator=g)[: nseq * maxb].view(nseq, maxb).to(torch.int32)
    q = torch.randn(nseq, hq * 128, device=dev, generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    return arena, bt, q, sl


def _close(a, b, tol=2e-2):
    err = (a.float() - b.float()).abs().max().item()
    assert err <= tol * b.float().abs().max().item() + 1e-3, err


def test_noalloc_decode_matches_workspace_path_twice(cuda_dev):
    from lake_b200 import ops

    fn, scratch_bytes = _lib()
    scale = 1 / math.sqrt(128)
    for seed, (nseq, hq, hkv, lens) in enumerate([(3, 8, 2, [4096, 17, 2500]), (2, 32, 8, [1000, 3000])]):
        arena, bt, q, sl = _case(cuda_dev, seed, nseq, hq, hkv, lens)
        splits = ops.decode_splits(nseq, hkv, bt.shape[1])
        assert splits > 1, "the case must exercise the split-KV scratch"
        assert 0 < scratch_bytes(nseq, hq, hkv, splits) <= 8 << 20
        want = ops.paged_decode_attention(q, arena, 1, bt, sl, hq, hkv, scale, splits=splits)
        out = torch.empty_like(q)
        before = torch.cuda.memory_allocated(cuda_dev)
        rc = _call(fn, q, out, arena, 1, hq, hkv, bt, sl, scale, splits)
        torch.cuda.synchronize()
        assert rc == 0, rc
        assert torch.cuda.memory_allocated(cuda_dev) == before
        _close(out, want)


def test_noalloc_decode_rejects_oversized_batch(cuda_dev):
    fn, scratch_bytes = _lib()
    nseq, hq, hkv = 64, 128, 8
    splits = 32
    assert scratch_bytes(nseq, hq, hkv, splits) > 8 << 20
    arena, bt, q, sl = _case(cuda_dev, 7, nseq, hq, hkv, [32] * nseq)
    out = torch.zeros_like(q)
    rc = _call(fn, q, out, arena, 1, hq, hkv, bt, sl, 0.1, splits)
    assert rc == ETOO_LARGE
    assert out.abs().sum().item() == 0  # nothing launched
