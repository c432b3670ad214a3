"""Allocation-free decode attention entry point, called through its exported C
symbol. It must agree with the regular split-KV decode path (which takes its
scratch from caller-provided workspaces) on two calls in a row, and it must
refuse a batch whose partial results do not fit its fixed scratch array.

This file is collected last so that a run stopping at the first failure has
already run every other test."""
import ctypes
import gc
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ETOO_LARGE = -100
EARG = -102


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


def _oracle(q, arena, layer, bt, sl, hq, hkv, scale):
    from lake_b200.oracle import ops_ref as ref

    n = sl.shape[0]
    qs = torch.arange(n + 1, dtype=torch.int32)
    pos = (sl.cpu() - 1).to(torch.int32)
    return ref.paged_attention(q[:n].float().cpu(), arena.float().cpu(), layer, bt.cpu(), sl.cpu(), qs, pos, hq, hkv,
                               scale)


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
        outs = [torch.empty_like(q) for _ in range(3)]
        # the first call on a device may load the library's GPU module (which creates the fixed
        # scratch array); the calls after it must not change the device's free memory at all
        assert _call(fn, q, outs[0], arena, 1, hq, hkv, bt, sl, scale, splits) == 0
        torch.cuda.synchronize()
        gc.collect()  # tensors left by earlier tests must not be freed inside the measured window
        free0 = torch.cuda.mem_get_info(cuda_dev)[0]
        alloc0 = torch.cuda.memory_allocated(cuda_dev)
        for out in outs[1:]:  # the same shape twice, over the previous call's scratch contents
            assert _call(fn, q, out, arena, 1, hq, hkv, bt, sl, scale, splits) == 0
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info(cuda_dev)[0] >= free0  # the driver handed out nothing
        assert torch.cuda.memory_allocated(cuda_dev) <= alloc0  # nor did torch's allocator
        for out in outs:
            _close(out, want)
        assert torch.equal(outs[1], outs[2])  # deterministic over reused scratch
        _close(outs[2].float().cpu(), _oracle(q, arena, 1, bt, sl, hq, hkv, scale))


def test_noalloc_decode_rejects_bad_arguments(cuda_dev):
    fn, _ = _lib()
    arena, bt, q, sl = _case(cuda_dev, 3, 2, 8, 2, [100, 200])
    out = torch.zeros_like(q)
    for layer in (-1, 2):  # the arena has 2 layers
        assert _call(fn, q, out, arena, layer, 8, 2, bt, sl, 0.1, 0) == EARG
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), arena.data_ptr(), arena.shape[0], arena.shape[1],
            0, 8, 2, bt.data_ptr(), 0, sl.data_ptr(), 2, 0.1, 0, ctypes.c_void_p(stream))
    assert rc == EARG  # bt_stride 0
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0  # nothing launched


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_decode_on_two_devices_in_one_process(cuda_dev):
    """The scratch address and the kernels' shared-memory limit are both per device: the second
    device's first call must set them up for that device, not reuse the first device's."""
    from lake_b200 import ops

    fn, _ = _lib()
    scale = 1 / math.sqrt(128)
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            arena, bt, q, sl = _case(dev, 11 + d, 3, 8, 2, [4096, 17, 2500])
            splits = ops.decode_splits(3, 2, bt.shape[1])
            want = ops.paged_decode_attention(q, arena, 1, bt, sl, 8, 2, scale, splits=splits)
            out = torch.empty_like(q)
            assert _call(fn, q, out, arena, 1, 8, 2, bt, sl, scale, splits) == 0
            torch.cuda.synchronize(dev)
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
