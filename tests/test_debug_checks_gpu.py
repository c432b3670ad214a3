"""Bounds-checked debug build (lake_b200/_C_debug.so, ``python -m lake_b200._build --debug``).

Index checks in the kernels record "index out of bounds" in the status word and skip the
access instead of touching memory outside the buffer. The GPU case runs in a child process
with LAKEB_DEBUG_CHECKS=1 and feeds out-of-range page ids only after it has confirmed that the
loaded extension is the checked build; the paged-attention case is harmless in any build
(its K/V pages arrive by TMA, which fills out-of-range rows with zeros).
"""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import math, sys
import torch
from lake_b200 import ops
from lake_b200.ops import core
from lake_b200.ops._ext import native

if not native().debug_checks():
    sys.exit(77)  # not the checked build: feed it no bad index
dev = torch.device("cuda:0")
g = torch.Generator(device=dev).manual_seed(0)
nblocks, hq, hkv, layers = 40, 8, 2, 1
arena = (torch.randn(nblocks, layers, 2, hkv, 16, 128, device=dev, generator=g) * 0.5).to(torch.bfloat16)
bt = torch.arange(2 * 10, device=dev, dtype=torch.int32).view(2, 10)
sl = torch.tensor([150, 60], dtype=torch.int32, device=dev)
q = torch.randn(2, hq * 128, device=dev, generator=g).to(torch.bfloat16)
scale = 1 / math.sqrt(128)

def want():  # the CPU path of the same op is the fp32 oracle
    return ops.paged_decode_attention(q.float().cpu(), arena.float().cpu(), 0, bt.cpu(), sl.cpu(), hq, hkv, scale)

# 1. a block-table entry past the arena: reported, the kernel reads page 0 instead
bad = bt.clone()
bad[0, 3] = nblocks + 5
ops.paged_decode_attention(q, arena, 0, bad, sl, hq, hkv, scale)
torch.cuda.synchronize()
try:
    core.check_status(dev)
    sys.exit("no bounds error reported for a page id past the arena")
except RuntimeError as e:
    assert "out of bounds" in str(e), e
# the context is intact: a clean call matches the fp32 oracle
out = ops.paged_decode_attention(q, arena, 0, bt, sl, hq, hkv, scale)
core.check_status(dev)
err = (out.float().cpu() - want()).abs().max().item()
assert err < 3e-2, err

# 2. page copy with one destination page past the buffer: that page is skipped, the rest land
src = torch.randn(8, 1024, device=dev, generator=g)
dst = torch.zeros(6, 1024, device=dev)
pb = 1024 * 4
ops.page_copy(src, dst, torch.tensor([1, 2, 3], device=dev), torch.tensor([0, 99, 5], device=dev), pb)
torch.cuda.synchronize()
try:
    core.check_status(dev)
    sys.exit("no bounds error reported for a page copy past the buffer")
except RuntimeError as e:
    assert "out of bounds" in str(e), e
assert torch.equal(dst[0], src[1]) and torch.equal(dst[5], src[3])
assert dst[1:5].abs().sum().item() == 0
print("debug checks ok")
'''


@pytest.mark.gpu
def test_debug_build_reports_out_of_range_indices(cuda_dev):
    if not os.path.exists(os.path.join(ROOT, "lake_b200", "_C_debug.so")):
        pytest.skip("debug build absent (python -m lake_b200._build --debug)")
    env = dict(os.environ, LAKEB_DEBUG_CHECKS="1")
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    if r.returncode == 77:
        pytest.skip("loaded extension is not the checked build")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "debug checks ok" in r.stdout


def test_debug_build_rules():
    """The checked build is its own target: -DLAKEB_DEBUG_CHECKS, module _C_debug, no host library."""
    from lake_b200 import _build

    text = open(_build.write_ninja(debug=True)).read()
    assert "-DLAKEB_DEBUG_CHECKS" in text and "_C_debug.so" in text and "-DLAKEB_MODULE=_C_debug" in text
    assert "_host.so" not in text
    rel = open(_build.write_ninja(debug=False)).read()
    assert "-DLAKEB_DEBUG_CHECKS" not in rel and "_C.so" in rel
