"""Block-scaled fp8 (e4m3) weights: one fp32 scale per 128 x 128 block.

``quantize_blockwise(w)`` turns a bf16/fp32 weight [N, K] into ``Fp8Weight``:
e4m3 bytes [N, K] (uint8 view) and scales [ceil(N/128), ceil(K/128)] with
``scale = amax(block) / 448`` (448 = largest finite e4m3). GEMMs given an
``Fp8Weight`` run the W8A16 path of the tcgen05 GEMM: converter warps
dequantise each staged fp8 tile to bf16 in shared memory (value x block scale)
and the tensor cores run bf16 MMAs, so weight bytes read from HBM halve.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

E4M3_MAX = 448.0
BLOCK = 128


@dataclass
class Fp8Weight:
    q: torch.Tensor  # uint8 [N, K] (e4m3 bit patterns)
    s: torch.Tensor  # fp32 [ceil(N/128), ceil(K/128)]
    swiglu_tile: int = 256  # gate/up interleave of a SwiGLU weight: rows [gate tile/2 | up tile/2] per tile

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    @property
    def is_cuda(self):
        return self.q.is_cuda

    def dequant(self, dtype=torch.float32, swiglu_tile: int | None = None) -> torch.Tensor:
        """Dense weight; `swiglu_tile` re-lays a SwiGLU weight out in that gate/up interleave."""
        n, k = self.q.shape
        w = self.q.view(torch.float8_e4m3fn).to(torch.float32)
        s = self.s.repeat_interleave(BLOCK, 0)[:n].repeat_interleave(BLOCK, 1)[:, :k]
        d = w * s
        if swiglu_tile == 256 and self.swiglu_tile == 128:  # [half][gate|up] -> [gate|up][half] per 256 rows
            d = d.view(n // 256, 2, 2, 64, k).permute(0, 2, 1, 3, 4).reshape(n, k)
        return d.to(dtype)

    def rows(self, a: int, b: int) -> "Fp8Weight":
        """Rows [a, b) (block-aligned a) as a new weight, e.g. one rank's tensor-parallel shard."""
        assert a % BLOCK == 0
        return Fp8Weight(self.q[a:b].contiguous(), self.s[a // BLOCK:(b + BLOCK - 1) // BLOCK].contiguous(),
                         self.swiglu_tile)

    def cols(self, a: int, b: int) -> "Fp8Weight":
        assert a % BLOCK == 0
        return Fp8Weight(self.q[:, a:b].contiguous(), self.s[:, a // BLOCK:(b + BLOCK - 1) // BLOCK].contiguous(),
                         self.swiglu_tile)


def quantize_blockwise(w: torch.Tensor) -> Fp8Weight:
    n, k = w.shape
    nb, kb = (n + BLOCK - 1) // BLOCK, (k + BLOCK - 1) // BLOCK
    wf = w.float()
    pad = torch.zeros(nb * BLOCK, kb * BLOCK, dtype=torch.float32, device=w.device)
    pad[:n, :k] = wf
    blocks = pad.view(nb, BLOCK, kb, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    s = amax / E4M3_MAX
    q = (blocks / s[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).view(nb * BLOCK, kb * BLOCK)[:n, :k]
    return Fp8Weight(q.contiguous().to(torch.float8_e4m3fn).view(torch.uint8), s.contiguous())


def quantize_gate_up(w: torch.Tensor) -> Fp8Weight:
    """Block-scaled e4m3 of a SwiGLU weight in the 256-row interleave ([gate 128 | up 128] per 256
    rows), re-interleaved per 128 rows ([gate 64 | up 64]) first: the fp8 GEMMs run 128-wide tiles
    (one weight scale block per tile), each holding the gate and up rows of 64 outputs."""
    n, k = w.shape
    assert n % 256 == 0
    w = w.view(n // 256, 2, 2, 64, k).permute(0, 2, 1, 3, 4).reshape(n, k)  # [blk][gate|up][half] -> [blk][half][gate|up]
    q = quantize_blockwise(w)
    q.swiglu_tile = 128
    return q


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference of the W8A8 activation quantisation: e4m3 values (as float32) and fp32 scales
    [M, K/128], s = amax(|128-block|) / 448 (1 for an all-zero block), q = x * (1 / s) rounded to
    nearest e4m3 (saturating at 448)."""
    m, k = x.shape
    xb = x.float().view(m, k // BLOCK, BLOCK)
    amax = xb.abs().amax(-1)
    # tensor / tensor and reciprocal are IEEE divisions (a Python-scalar divisor would become a
    # multiplication by its reciprocal), as in the kernel
    s = torch.where(amax > 0, amax / torch.full_like(amax, E4M3_MAX), torch.ones_like(amax))
    q = (xb * torch.reciprocal(s)[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).to(torch.float32)
    return q.view(m, k), s


def unpack(w):
    """(tensor, scale-or-None) for the native bindings."""
    if isinstance(w, Fp8Weight):
        return w.q, w.s
    return w, None
