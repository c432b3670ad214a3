// QKV projection epilogue shared by the single-SM and the two-SM tcgen05 GEMMs: for one
// 128-wide head of one accumulator row, optional per-head RMSNorm (Qwen3), RoPE, and the
// stores (q rows to C; k / v rows into the paged KV arena and, for PD-split, into the decode
// instance's arena through its peer mapping).
#pragma once

#include "common.cuh"
#include "lakeb_kernels.h"

namespace lakeb {
namespace {

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
    u.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    u.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    u.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    d[i] = u;
  }
}

// Warp-collective store of one 64-byte piece per lane (32 fp32 -> bf16) to `dst` (this lane's
// row; nullptr: no store). The pieces pass through `stage` (2 KB of this warp's shared memory)
// so that each store instruction writes 8 rows x 64 contiguous bytes instead of 32 rows x 16
// bytes: over NVLink (peer arenas) that is 8 runs of 64 bytes rather than 32 scattered 16-byte
// writes. Chunk c of row r sits at r*4 + ((c + r/2) & 3) so both the row-wise writes and the
// chunk-wise reads are free of bank conflicts. Every lane of the warp must call it.
__device__ __forceinline__ void warp_store_rows64(uint4* stage, __nv_bfloat16* dst, const float* v, int lane) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    u.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    u.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    u.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    stage[lane * 4 + ((c + (lane >> 1)) & 3)] = u;
  }
  __syncwarp();
  const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), c = lane & 3;
    const unsigned long long d = __shfl_sync(0xffffffffu, mine, r);
    const uint4 u = stage[r * 4 + ((c + (r >> 1)) & 3)];
    if (d) reinterpret_cast<uint4*>(d)[c] = u;
  }
  __syncwarp();
}

__device__ __forceinline__ __nv_bfloat16* kv_ptr(const KVArenaView& kv, int64_t slot, int head, int which) {
  const int64_t blk = slot / kv.block_size;
  const int64_t off = slot - blk * kv.block_size;
  return kv.base + blk * kv.block_stride + kv.layer_offset + which * kv.kv_stride + head * kv.head_stride +
         off * 128;
}

// Head `head` of accumulator row `row` (this thread's TMEM lane; `tbase` addresses the head's
// 128 fp32 columns). Every lane of the warp calls it (the TMEM loads are warp-aligned). With
// `stage` (2 KB of this warp's shared memory) the peer-arena K/V stores are coalesced per warp.
__device__ __forceinline__ void qkv_head_epilogue(const GemmArgs& p, uint32_t tbase, int head, int row, bool row_ok,
                                                  uint4* stage = nullptr) {
  const int lane = threadIdx.x & 31;
  const bool is_q = head < p.n_q_heads;
  const bool is_k = !is_q && head < p.n_q_heads + p.n_kv_heads;
  int pos = 0;
  int64_t slot = -1, pslot = -1;
  if (row_ok) {
    pos = p.positions[row];
    if (!is_q) {
      slot = p.slots ? p.slots[row] : -1;
      if (p.peer_kv.base && p.peer_slots) pslot = p.peer_slots[row];
      // debug build: a slot past the arena is reported and its store skipped
      if (slot >= 0 && !in_bounds(p.kv.num_slots <= 0 || slot < p.kv.num_slots, p.status)) slot = -1;
      if (pslot >= 0 && !in_bounds(p.peer_kv.num_slots <= 0 || pslot < p.peer_kv.num_slots, p.status))
        pslot = -1;
    }
  }
  if (is_q || is_k) {
    const int kvh = head - p.n_q_heads;
    // per-head RMSNorm before RoPE (Qwen3): one pass over the head's 128 accumulators first
    const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
    float inv = 1.f;
    if (nw) {
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) ss += __uint_as_float(r[j]) * __uint_as_float(r[j]);
      }
      inv = rsqrtf(ss * (1.f / 128.f) + p.qk_eps);
    }
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      uint32_t r1[32], r2[32];
      tmem_ld32(tbase + half * 32, r1);
      tmem_ld32(tbase + 64 + half * 32, r2);
      tmem_ld_wait();
      float o1[32], o2[32];
      if (row_ok) {
        const float2* cs = p.rope_cs + static_cast<int64_t>(pos) * 64 + half * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float2 c = cs[j];
          float x1 = __uint_as_float(r1[j]);
          float x2 = __uint_as_float(r2[j]);
          if (nw) {
            x1 *= inv * __bfloat162float(nw[half * 32 + j]);
            x2 *= inv * __bfloat162float(nw[64 + half * 32 + j]);
          }
          o1[j] = x1 * c.x - x2 * c.y;
          o2[j] = x2 * c.x + x1 * c.y;
        }
        if (is_q) {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + row * p.ldc + head * 128;
          store_bf16x32(dst + half * 32, o1);
          store_bf16x32(dst + 64 + half * 32, o2);
        } else {
          if (slot >= 0) {
            __nv_bfloat16* dst = kv_ptr(p.kv, slot, kvh, 0);
            store_bf16x32(dst + half * 32, o1);
            store_bf16x32(dst + 64 + half * 32, o2);
          }
          if (pslot >= 0 && !stage) {
            __nv_bfloat16* dst = kv_ptr(p.peer_kv, pslot, kvh, 0);
            store_bf16x32(dst + half * 32, o1);
            store_bf16x32(dst + 64 + half * 32, o2);
          }
        }
      }
      if (is_k && stage && p.peer_kv.base) {  // warp-uniform: the head is the same for every lane
        __nv_bfloat16* dst = pslot >= 0 ? kv_ptr(p.peer_kv, pslot, kvh, 0) : nullptr;
        warp_store_rows64(stage, dst ? dst + half * 32 : nullptr, o1, lane);
        warp_store_rows64(stage, dst ? dst + 64 + half * 32 : nullptr, o2, lane);
      }
    }
  } else {
    const int kvh = head - p.n_q_heads - p.n_kv_heads;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(tbase + c * 32, r);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if (row_ok) {
        if (slot >= 0) store_bf16x32(kv_ptr(p.kv, slot, kvh, 1) + c * 32, v);
        if (pslot >= 0 && !stage) store_bf16x32(kv_ptr(p.peer_kv, pslot, kvh, 1) + c * 32, v);
      }
      if (stage && p.peer_kv.base)
        warp_store_rows64(stage, pslot >= 0 ? kv_ptr(p.peer_kv, pslot, kvh, 1) + c * 32 : nullptr, v, lane);
    }
  }
}

}  // namespace
}  // namespace lakeb
