// Persistent bf16 GEMM for sm_100a: TMA -> shared memory (128-byte swizzle),
// tcgen05.mma with fp32 accumulators in tensor memory, warp-specialised.
//
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  : epilogue (tcgen05.ld -> registers -> fused op -> global)
//
// The two accumulator buffers in TMEM let the epilogue of tile t overlap the
// main loop of tile t+1. Epilogues are fused per call site of the transformer:
// plain store, residual add (o_proj / down_proj), SwiGLU (gate_up), the QKV
// projection with RoPE and the paged-KV write (local arena and, for
// prefill->decode disaggregation, the decode GPU's arena through P2P stores),
// and a greedy-argmax over the vocabulary (lm_head) that never materialises
// logits.
//
// Reference parity: replaces the nn.Linear shells of the reference model
// (python/lake/engine/model_executor/models/qwen/qwen3.py:100-113,133-147,230-240),
// which never execute there.
#include "common.cuh"
#include <cuda_fp8.h>

#include "lakeb_kernels.h"
#include "qkv_epilogue.cuh"
#include "tma_host.h"

namespace lakeb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

template <int BN, int STAGES, bool W8 = false>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kB8Bytes = W8 ? BN * kBK : 0;  // fp8 staging of B (W8A16)
  static constexpr int kStageBytes = kABytes + kBBytes + kB8Bytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[S], empty[S], land[S] (W8), tmem_full[3], tmem_empty[3] (two accumulators; W8A8: three
  // k-block partials), final_ready, final_free (W8A8), tmem slot, abort flag, split flag
  static constexpr int kBytes = kBarOffset + (3 * STAGES + 8) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

// Threads per CTA: TMA warp, MMA warp, 4 epilogue warps (+ 4 fp8 converter warps for W8A16; W8A8:
// 8 epilogue warps, two per TMEM lane quarter, each promoting 64 of the tile's 128 columns).
template <bool W8, bool A8 = false>
constexpr int threads_of() {
  return (W8 || A8) ? 320 : 192;
}

// Dequantise one 64-byte fp8 row (64 e4m3 values of one output column n) into a bf16 row of the
// 128-byte-swizzled K-major B tile, scaled by the row's block scale.
__device__ __forceinline__ void convert_fp8_row(const uint8_t* src, uint8_t* dst_row, int row, float scale) {
  const int sw = row & 7;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = reinterpret_cast<const uint4*>(src)[q];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t out[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] & 0xFFFFu), __NV_E4M3);
      const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] >> 16), __NV_E4M3);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
      out[2 * i] = pack_bf16x2(a.x * scale, a.y * scale);
      out[2 * i + 1] = pack_bf16x2(b.x * scale, b.y * scale);
    }
    // 16 fp8 in -> 32 bytes of bf16 out = chunks 2q, 2q+1 of the 128-byte row
    *reinterpret_cast<uint4*>(dst_row + (((2 * q) ^ sw) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<uint4*>(dst_row + (((2 * q + 1) ^ sw) << 4)) = make_uint4(out[4], out[5], out[6], out[7]);
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float* v) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = s[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[8 * i + 2 * j] = f.x;
      v[8 * i + 2 * j + 1] = f.y;
    }
  }
}

// Tile t -> (m-block, n-block): m fastest, rotated so the walk starts at tp.m_rot.
// For a grouped GEMM the m-blocks of all groups are enumerated together
// (group-major), so m_blk indexes A rows directly.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int m_rot, int& m_blk, int& n_blk) {
  n_blk = tile / num_m;
  m_blk = tile - n_blk * num_m + m_rot;
  if (m_blk >= num_m) m_blk -= num_m;
}

// Grouped GEMM: is this m-block inside its group's valid rows? (always true otherwise)
__device__ __forceinline__ bool tile_live(const GemmArgs& p, int m_blk, int num_m_group, int& group) {
  if (!p.groups) {
    group = 0;
    return true;
  }
  group = m_blk / num_m_group;
  return (m_blk - group * num_m_group) * 128 < __ldg(p.group_count + group);
}

// Work distribution, identical in every role of a CTA. Data-parallel: CTA c takes tiles c, c + G,
// ... with their whole K range. Stream-K (p.streamk): the num_tiles x kbs (tile, k-block) units are
// cut into G equal contiguous ranges, one per CTA, so every SM streams the same number of weight
// bytes however few tiles there are; a tile cut between CTAs is summed in the fp32 workspace.
struct WorkIter {
  int cur, end, kbs;
  bool sk;
  __device__ WorkIter(const GemmArgs& p, int num_tiles, int kbs_) : kbs(kbs_), sk(p.streamk != 0) {
    if (sk) {
      const long long total = static_cast<long long>(num_tiles) * kbs;
      cur = static_cast<int>(blockIdx.x * total / gridDim.x);
      end = static_cast<int>((blockIdx.x + 1) * total / gridDim.x);
    } else {
      cur = blockIdx.x;
      end = num_tiles;
    }
  }
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (cur >= end) return false;
    if (sk) {
      tile = cur / kbs;
      kb0 = cur - tile * kbs;
      kb1 = min(kbs, end - tile * kbs);
      cur = tile * kbs + kb1;
    } else {
      tile = cur;
      kb0 = 0;
      kb1 = kbs;
      cur += gridDim.x;
    }
    return true;
  }
};

// Stream-K: the CTA whose range holds unit u (inverse of the range cut above).
__device__ __forceinline__ int sk_owner(long long u, long long total, int grid) {
  return static_cast<int>(((u + 1) * grid - 1) / total);
}

// Two-lane fp32 fused multiply-add (one f32x2 instruction).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T with e4m3 operands (both K-major, K = 32 per
// instruction, the same 32 bytes of a 128-byte swizzle row that one bf16 K = 16 step covers).
__device__ __forceinline__ void umma_e4m3(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Instruction descriptor: e4m3 x e4m3 -> fp32 (A and B format fields 0 = E4M3), both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// A8: W8A8 (fp8 A and B in shared memory, kind::f8f6f4, 128-deep k-blocks, scales applied per
// k-block by the epilogue warps); W8: W8A16 (fp8 B converted to bf16 in shared memory).
template <int BN, int STAGES, int EPI, bool W8 = false, bool A8 = false>
__global__ void __launch_bounds__(threads_of<W8, A8>(), 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs p) {
  using S = GemmSmem<BN, STAGES, W8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* land = empty + STAGES;  // W8: A + fp8 B landed (the converters then fill full[])
  uint64_t* tmem_full = land + STAGES;
  uint64_t* tmem_empty = tmem_full + 3;
  uint64_t* final_ready = tmem_empty + 3;  // W8A8: both column halves of the tile's sum are in TMEM
  uint64_t* final_free = final_ready + 1;  // W8A8: the epilogue has read the previous tile's sum
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_last = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_m_group = p.groups ? p.group_rows / kBM : num_m;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  // k-blocks: 64 bf16 or 128 e4m3, 128 bytes of a row either way
  const int num_kb_all = A8 ? (p.K + 127) / 128 : (p.K + kBK - 1) / kBK;
  // two accumulators (A8: three k-block partials and the final sum)
  constexpr int kAccCols = A8 ? 4 * BN : 2 * BN;
  constexpr uint32_t kTmemCols = (kAccCols <= 32) ? 32 : (kAccCols <= 64 ? 64 : (kAccCols <= 128 ? 128 : (kAccCols <= 256 ? 256 : 512)));

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], W8 ? 128 : 1);
      mbar_init(&empty[s], 1);
      mbar_init(&land[s], 1);
    }
    for (int a = 0; a < 3; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], A8 ? 256 : 128);
    }
    mbar_init(final_ready, 128);
    mbar_init(final_free, 128);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      // all-gather -> GEMM: A rows of a peer's shard are read only after its push landed
      const bool ag = p.tp.ag_cnt != nullptr;
      if (p.groups) fence_proxy_async_global();  // rows other GPUs stored (expert dispatch) before TMA reads
      const unsigned long long ag_target = ag ? (p.tp.ag_base ? *p.tp.ag_base : 0ull) + p.tp.ag_off : 0ull;
      uint32_t ready = 0;
      WorkIter it(p, num_tiles, num_kb_all);
      int tile, kb0, kb1;
      while (ok && it.next(tile, kb0, kb1)) {
        int m_blk, n_blk, grp;
        tile_coords(tile, num_m, p.tp.m_rot, m_blk, n_blk);
        if (!tile_live(p, m_blk, num_m_group, grp)) continue;
        if (ag) {
          const int r0 = m_blk * kBM;
          const int r1 = min(p.M, r0 + kBM) - 1;
          const int sh0 = p.tp.ag_all ? 0 : r0 / p.tp.rows_per_rank;
          const int sh1 = p.tp.ag_all ? p.tp.world - 1 : r1 / p.tp.rows_per_rank;
          for (int sh = sh0; sh <= sh1 && ok; ++sh) {
            if ((ready >> sh) & 1u) continue;
            ok = wait_counter(p.tp.ag_cnt + sh, ag_target, abort_flag, p.status);
            ready |= 1u << sh;
          }
          if (!ok) break;
          fence_proxy_async_global();  // peer stores (generic proxy) before this CTA's TMA reads
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          if constexpr (W8) {
            uint8_t* sb8 = sb + S::kBBytes;
            mbar_expect_tx(&land[stage], S::kABytes + S::kB8Bytes);
            tma_load_2d(sa, &tmA, &land[stage], kb * kBK, m_blk * kBM);
            tma_load_2d(sb8, &tmB, &land[stage], kb * kBK, grp * p.N + n_blk * BN);
          } else {
            const int kx = kb * (A8 ? 128 : kBK);  // element offset along K (bytes for e4m3)
            mbar_expect_tx(&full[stage], S::kStageBytes);
            tma_load_2d(sa, &tmA, &full[stage], kx, m_blk * kBM);
            tma_load_2d(sb, &tmB, &full[stage], kx, grp * p.N + n_blk * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain loads already in flight before the CTA's shared memory is released.
        for (int s = 0; s < STAGES; ++s) mbar_wait(W8 ? &land[s] : &full[s], 0, nullptr, nullptr, 50000000ull);
      }
    }
  } else if (A8 && warp == 1) {
    // ------------------------------------------------------------ MMA issuer (W8A8)
    // each k-block goes to its own TMEM partial (alternating two), handed to the epilogue warps
    if (lane == 0) {
      constexpr uint32_t idesc8 = umma_idesc_e4m3(kBM, BN);
      uint32_t stage = 0, phase = 0, g = 0;
      bool ok = true;
      WorkIter it(p, num_tiles, num_kb_all);
      int tile, kb0, kb1;
      while (ok && it.next(tile, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int b = g % 3;
          if (!mbar_wait(&tmem_empty[b], ((g / 3) & 1) ^ 1, abort_flag, p.status) ||
              !mbar_wait(&full[stage], phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint64_t ad = umma_desc_sw128(sa);
          const uint64_t bd = umma_desc_sw128(sa + S::kABytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)  // 32 e4m3 (32 bytes) along K per instruction
            umma_e4m3(tmem_base + b * BN, ad + 2 * k, bd + 2 * k, idesc8, k != 0);
          umma_commit(&empty[stage]);
          umma_commit(&tmem_full[b]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int t = 0;
      WorkIter it(p, num_tiles, num_kb_all);
      int tile, kb0, kb1;
      while (ok && it.next(tile, kb0, kb1)) {
        {
          int m_blk, n_blk, grp;
          tile_coords(tile, num_m, p.tp.m_rot, m_blk, n_blk);
          if (!tile_live(p, m_blk, num_m_group, grp)) continue;
        }
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
          const uint64_t ad = umma_desc_sw128(sa);
          const uint64_t bd = umma_desc_sw128(sb);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // advance 16 elements (32 bytes) along K inside the swizzle row
            umma_f16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb != kb0) || (k != 0));
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tmem_full[acc]);
        ++t;
      }
    }
  } else if (W8 && warp >= 6) {
    // ------------------------------------------------------------ fp8 -> bf16 converters (W8A16)
    const int ct = threadIdx.x - 192;  // 0..127: rows ct and ct + 128 of the B tile
    uint32_t stage = 0, phase = 0;
    WorkIter it(p, num_tiles, num_kb_all);
    int tile, kb0, kb1;
    while (it.next(tile, kb0, kb1)) {
      int m_blk, n_blk, grp;
      tile_coords(tile, num_m, p.tp.m_rot, m_blk, n_blk);
      if (!tile_live(p, m_blk, num_m_group, grp)) continue;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&land[stage], phase, abort_flag, p.status)) {
          ok = false;
          break;
        }
        uint8_t* sb = smem + stage * S::kStageBytes + S::kABytes;
        const uint8_t* sb8 = sb + S::kBBytes;
        for (int row = ct; row < BN; row += 128) {
          const int n = grp * p.N + n_blk * BN + row;
          const float sc = (n_blk * BN + row < p.N) ? __ldg(p.b_scale + static_cast<int64_t>(n >> 7) * p.b_scale_ld +
                                                            ((kb * kBK) >> 7))
                                                    : 0.f;
          convert_fp8_row(sb8 + row * kBK, sb + row * 128, row, sc);
        }
        fence_proxy_async_smem();  // generic stores -> visible to the tensor core's operand reads
        mbar_arrive(&full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int t = 0;
    WorkIter it(p, num_tiles, num_kb_all);
    int tile, kb0, kb1;
    // the fused epilogue of one tile whose fp32 accumulator sits at `tbase` in tensor memory
    auto tile_epilogue = [&](uint32_t tbase, int n_blk, int row, bool row_ok) {
        if constexpr (EPI == kEpiStoreBf16 || EPI == kEpiResidual || EPI == kEpiStoreF32) {
  #pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tbase + c * 32, r);
            tmem_ld_wait();
            const int col0 = n_blk * BN + c * 32;
            if (row_ok && col0 < p.N) {
              float v[32];
  #pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
              if constexpr (EPI == kEpiStoreF32) {
                float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) + row * p.ldc + col0);
  #pragma unroll
                for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
              } else {
                if constexpr (EPI == kEpiResidual) {
                  float rv[32];
                  load_bf16x32(p.R + row * p.ldr + col0, rv);
  #pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] += rv[j];
                }
                store_bf16x32(reinterpret_cast<__nv_bfloat16*>(p.C) + row * p.ldc + col0, v);
              }
            }
          }
        } else if constexpr (EPI == kEpiRSPush) {
          // partial sums of this rank's K-slice go straight to the row's owner (P2P stores over NVLink)
          __nv_bfloat16* dst_row = nullptr;
          if (row_ok) {
            const int d = row / p.tp.rows_per_rank;
            const int lr = row - d * p.tp.rows_per_rank;
            dst_row = p.tp.rs_recv[d] + (static_cast<int64_t>(p.tp.rank) * p.tp.rows_per_rank + lr) * p.ldc;
          }
  #pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tbase + c * 32, r);
            tmem_ld_wait();
            const int col0 = n_blk * BN + c * 32;
            if (row_ok && col0 < p.N) {
              float v[32];
  #pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
              store_bf16x32(dst_row + col0, v);
            }
          }
        } else if constexpr (EPI == kEpiScatter) {
          // indirect row store: the token slot this gathered row came from (local or a peer's buffer)
          __nv_bfloat16* dst_row = nullptr;
          if (row_ok) {
            const int slot = p.row_slot[row];
            if (slot >= 0) dst_row = p.tp.rs_recv[p.row_rank ? p.row_rank[row] : 0] + static_cast<int64_t>(slot) * p.ldc;
          }
  #pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tbase + c * 32, r);
            tmem_ld_wait();
            const int col0 = n_blk * BN + c * 32;
            if (dst_row && col0 < p.N) {
              float v[32];
  #pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
              store_bf16x32(dst_row + col0, v);
            }
          }
        } else if constexpr (EPI == kEpiSwiGLU) {
          constexpr int H = BN / 2;
  #pragma unroll 1
          for (int c = 0; c < H / 32; ++c) {
            uint32_t g[32], u[32];
            tmem_ld32(tbase + c * 32, g);
            tmem_ld32(tbase + H + c * 32, u);
            tmem_ld_wait();
            const int col0 = n_blk * H + c * 32;
            if (row_ok) {
              float v[32];
  #pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
              store_bf16x32(reinterpret_cast<__nv_bfloat16*>(p.C) + row * p.ldc + col0, v);
            }
          }
        } else if constexpr (EPI == kEpiQKV) {
          static_assert(BN == 128, "QKV epilogue maps one 128-wide head per tile");
          qkv_head_epilogue(p, tbase, n_blk, row, row_ok);
        } else if constexpr (EPI == kEpiArgmax) {
          unsigned long long best = 0ull;
  #pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tbase + c * 32, r);
            tmem_ld_wait();
            const int col0 = n_blk * BN + c * 32;
            if (row_ok && col0 < p.N) {
              uint32_t allow = 0xFFFFFFFFu;
              if (p.bitmask) allow = p.bitmask[static_cast<int64_t>(row) * p.bitmask_words + (col0 >> 5)];
  #pragma unroll
              for (int j = 0; j < 32; ++j) {
                if ((allow >> j) & 1u) {
                  const unsigned long long key =
                      (static_cast<unsigned long long>(float_order_key(__uint_as_float(r[j]))) << 32) |
                      static_cast<unsigned long long>(0xFFFFFFFFu -
                                                      static_cast<uint32_t>(col0 + j + p.tp.col_offset));
                  best = key > best ? key : best;
                }
              }
            }
          }
          if (row_ok && best) atomicMax(p.amax + row, best);
        }
    };
    if constexpr (A8) {
      // W8A8: one 128-deep k-block per TMEM partial (three, rotating with the MMA issuer). Warps 2-9
      // promote: warp pair (w, w + 4) shares a TMEM lane quarter, each summing 64 columns of its 32
      // rows as partial x (activation scale x weight block scale) in fp32 registers. At the tile's
      // end both halves go to the fourth TMEM region, which warps 2-5 read like any accumulator
      // in the shared epilogue (final_ready / final_free hand the region over, with bounded waits).
      static_assert(!A8 || BN == 128, "W8A8 tiles are one weight scale block wide");
      const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
      const int hc = (warp - 2) >> 2;  // column half of this warp
      const uint32_t fb = tmem_base + 3 * BN + lane_off;
      uint32_t g = 0, tt = 0;
      while (it.next(tile, kb0, kb1)) {
        int m_blk, n_blk;
        tile_coords(tile, num_m, p.tp.m_rot, m_blk, n_blk);
        const int row = m_blk * kBM + row_in_tile;
        const bool row_ok = row < p.M;
        const float* sa_row = p.a_scale + static_cast<int64_t>(row_ok ? row : 0) * p.a_scale_ld;
        const float* sb_row = p.b_scale + static_cast<int64_t>(n_blk) * p.b_scale_ld;
        float2 sum[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) sum[i] = make_float2(0.f, 0.f);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int b = g % 3;
          if (!mbar_wait(&tmem_full[b], (g / 3) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float sc = (row_ok ? __ldg(sa_row + kb) : 0.f) * __ldg(sb_row + kb);
          const uint32_t pb = tmem_base + b * BN + lane_off + hc * 64;
          uint32_t r0[32], r1[32];
          tmem_ld32(pb, r0);
          tmem_ld32(pb + 32, r1);
          tmem_ld_wait();
          tc_fence_before();
          mbar_arrive(&tmem_empty[b]);  // the partial is in registers: the MMA may overwrite it
          const float2 s2 = make_float2(sc, sc);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            sum[j] = ffma2(make_float2(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1])), s2, sum[j]);
            sum[16 + j] = ffma2(make_float2(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1])), s2,
                                sum[16 + j]);
          }
        }
        if (!ok) break;
        // warps 6-9 write their half only after warps 2-5 have read the previous tile's sum
        if (hc == 1 && tt > 0 && !mbar_wait(final_free, (tt - 1) & 1, abort_flag, p.status)) break;
        tc_fence_after();
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            r[2 * j] = __float_as_uint(sum[16 * c + j].x);
            r[2 * j + 1] = __float_as_uint(sum[16 * c + j].y);
          }
          tmem_st32(fb + hc * 64 + c * 32, r);
        }
        tmem_st_wait();
        tc_fence_before();
        if (hc == 1) {
          mbar_arrive(final_ready);
        } else {
          if (!mbar_wait(final_ready, tt & 1, abort_flag, p.status)) break;  // the other half is in
          tc_fence_after();
          tile_epilogue(fb, n_blk, row, row_ok);
          tc_fence_before();
          mbar_arrive(final_free);
        }
        ++tt;
      }
    } else {
      while (it.next(tile, kb0, kb1)) {
        int m_blk, n_blk, grp;
        tile_coords(tile, num_m, p.tp.m_rot, m_blk, n_blk);
        if (!tile_live(p, m_blk, num_m_group, grp)) continue;
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        ++t;
        if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t tbase = tmem_base + acc * BN + (static_cast<uint32_t>(q * 32) << 16);
        const int row = m_blk * kBM + row_in_tile;
        const bool row_ok = row < p.M && (!p.groups || row - grp * p.group_rows < __ldg(p.group_count + grp));

        if (p.streamk && (kb0 != 0 || kb1 != num_kb_all)) {
          // Stream-K: this CTA holds part of the tile's K range. Add it into the tile's workspace
          // slot (named by the tile's last contributor, unique per cut tile); the last contributor
          // to arrive loads the full sum back into its accumulator and runs the epilogue below.
          const long long total = static_cast<long long>(num_tiles) * num_kb_all;
          const long long u_first = static_cast<long long>(tile) * num_kb_all;
          const int first = sk_owner(u_first, total, gridDim.x);
          const int slot = sk_owner(u_first + num_kb_all - 1, total, gridDim.x);
          float* wrow = p.split_ws + (static_cast<int64_t>(slot) * kBM + row_in_tile) * BN;
  #pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tbase + c * 32, r);
            tmem_ld_wait();
            if (row_ok) {
  #pragma unroll
              for (int i = 0; i < 8; ++i)
                asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(wrow + c * 32 + 4 * i),
                             "f"(__uint_as_float(r[4 * i])), "f"(__uint_as_float(r[4 * i + 1])),
                             "f"(__uint_as_float(r[4 * i + 2])), "f"(__uint_as_float(r[4 * i + 3]))
                             : "memory");
            }
          }
          __threadfence();
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (warp == 2 && lane == 0) *split_last = atomicAdd(p.split_cnt + slot, 1) == slot - first;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (!*split_last) {
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
            continue;
          }
          __threadfence();
          // tcgen05.st is warp-aligned: every lane issues it (rows past M store zeros)
  #pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            float4* src = reinterpret_cast<float4*>(wrow + c * 32);
  #pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
              if (row_ok) {
                f = __ldcg(src + i);
                __stcg(src + i, make_float4(0.f, 0.f, 0.f, 0.f));
              }
              r[4 * i] = __float_as_uint(f.x);
              r[4 * i + 1] = __float_as_uint(f.y);
              r[4 * i + 2] = __float_as_uint(f.z);
              r[4 * i + 3] = __float_as_uint(f.w);
            }
            tmem_st32(tbase + c * 32, r);
          }
          tmem_st_wait();
          if (warp == 2 && lane == 0) p.split_cnt[slot] = 0;
        }
        tile_epilogue(tbase, n_blk, row, row_ok);
        tc_fence_before();
        mbar_arrive(&tmem_empty[acc]);
      }
    }
    // Cross-GPU signal: this CTA's stores are visible system-wide before the counters move.
    // (every epilogue thread reaches the named barrier; only a CTA that did not abort signals)
    if (p.tp.rs_cnt[0] || p.tp.done_cnt[0]) {
      __threadfence_system();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0 && !*abort_flag) {
        for (int d = 0; d < p.tp.world; ++d) {
          if (p.tp.rs_cnt[d]) red_add_release_sys(p.tp.rs_cnt[d] + p.tp.rank, 1ull);
          if (p.tp.done_cnt[d]) red_add_release_sys(p.tp.done_cnt[d] + p.tp.rank, 1ull);
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

int grid_for(int M, int N, int BN, int max_ctas) {
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  int grid = max_ctas > 0 ? max_ctas : num_sms();
  return grid > tiles ? tiles : grid;
}

template <int BN, int STAGES, int EPI, bool W8 = false>
int launch(const GemmArgs& a, cudaStream_t stream) {
  using S = GemmSmem<BN, STAGES, W8>;
  static_assert(S::kAlloc <= 227 * 1024, "shared memory");
  CUtensorMap ma, mb;
  if (!make_bf16_map(&ma, a.A, a.M, a.K, a.lda, kBM)) return -10;
  const int64_t brows = static_cast<int64_t>(a.N) * (a.groups ? a.groups : 1);
  if constexpr (W8) {
    if (!make_u8_map(&mb, a.B8, brows, a.K, a.ldb8, BN, kBK)) return -11;
  } else {
    if (!make_bf16_map(&mb, a.B, brows, a.K, a.ldb, BN)) return -11;
  }
  auto kern = gemm_bf16_kernel<BN, STAGES, EPI, W8>;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(kern), S::kAlloc)) return e;
  int grid = grid_for(a.M, a.N, BN, a.max_ctas);
  if (a.streamk) grid = a.streamk;  // the dispatcher's stream-K grid
  kern<<<grid, threads_of<W8>(), S::kAlloc, stream>>>(ma, mb, a);
  return cudaGetLastError();
}

// W8A8 launch: e4m3 A (quantised activations) and B (weights), 128 x 128 tiles (one weight scale
// block per tile), six 32 KB stages.
template <int EPI>
int launch_a8(const GemmArgs& a, cudaStream_t stream) {
  using S = GemmSmem<128, 6>;
  CUtensorMap ma, mb;
  if (!make_fp8_sw128_map(&ma, a.A8, a.M, a.K, a.lda8, kBM)) return -10;
  if (!make_fp8_sw128_map(&mb, a.B8, a.N, a.K, a.ldb8, 128)) return -11;
  auto kern = gemm_bf16_kernel<128, 6, EPI, false, true>;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(kern), S::kAlloc)) return e;
  kern<<<grid_for(a.M, a.N, 128, 0), threads_of<false, true>(), S::kAlloc, stream>>>(ma, mb, a);
  return cudaGetLastError();
}

// Block-scaled e4m3 quantisation: one warp per (row, 128-column block), four values per lane.
__global__ void __launch_bounds__(256) quantize_fp8_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                 int M, int kblocks, uint8_t* __restrict__ q,
                                                                 int64_t ldq, float* __restrict__ s, int s_ld) {
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= M * kblocks) return;
  const int m = w / kblocks, kb = w - m * kblocks;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + static_cast<int64_t>(m) * ldx + kb * 128 + lane * 4);
  const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  float amax = fmaxf(fmaxf(fabsf(v01.x), fabsf(v01.y)), fmaxf(fabsf(v23.x), fabsf(v23.y)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / scale;
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v01.x * inv, v01.y * inv), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v23.x * inv, v23.y * inv), __NV_SATFINITE, __NV_E4M3);
  *reinterpret_cast<uint32_t*>(q + static_cast<int64_t>(m) * ldq + kb * 128 + lane * 4) =
      static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  if (lane == 0) s[static_cast<int64_t>(m) * s_ld + kb] = scale;
}

// Tile width: 256 keeps the tensor cores busiest, but a small M (decode batches) leaves most SMs
// idle with 128x256 tiles, so epilogues that do not depend on the tile width step down to 128
// columns when 256-wide tiles would cover less than ~3/4 of the SMs. SwiGLU (256-row gate/up interleave),
// QKV (one 128-wide head per tile), argmax and grouped GEMMs keep their widths.
int bn_for(int M, int N, int epi, bool grouped) {
  if (epi == kEpiQKV) return 128;
  // (scatter runs only inside grouped GEMMs: the host sizes its counter waits with gemm_grid)
  if (epi == kEpiSwiGLU || epi == kEpiArgmax || epi == kEpiScatter || grouped) return 256;
  const int target = (num_sms() * 3) / 4;
  const int mb = (M + kBM - 1) / kBM;
  // (64-wide tiles measured slower than 128 at M=256: the K loop per CTA is latency-bound either way)
  return mb * ((N + 255) / 256) >= target ? 256 : 128;
}

template <int EPI>
int launch_bn(const GemmArgs& a, cudaStream_t stream) {
  switch (bn_for(a.M, a.N, EPI, a.groups != 0)) {
    case 128:
      return launch<128, 6, EPI>(a, stream);
    default:
      return launch<256, 4, EPI>(a, stream);
  }
}

}  // namespace

static int g_pair_mode = 0;

// The two-SM kernel takes large plain / residual / SwiGLU / fp32 GEMMs, including the
// tensor-parallel all-gather GEMMs and the reduce-scatter push GEMM, and the QKV GEMM when its
// heads pair up into 256-wide tiles (LAKEB_GEMM_PAIR=2 keeps QKV on the single-SM kernel);
// argmax, grouped and fp8 GEMMs stay on the single-SM kernel.
static bool use_pair(int M, int N, int epi, bool grouped, int max_ctas, bool done_signal) {
  if (!g_pair_mode || M < 512 || grouped || max_ctas != 0 || done_signal) return false;
  if (epi == kEpiQKV) return g_pair_mode == 1 && N % 256 == 0;
  return epi == kEpiStoreBf16 || epi == kEpiResidual || epi == kEpiSwiGLU || epi == kEpiStoreF32 ||
         epi == kEpiRSPush;
}

// Per-device stream-K workspace: fp32 partial tiles (zero between uses: the finishing CTA zeroes
// what it read), one slot of 128 x 256 floats per CTA, and one arrival counter per slot. It is
// allocated outside any graph capture (gemm_workspace_init, or the first eager GEMM on the
// device); until it exists every GEMM runs data-parallel, and gemm_grid() plans the same way.
constexpr int kSkMaxSlots = 1024;
constexpr int64_t kSkWsFloats = static_cast<int64_t>(kSkMaxSlots) * 128 * 256;
static float* s_sk_ws[16] = {};
static int* s_sk_cnt[16] = {};

static int cur_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return -1;
  return dev;
}

bool gemm_workspace_init() {
  const int dev = cur_device();
  if (dev < 0) return false;
  if (s_sk_ws[dev]) return true;
  void* w = nullptr;
  void* c = nullptr;
  if (cudaMalloc(&w, kSkWsFloats * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cudaMalloc(&c, kSkMaxSlots * sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w);
    return false;
  }
  cudaMemset(w, 0, kSkWsFloats * sizeof(float));
  cudaMemset(c, 0, kSkMaxSlots * sizeof(int));
  cudaDeviceSynchronize();
  s_sk_ws[dev] = static_cast<float*>(w);
  s_sk_cnt[dev] = static_cast<int*>(c);
  return true;
}

static bool sk_workspace(float** ws, int** cnt) {
  const int dev = cur_device();
  if (dev < 0 || !s_sk_ws[dev]) return false;
  *ws = s_sk_ws[dev];
  *cnt = s_sk_cnt[dev];
  return true;
}

// Stream-K grid for a tiles x kbs problem, or 0 for data-parallel. A cut tile costs its CTAs an
// fp32 partial (red.add) and its finisher a reload before the epilogue, which only pays when the
// busiest CTA streams at most half the k-blocks it would with whole tiles: decode-size QKV,
// o_proj and down (32-48 tiles on 148 SMs). Measured on B200 at M = 80: gate_up (112 tiles, every
// tile cut in two) was 1.6x slower under stream-K than whole tiles. At least 4 k-blocks per CTA.
static int streamk_grid(int tiles, int kbs) {
  const int sms = num_sms();
  const long long total = static_cast<long long>(tiles) * kbs;
  const long long dp = static_cast<long long>((tiles + sms - 1) / sms) * kbs;
  int g = sms < kSkMaxSlots ? sms : kSkMaxSlots;
  if (total < 4LL * g) g = static_cast<int>(total / 4);
  if (g < 2) return 0;
  const long long sk = (total + g - 1) / g;
  return sk * 2 <= dp ? g : 0;
}

static bool sk_epilogue(int epi) {
  return epi == kEpiStoreBf16 || epi == kEpiResidual || epi == kEpiStoreF32 || epi == kEpiSwiGLU ||
         epi == kEpiQKV || epi == kEpiArgmax || epi == kEpiRSPush;
}

static int tile_width(int M, int N, int epi, bool w8) {
  // fp8 SwiGLU weights interleave gate and up per 128 rows ([gate 64 | up 64]): 128-wide tiles
  if (w8) return (epi == kEpiQKV || epi == kEpiSwiGLU) ? 128 : 256;
  return bn_for(M, N, epi, false);
}

static int g_streamk_mode = 1;
void set_gemm_streamk_mode(int mode) { g_streamk_mode = mode; }

// Stream-K grid this call will use (0 = data-parallel).
static int plan_streamk(int M, int N, int K, int epi, bool grouped, int max_ctas, bool w8) {
  if (!g_streamk_mode || grouped || max_ctas > 0 || !sk_epilogue(epi)) return 0;
  float* ws;
  int* cnt;
  if (!sk_workspace(&ws, &cnt)) return 0;
  const int bn = tile_width(M, N, epi, w8);
  const int tiles = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  return streamk_grid(tiles, (K + kBK - 1) / kBK);
}

int gemm_grid(int M, int N, int K, int epi, int max_ctas, bool w8) {
  if (!w8 && use_pair(M, N, epi, false, max_ctas, false)) return gemm_pair_grid(M, N);
  const int g = plan_streamk(M, N, K, epi, false, max_ctas, w8);
  if (g) return g;
  return grid_for(M, N, tile_width(M, N, epi, w8), max_ctas);
}

void set_gemm_pair_mode(int mode) { g_pair_mode = mode; }
int gemm_pair_mode() { return g_pair_mode; }

// W8A8 activation workspace per device: e4m3 rows [M x K] and their scales [M x K/128], reserved
// outside any graph capture (gemm_w8a8_reserve); a GEMM that does not fit runs as W8A16. Every
// W8A8 GEMM of a device quantises into the same buffer, so W8A8 GEMMs run on one stream at a time
// (as the engine issues them); two streams issuing them concurrently would overwrite each other's
// activations.
static int g_w8a8_min_m = 256;
void set_gemm_w8a8_min_m(int m) { g_w8a8_min_m = m; }
static uint8_t* s_a8_q[16] = {};
static float* s_a8_s[16] = {};
static int64_t s_a8_cap[16] = {};  // elements of s_a8_q

bool gemm_w8a8_reserve(int64_t M, int64_t K) {
  const int dev = cur_device();
  if (dev < 0 || M <= 0 || K <= 0) return false;
  const int64_t need = M * ((K + 127) / 128 * 128);
  if (s_a8_cap[dev] >= need) return true;
  uint8_t* q = nullptr;
  float* sc = nullptr;
  if (cudaMalloc(&q, need) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cudaMalloc(&sc, need / 128 * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(q);
    return false;
  }
  cudaDeviceSynchronize();  // the previous buffers may still be read by queued kernels
  cudaFree(s_a8_q[dev]);
  cudaFree(s_a8_s[dev]);
  s_a8_q[dev] = q;
  s_a8_s[dev] = sc;
  s_a8_cap[dev] = need;
  return true;
}

static bool a8_workspace(int64_t elems, uint8_t** q, float** sc) {
  const int dev = cur_device();
  if (dev < 0 || s_a8_cap[dev] < elems) return false;
  *q = s_a8_q[dev];
  *sc = s_a8_s[dev];
  return true;
}

// W8A8 takes plain single-GPU fp8 GEMMs at prefill sizes; tensor-parallel (peer-signalling or
// peer-waiting), grouped and CTA-capped calls stay W8A16.
static bool a8_eligible(const GemmArgs& a, int epi) {
  if (g_w8a8_min_m <= 0 || a.M < g_w8a8_min_m || a.groups || a.max_ctas || !a.A || !a.b_scale) return false;
  if (a.tp.ag_cnt || a.tp.rs_cnt[0] || a.tp.done_cnt[0] || a.K % 128 || a.lda % 8 || a.ldb8 % 16) return false;
  if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B8) & 15)) return false;
  return epi == kEpiStoreBf16 || epi == kEpiResidual || epi == kEpiSwiGLU || epi == kEpiStoreF32 ||
         epi == kEpiQKV || epi == kEpiArgmax;
}

int quantize_fp8_rows(const __nv_bfloat16* x, int64_t ldx, int M, int K, uint8_t* q, int64_t ldq, float* s,
                      int s_ld, cudaStream_t stream) {
  if (M <= 0) return 0;
  if (K % 128 || ldx % 4 || ldq % 4 || (reinterpret_cast<uintptr_t>(x) & 7) || (reinterpret_cast<uintptr_t>(q) & 3))
    return -12;
  const int64_t warps = static_cast<int64_t>(M) * (K / 128);
  quantize_fp8_rows_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(x, ldx, M, K / 128, q, ldq, s,
                                                                                       s_ld);
  return cudaGetLastError();
}

int gemm_bf16(const GemmArgs& a_in, int epi, cudaStream_t stream) {
  if (a_in.M <= 0 || a_in.N <= 0 || a_in.K <= 0) return 0;
  GemmArgs a = a_in;
  {
    // first eager GEMM on a device allocates the stream-K workspace (never inside a capture)
    const int dev = cur_device();
    if (dev >= 0 && !s_sk_ws[dev]) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone)
        gemm_workspace_init();
      cudaGetLastError();
    }
  }
  if (epi == kEpiRSPush && (a.tp.world < 1 || a.tp.world > kMaxTP || a.tp.rows_per_rank <= 0 ||
                            a.M != a.tp.world * a.tp.rows_per_rank))
    return -5;
  if (a.tp.ag_cnt && !a.tp.ag_all && (a.tp.rows_per_rank <= 0 || a.M > a.tp.world * a.tp.rows_per_rank)) return -6;
  if (a.tp.ag_cnt && (a.tp.world < 1 || a.tp.world > kMaxTP)) return -6;
  if (epi == kEpiQKV && a.N != (a.n_q_heads + 2 * a.n_kv_heads) * 128) return -3;
  const bool w8 = a.B8 != nullptr;
  if (w8 && a8_eligible(a, epi)) {
    // W8A8: quantise this call's activations into the device workspace, then the fp8 MMA kernel
    uint8_t* q = nullptr;
    float* sc = nullptr;
    if (a8_workspace(static_cast<int64_t>(a.M) * a.K, &q, &sc)) {
      const int kbs = a.K / 128;
      if (int e = quantize_fp8_rows(a.A, a.lda, a.M, a.K, q, a.K, sc, kbs, stream)) return e;
      a.A8 = q;
      a.lda8 = a.K;
      a.a_scale = sc;
      a.a_scale_ld = kbs;
      switch (epi) {
        case kEpiStoreBf16: return launch_a8<kEpiStoreBf16>(a, stream);
        case kEpiResidual: return launch_a8<kEpiResidual>(a, stream);
        case kEpiSwiGLU: return launch_a8<kEpiSwiGLU>(a, stream);
        case kEpiStoreF32: return launch_a8<kEpiStoreF32>(a, stream);
        case kEpiQKV: return launch_a8<kEpiQKV>(a, stream);
        case kEpiArgmax: return launch_a8<kEpiArgmax>(a, stream);
        default: break;
      }
    }
  }
  // plan order shared with gemm_grid(): two-SM kernel, else stream-K, else data-parallel
  if (!w8 && use_pair(a.M, a.N, epi, a.groups != 0, a.max_ctas, a.tp.done_cnt[0] != nullptr))
    return gemm_bf16_pair(a, epi, stream);
  a.streamk = plan_streamk(a.M, a.N, a.K, epi, a.groups != 0, a.max_ctas, w8);
  if (a.streamk) sk_workspace(&a.split_ws, &a.split_cnt);
  if (w8) {  // fp8 weights: converter-warp kernel (no two-SM variant)
    if (!a.b_scale || a.b_scale_ld <= 0 || (a.K % 64) || (a.ldb8 % 16) ||
        (reinterpret_cast<uintptr_t>(a.B8) & 15) || (reinterpret_cast<uintptr_t>(a.A) & 15))
      return -9;
    switch (epi) {
      case kEpiStoreBf16: return launch<256, 3, kEpiStoreBf16, true>(a, stream);
      case kEpiResidual: return launch<256, 3, kEpiResidual, true>(a, stream);
      case kEpiSwiGLU: return launch<128, 5, kEpiSwiGLU, true>(a, stream);
      case kEpiStoreF32: return launch<256, 3, kEpiStoreF32, true>(a, stream);
      case kEpiArgmax: return launch<256, 3, kEpiArgmax, true>(a, stream);
      case kEpiQKV: return launch<128, 5, kEpiQKV, true>(a, stream);
      case kEpiRSPush: return launch<256, 3, kEpiRSPush, true>(a, stream);
      default:
        return -4;
    }
  }
  if (a.groups && (a.group_rows % kBM || !a.group_count || a.M != a.groups * a.group_rows)) return -8;
  if ((a.K % 8) || (a.lda % 8) || (a.ldb % 8) || (a.N % 32)) return -1;
  if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15)) return -2;
  switch (epi) {
    case kEpiStoreBf16:
      return launch_bn<kEpiStoreBf16>(a, stream);
    case kEpiResidual:
      return launch_bn<kEpiResidual>(a, stream);
    case kEpiSwiGLU:
      return launch<256, 4, kEpiSwiGLU>(a, stream);
    case kEpiQKV:
      return launch<128, 6, kEpiQKV>(a, stream);
    case kEpiArgmax:
      return launch<256, 4, kEpiArgmax>(a, stream);
    case kEpiStoreF32:
      return launch_bn<kEpiStoreF32>(a, stream);
    case kEpiScatter:
      if (!a.row_slot || !a.tp.rs_recv[0]) return -7;
      return launch<256, 4, kEpiScatter>(a, stream);
    case kEpiRSPush:
      return launch_bn<kEpiRSPush>(a, stream);
    default:
      return -4;
  }
}

}  // namespace lakeb
