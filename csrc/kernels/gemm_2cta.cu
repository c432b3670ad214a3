// Two-SM tcgen05 GEMM for large M (prefill-sized projections) on sm_100a.
//
// A cluster of two CTAs (one per SM) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2: each CTA stages its own 128 rows of A and its own
// 128 rows (output columns) of B per K step, so a stage is 32 KB per CTA
// instead of 48 KB and six stages fit, and each MMA instruction does twice the
// work of the single-SM 128 x 256 form. The even CTA of the pair issues the
// MMAs into both CTAs' tensor memory (each holds 128 accumulator rows).
//
//   warp 0     : TMA producer of this CTA's own halves (each CTA loads only what it
//                stages; the pair's loads complete on the even CTA's full barrier)
//   warp 1     : TMEM allocation (both CTAs); MMA issue + commits (even CTA)
//   warps 2..5 : epilogue of this CTA's 128 rows (store / residual / SwiGLU / fp32 /
//                tensor-parallel reduce-scatter push to the row owner's buffer / QKV with
//                RoPE and the paged K/V stores, two heads per tile)
//
// Tensor-parallel variants: with tp.ag_cnt set the producer waits, per 128-row
// half, for the all-gather counters of the row shards it reads; with
// tp.rs_cnt set every CTA bumps each owner's counter once its pushes are
// visible (one count per CTA, gemm_pair_grid() of them per launch).
//
// Barriers: full[s] on the even CTA expects both CTAs' bytes; empty[s] and
// tmem_full[a] live in both CTAs and receive one commit from the MMA issuer
// each; tmem_empty[a] on the even CTA counts both CTAs' 256 epilogue threads.
// Every wait is bounded (2 s) and reports through the status word.
#include "common.cuh"
#include "lakeb_kernels.h"
#include "qkv_epilogue.cuh"
#include "tma_host.h"

namespace lakeb {
namespace {

constexpr int kBM2 = 128;     // rows per CTA (256 per pair)
constexpr int kBN2 = 256;     // output columns per pair tile (128 per CTA stage)
constexpr int kBK2 = 64;
constexpr int kStages2 = 6;
constexpr int kThreads2 = 192;
constexpr int kStageBytes2 = kBM2 * kBK2 * 2 + (kBN2 / 2) * kBK2 * 2;  // 32 KB
constexpr int kStageOutOff2 = kStages2 * kStageBytes2;  // 4 epilogue warps x 2 KB: coalesced peer stores
constexpr int kBarOff2 = kStageOutOff2 + 4 * 2048;
constexpr int kSmem2 = kBarOff2 + (2 * kStages2 + 4) * 8 + 16 + 1024;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory completing on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive (once every prior MMA of the pair completed) on an mbarrier given by its cluster address.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// Pair tile t -> (256-row m-block, n-block), m fastest; tp.m_rot is in 128-row units.
__device__ __forceinline__ void pair_tile(int tile, int num_m, int m_rot128, int& m_blk, int& n_blk) {
  n_blk = tile / num_m;
  m_blk = tile - n_blk * num_m + m_rot128 / 2;
  if (m_blk >= num_m) m_blk -= num_m;
}

__device__ __forceinline__ void store32_bf16(__nv_bfloat16* dst, const float* v) {
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
__device__ __forceinline__ void load32_bf16(const __nv_bfloat16* src, float* v) {
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

template <int EPI>
__global__ void __launch_bounds__(kThreads2, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff2);
  uint64_t* empty = full + kStages2;
  uint64_t* tmem_full = empty + kStages2;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t crank = cluster_rank();
  const bool leader = crank == 0;
  const int pair = blockIdx.x / 2;
  const int npairs = gridDim.x / 2;
  const int num_m = (p.M + 2 * kBM2 - 1) / (2 * kBM2);
  const int num_n = (p.N + kBN2 - 1) / kBN2;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + kBK2 - 1) / kBK2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_leader0 = map_to_rank(&full[0], 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      // all-gather -> GEMM: this CTA's A rows of a peer's shard are read only after its push landed
      const bool ag = p.tp.ag_cnt != nullptr;
      const unsigned long long ag_target = ag ? (p.tp.ag_base ? *p.tp.ag_base : 0ull) + p.tp.ag_off : 0ull;
      uint32_t ready = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int m_blk, n_blk;
        pair_tile(tile, num_m, p.tp.m_rot, m_blk, n_blk);
        if (ag) {
          const int r0 = m_blk * 2 * kBM2 + crank * kBM2;
          const int r1 = min(p.M, r0 + kBM2) - 1;
          const int sh0 = p.tp.ag_all ? 0 : r0 / p.tp.rows_per_rank;
          const int sh1 = p.tp.ag_all ? p.tp.world - 1 : (r0 <= r1 ? r1 / p.tp.rows_per_rank : -1);
          for (int sh = sh0; sh <= sh1 && ok; ++sh) {
            if ((ready >> sh) & 1u) continue;
            ok = wait_counter(p.tp.ag_cnt + sh, ag_target, abort_flag, p.status);
            ready |= 1u << sh;
          }
          if (!ok) break;
          fence_proxy_async_global();
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * kStageBytes2;
          uint8_t* sb = sa + kBM2 * kBK2 * 2;
          if (leader) mbar_expect_tx(&full[stage], 2 * kStageBytes2);
          const uint32_t bar = full_leader0 + stage * 8;
          tma_load_2d_pair(sa, &tmA, bar, kb * kBK2, m_blk * 2 * kBM2 + crank * kBM2);
          tma_load_2d_pair(sb, &tmB, bar, kb * kBK2, n_blk * kBN2 + crank * (kBN2 / 2));
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * kBM2, kBN2);
      const uint32_t empty_peer0 = map_to_rank(&empty[0], 1);
      const uint32_t tfull_peer0 = map_to_rank(&tmem_full[0], 1);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int t = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++t) {
        const int acc = t & 1;
        if (!mbar_wait(&tmem_empty[acc], ((t >> 1) & 1) ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN2;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes2);
          const uint32_t sb = sa + kBM2 * kBK2 * 2;
          const uint64_t ad = umma_desc_sw128(sa);
          const uint64_t bd = umma_desc_sw128(sb);
#pragma unroll
          for (int k = 0; k < kBK2 / 16; ++k) umma_f16_pair(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair(smem_u32(&empty[stage]));     // this CTA's stage is free
          umma_commit_pair(empty_peer0 + stage * 8);     // and the peer's
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit_pair(smem_u32(&tmem_full[acc]));
        umma_commit_pair(tfull_peer0 + acc * 8);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const uint32_t tempty_leader0 = map_to_rank(&tmem_empty[0], 0);
    int t = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++t) {
      int m_blk, n_blk;
      pair_tile(tile, num_m, p.tp.m_rot, m_blk, n_blk);
      const int acc = t & 1;
      if (!mbar_wait(&tmem_full[acc], (t >> 1) & 1, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + acc * kBN2 + (static_cast<uint32_t>(q * 32) << 16);
      const int row = m_blk * 2 * kBM2 + crank * kBM2 + row_in_tile;
      const bool row_ok = row < p.M;
      if constexpr (EPI == kEpiQKV) {
        // this CTA's 256 accumulator columns are two whole heads (RoPE, K/V to the arena(s))
        uint4* stage = reinterpret_cast<uint4*>(smem + kStageOutOff2 + q * 2048);
        qkv_head_epilogue(p, tbase, 2 * n_blk, row, row_ok, stage);
        qkv_head_epilogue(p, tbase + 128, 2 * n_blk + 1, row, row_ok, stage);
      } else if constexpr (EPI == kEpiRSPush) {
        // partial rows of this rank's K-slice go straight to the row's owner (P2P stores over
        // NVLink), staged per warp so each store instruction writes 8 rows x 64 contiguous bytes
        __nv_bfloat16* dst_row = nullptr;
        if (row_ok) {
          const int d = row / p.tp.rows_per_rank;
          const int lr = row - d * p.tp.rows_per_rank;
          dst_row = p.tp.rs_recv[d] + (static_cast<int64_t>(p.tp.rank) * p.tp.rows_per_rank + lr) * p.ldc;
        }
        uint4* stage = reinterpret_cast<uint4*>(smem + kStageOutOff2 + q * 2048);
#pragma unroll 1
        for (int c = 0; c < kBN2 / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
          const int col0 = n_blk * kBN2 + c * 32;
          if (col0 < p.N) {  // warp-uniform
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            warp_store_rows64(stage, dst_row ? dst_row + col0 : nullptr, v, lane);
          }
        }
      } else if constexpr (EPI == kEpiSwiGLU) {
        constexpr int H = kBN2 / 2;
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
            store32_bf16(reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc + col0, v);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kBN2 / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
          const int col0 = n_blk * kBN2 + c * 32;
          if (row_ok && col0 < p.N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if constexpr (EPI == kEpiStoreF32) {
              float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc +
                                                      col0);
#pragma unroll
              for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
              if constexpr (EPI == kEpiResidual) {
                float rv[32];
                load32_bf16(p.R + static_cast<int64_t>(row) * p.ldr + col0, rv);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += rv[j];
              }
              store32_bf16(reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc + col0, v);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(tempty_leader0 + acc * 8);
    }
    // cross-GPU signal (reduce-scatter push): this CTA's stores are visible system-wide first
    if (p.tp.rs_cnt[0]) {
      __threadfence_system();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0 && !*abort_flag)
        for (int d = 0; d < p.tp.world; ++d) red_add_release_sys(p.tp.rs_cnt[d] + p.tp.rank, 1ull);
    }
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers or read its TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512));
  }
}

template <int EPI>
int launch_pair(const GemmArgs& a, cudaStream_t stream) {
  CUtensorMap ma, mb;
  if (!make_bf16_map(&ma, a.A, a.M, a.K, a.lda, kBM2)) return -10;
  if (!make_bf16_map(&mb, a.B, a.N, a.K, a.ldb, kBN2 / 2)) return -11;
  auto kern = gemm_pair_kernel<EPI>;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(kern), kSmem2)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemm_pair_grid(a.M, a.N), 1, 1);
  cfg.blockDim = dim3(kThreads2, 1, 1);
  cfg.dynamicSmemBytes = kSmem2;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

int gemm_bf16_pair(const GemmArgs& a, int epi, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return 0;
  if ((a.K % 8) || (a.lda % 8) || (a.ldb % 8) || (a.N % 32)) return -1;
  if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15)) return -2;
  switch (epi) {
    case kEpiStoreBf16:
      return launch_pair<kEpiStoreBf16>(a, stream);
    case kEpiResidual:
      return launch_pair<kEpiResidual>(a, stream);
    case kEpiSwiGLU:
      return launch_pair<kEpiSwiGLU>(a, stream);
    case kEpiStoreF32:
      return launch_pair<kEpiStoreF32>(a, stream);
    case kEpiRSPush:
      return launch_pair<kEpiRSPush>(a, stream);
    case kEpiQKV:
      if (a.N % kBN2 || a.N != (a.n_q_heads + 2 * a.n_kv_heads) * 128) return -3;
      return launch_pair<kEpiQKV>(a, stream);
    default:
      return -4;
  }
}

int gemm_pair_grid(int M, int N) {
  const int tiles = ((M + 2 * kBM2 - 1) / (2 * kBM2)) * ((N + kBN2 - 1) / kBN2);
  int pairs = num_sms() / 2;
  if (pairs > tiles) pairs = tiles;
  return 2 * pairs;
}

}  // namespace lakeb
