// Causal prefill attention on the 5th-generation tensor cores (sm_100a).
//
// One CTA = 128 query rows of one query head. Per 128-key tile j of the paged
// context:
//   S_j   = Q K_j^T        tcgen05.mma (M=128, N=128, K=128), fp32 in TMEM (2 buffers)
//   P_j   = exp2(S_j*scale - m_j)   softmax warpgroup: tcgen05.ld S rows, row max/sum,
//                                   bf16 P written to shared memory (128-byte swizzle)
//   O~_j  = P_j V_j        tcgen05.mma with V as an MN-major operand, fp32 in TMEM
//   O    <- O*alpha_j + O~_{j-1}    rescale-and-add in registers of the softmax warps
// so the tensor core computes S_{j+1} and O~_j while the softmax warps work on
// tile j. K/V pages (16 tokens x 64 dims boxes) are fetched by TMA through the
// block table into a [dim half][key][64 dims] layout that serves both as the
// K-major B operand of QK^T and the MN-major B operand of PV.
//
// Warp roles: 0 = TMA producer, 1 = TMEM allocator + MMA issuer, 2..5 = softmax
// and epilogue (thread = query row). All waits are bounded (common.cuh).
//
// Reference parity: python/lake/kernels/attn_ref.py:13-56 (causal and
// residual-query attention) and the SDPA backend of
// python/lake/engine/model_executor/layers/attentions/attention.py:83-125.
#include <math_constants.h>

#include "common.cuh"
#include "lakeb_kernels.h"
#include "tma_host.h"

namespace lakeb {
namespace {

constexpr int kTileK = 128;
constexpr int kHalfBytes = 128 * 128;  // 128 rows x 64 dims x 2 B = 16 KB
constexpr int kOperandBytes = 2 * kHalfBytes;  // 32 KB: two 64-dim halves
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kOperandBytes;          // 2 stages
constexpr int kVOff = kKOff + 2 * kOperandBytes;      // 2 stages
constexpr int kPOff = kVOff + 2 * kOperandBytes;      // 1 buffer
constexpr int kBarOff = kPOff + kOperandBytes;        // 192 KB
constexpr int kRedOff = kBarOff + 256;                // row-max / row-sum exchange, 2 KB
constexpr int kSmemBytes = kRedOff + 2 * 2 * 128 * 4 + 1024;
constexpr int kThreadsTC = 320;                       // producer, MMA, two softmax warpgroups
constexpr float kLog2e = 1.4426950408889634f;

// Shared-memory descriptor, MN-major operand with the 128-byte swizzle:
// 64-element MN chunks `lbo` bytes apart, 8-row K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// bf16 x bf16 -> fp32, A K-major, B MN-major.
// exp2 via the MUFU instruction (inputs here are <= 0 or -inf; results are probabilities).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__host__ __device__ constexpr uint32_t idesc_bf16_bmn(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ int64_t page_row_tc(const PagedAttnArgs& a, int64_t phys, int kv, int head) {
  return (((phys * a.num_layers + a.layer) * 2 + kv) * a.n_kv_heads + head) * 16;
}

__global__ void __launch_bounds__(kThreadsTC, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kvmap, const __grid_constant__ CUtensorMap qmap,
                            const PagedAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* o_full = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 14);

  // heavy (late) query tiles first: the grid is laid out in reverse tile order
  const int tile_idx = a.num_tiles - 1 - static_cast<int>(blockIdx.x);
  const int4 tile = a.tiles[tile_idx];
  const int seq = tile.x, qrow0 = tile.y, nq = tile.z, pos0 = tile.w;
  const int qh = blockIdx.y;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int kvh = qh / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = a.seq_lens[seq];
  const int nblk = (len + 15) >> 4;
  const int max_pos = min(pos0 + nq - 1, len - 1);
  const int n_tiles = max_pos < 0 ? 0 : max_pos / kTileK + 1;
  const int* bt = a.block_tables + static_cast<int64_t>(seq) * a.bt_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
    }
    mbar_init(p_full, 256);
    mbar_init(o_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      // ---------------------------------------------------------- producer
      mbar_expect_tx(q_full, kOperandBytes);
      tma_load_2d(smem + kQOff, &qmap, q_full, qh * 128, qrow0);
      tma_load_2d(smem + kQOff + kHalfBytes, &qmap, q_full, qh * 128 + 64, qrow0);
      bool ok = true;
      // Block-table entries are read one tile ahead, all eight at once, so no
      // global-load latency sits between consecutive TMA issues.
      int pg_next[8];
#pragma unroll
      for (int p = 0; p < 8; ++p) pg_next[p] = bt[min(p, nblk - 1)];
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        int pg[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          pg[p] = pg_next[p];
          if (!in_bounds(pg[p] >= 0 && pg[p] < a.num_blocks, a.status)) pg[p] = 0;  // debug build only
        }
        if (j + 1 < n_tiles) {
#pragma unroll
          for (int p = 0; p < 8; ++p) pg_next[p] = bt[min((j + 1) * 8 + p, nblk - 1)];
        }
        for (int kv = 0; kv < 2 && ok; ++kv) {
          uint64_t* empty = kv ? &v_empty[s] : &k_empty[s];
          uint64_t* full = kv ? &v_full[s] : &k_full[s];
          if (!mbar_wait(empty, ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + (kv ? kVOff : kKOff) + s * kOperandBytes;
          mbar_expect_tx(full, kOperandBytes);
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int y = static_cast<int>(page_row_tc(a, pg[p], kv, kvh));
            tma_load_2d(dst + p * 2048, &kvmap, full, 0, y);
            tma_load_2d(dst + kHalfBytes + p * 2048, &kvmap, full, 64, y);
          }
        }
      }
      // tail: the buffer-release arrivals of the last two tiles must land before the CTA exits
      for (int j = max(0, n_tiles - 2); j < n_tiles && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait(&k_empty[s], (j >> 1) & 1, abort_flag, a.status) &&
             mbar_wait(&v_empty[s], (j >> 1) & 1, abort_flag, a.status);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128);
      constexpr uint32_t idesc_o = idesc_bf16_bmn(128, 128);
      const uint32_t q_base = smem_u32(smem + kQOff);
      const uint32_t p_base = smem_u32(smem + kPOff);
      bool ok = mbar_wait(q_full, 0, abort_flag, a.status);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, a.status)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + kKOff + s * kOperandBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_f16(t_s[s], umma_desc_sw128(q_base + off), umma_desc_sw128(k_base + off), idesc_s, k > 0);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        return true;
      };
      for (int j = 0; j < min(2, n_tiles) && ok; ++j) ok = issue_s(j);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(p_full, j & 1, abort_flag, a.status)) break;
        if (!mbar_wait(&v_full[s], (j >> 1) & 1, abort_flag, a.status)) break;
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + kVOff + s * kOperandBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t aoff = (k >> 2) * kHalfBytes + (k & 3) * 32;  // 16 keys of P (K-major)
          const uint32_t boff = k * 2048;                              // 16 keys of V (MN-major)
          umma_f16(t_o, umma_desc_sw128(p_base + aoff), umma_desc_sw128_mn(v_base + boff, kHalfBytes), idesc_o,
                   k > 0);
        }
        umma_commit(o_full);
        umma_commit(&v_empty[s]);
        if (j + 2 < n_tiles) ok = issue_s(j + 2);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    // Two warpgroups: warpgroup g owns columns [64g, 64g+64) of every row, so a
    // row's max is combined through shared memory once per tile; the row sum is
    // combined once at the end (both halves use the same running max).
    const int g = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row in the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const uint32_t col0 = static_cast<uint32_t>(g * 64);
    const int qpos = pos0 + r;
    const float sl2 = a.scale * kLog2e;
    uint8_t* prow = smem + kPOff + g * kHalfBytes + r * 128;
    float* red = reinterpret_cast<float*>(smem + kRedOff);  // [2 parity][2 groups][128 rows]
    const int sw = r & 7;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    float m = -CUDART_INF_F, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, abort_flag, a.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kTileK + g * 64;
      const bool need_mask = (j * kTileK + kTileK - 1 > pos0) || (j * kTileK + kTileK > len);
      const int kmax = min(qpos, len - 1);  // last visible key of this row
      // pass 1: raw row max over this thread's 64 columns (scale > 0 commutes with max)
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(t_s[s] + lane_off + col0 + c * 32, v);
        tmem_ld_wait();
        if (!need_mask) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) mx = fmaxf(mx, fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 1])));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            mx = fmaxf(mx, (k0 + c * 32 + i <= kmax) ? __uint_as_float(v[i]) : -CUDART_INF_F);
        }
      }
      red[(s * 2 + g) * 128 + r] = mx;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      mx = fmaxf(red[(s * 2 + 0) * 128 + r], red[(s * 2 + 1) * 128 + r]) * sl2;
      const float m_new = fmaxf(m, mx);
      const float base = m_new == -CUDART_INF_F ? 0.f : m_new;
      const float alpha = ex2_approx(m - base);
      // fold the previous tile's P.V into the register accumulator
      if (j > 0) {
        if (!mbar_wait(o_full, (j - 1) & 1, abort_flag, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld32(t_o + lane_off + col0 + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha_prev, __uint_as_float(v[i]));
        }
      }
      // pass 2: P = exp2(S*scale - m) -> bf16 into this group's 64-key half of P (swizzled K-major rows)
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(t_s[s] + lane_off + col0 + c * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p0 = ex2_approx(fmaf(__uint_as_float(v[i]), sl2, -base));
          float p1 = ex2_approx(fmaf(__uint_as_float(v[i + 1]), sl2, -base));
          if (need_mask) {
            p0 = (k0 + c * 32 + i <= kmax) ? p0 : 0.f;
            p1 = (k0 + c * 32 + i + 1 <= kmax) ? p1 : 0.f;
          }
          rs0 += p0;
          rs1 += p1;
          pk[i >> 1] = pack_bf16x2(p0, p1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = c * 4 + q;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ sw) << 4)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      l = fmaf(l, alpha, rs0 + rs1);
      m = m_new;
      alpha_prev = alpha;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n_tiles > 0 && mbar_wait(o_full, (n_tiles - 1) & 1, abort_flag, a.status)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(t_o + lane_off + col0 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha_prev, __uint_as_float(v[i]));
      }
      const int par = n_tiles & 1;  // parity not used by the last tile's max exchange
      red[(par * 2 + g) * 128 + r] = l;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float lt = red[(par * 2 + 0) * 128 + r] + red[(par * 2 + 1) * 128 + r];
      if (r < nq) {
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        uint4* dst =
            reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(qrow0 + r) * a.out_stride + qh * 128 + g * 64);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          dst[v] = make_uint4(pack_bf16x2(o[8 * v] * inv, o[8 * v + 1] * inv),
                              pack_bf16x2(o[8 * v + 2] * inv, o[8 * v + 3] * inv),
                              pack_bf16x2(o[8 * v + 4] * inv, o[8 * v + 5] * inv),
                              pack_bf16x2(o[8 * v + 6] * inv, o[8 * v + 7] * inv));
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

static int g_prefill_kernel = 1;
void set_prefill_kernel(int mode) {
  // 0: one head per CTA; 1: two heads per CTA (default softmax variant); 10 + i: softmax variant i
  g_prefill_kernel = mode >= 10 ? 1 : mode;
  set_prefill_variant(mode >= 10 ? mode - 10 : -1);
}

int paged_prefill_tc(const PagedAttnArgs& a, int64_t q_rows, cudaStream_t stream) {
  if (a.num_tiles <= 0) return 0;
  if (g_prefill_kernel == 1 && prefill_pingpong_ok(a)) return paged_prefill_pingpong(a, q_rows, stream);
  if (a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads) return -1;
  if (a.q_stride % 8 || (reinterpret_cast<uintptr_t>(a.q) & 15)) return -2;
  CUtensorMap kvmap, qmap;
  const int64_t rows = a.num_blocks * a.num_layers * 2 * a.n_kv_heads * 16;
  if (rows >= (int64_t(1) << 31)) return -3;
  if (!make_bf16_map(&kvmap, a.arena, rows, 128, 128, 16, 64)) return -4;
  if (!make_bf16_map(&qmap, a.q, q_rows, static_cast<int64_t>(a.n_q_heads) * 128, a.q_stride, 128, 64)) return -5;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(paged_prefill_tc_kernel), kSmemBytes)) return e;
  dim3 grid(a.num_tiles, a.n_q_heads);
  paged_prefill_tc_kernel<<<grid, kThreadsTC, kSmemBytes, stream>>>(kvmap, qmap, a);
  return cudaGetLastError();
}

}  // namespace lakeb
