// Paged attention for sm_100a over the page-first KV arena
//   arena[num_blocks, layers, 2 (K,V), kv_heads, 16 tokens, 128 dims]  (bf16)
//
// K/V tiles are fetched with 2-D TMA boxes (16 tokens x 64 dims, 128-byte
// swizzle) addressed through the block table, so every page arrives in shared
// memory in a bank-conflict-free layout for ldmatrix. The score and value
// products run on the warp-level tensor cores (mma.m16n8k16); both kernels are
// bound by K/V bytes, not by math.
//
//  * paged_decode: one query token per sequence, all G = n_q/n_kv query heads of
//    a KV head share one pass over the pages (rows of the 16-row MMA tile),
//    four warps take one page each per stage, split-KV over the sequence when
//    the batch is too small to fill the GPU (partials combined by a second
//    kernel).
//  * paged_prefill: FlashAttention-2 style causal prefill over query tiles of
//    up to 64 tokens; the keys are the whole paged context, so chunked prefill
//    and prefix reuse (queries starting after a cached prefix) use the same path.
//
// Reference parity: replaces the pure-Python causal / residual-query attention
// (python/lake/kernels/attn_ref.py:13-56) and the SDPA backend
// (python/lake/engine/model_executor/layers/attentions/attention.py:83-125).
#include <math_constants.h>

#include "common.cuh"
#include "lakeb_kernels.h"
#include "mma_sync.cuh"
#include "tma_host.h"

namespace lakeb {
namespace {

constexpr int kStages = 3;
constexpr int kPageTokens = 16;
constexpr int kHeadDim = 128;
constexpr int kPageHalfBytes = kPageTokens * 64 * 2;  // 2 KB: 16 tokens x 64 dims
constexpr int kPageBytes = 2 * kPageHalfBytes;         // 4 KB: one head's K (or V) page
constexpr int kStageBytes = 4 * 2 * kPageBytes;        // 4 pages of K and V
constexpr int kSmemBytes = kStages * kStageBytes + 64 + 1024;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ int64_t page_row(const PagedAttnArgs& a, int64_t phys, int kv, int head) {
  return (((phys * a.num_layers + a.layer) * 2 + kv) * a.n_kv_heads + head) * kPageTokens;
}

// Issue the TMA loads of one page (K and V of one head) into `dst` (8 KB).
__device__ __forceinline__ void load_page(const CUtensorMap* map, const PagedAttnArgs& a, uint8_t* dst, uint64_t* bar,
                                          int64_t phys, int head) {
  const int yk = static_cast<int>(page_row(a, phys, 0, head));
  const int yv = static_cast<int>(page_row(a, phys, 1, head));
  tma_load_2d(dst, map, bar, 0, yk);
  tma_load_2d(dst + kPageHalfBytes, map, bar, 64, yk);
  tma_load_2d(dst + kPageBytes, map, bar, 0, yv);
  tma_load_2d(dst + kPageBytes + kPageHalfBytes, map, bar, 64, yv);
}

// S(16 x 16 tokens) = Q(16 x 128) . K_page^T   (two n-tiles of 8 tokens)
__device__ __forceinline__ void qk_page(const uint32_t (&qa)[8][4], uint32_t kbase, int lane, float (&s)[2][4]) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
  const int j = lane >> 3, r = lane & 7;
  const int token = (j >> 1) * 8 + r;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int chunk = 2 * kk + (j & 1);
    const uint32_t addr = kbase + (chunk >> 3) * kPageHalfBytes + sw128_off(token, chunk & 7);
    uint32_t k0, k1, k2, k3;
    ldsm_x4(addr, k0, k1, k2, k3);
    mma_bf16_16816(s[0], qa[kk], k0, k1);
    mma_bf16_16816(s[1], qa[kk], k2, k3);
  }
}

// O(16 x 128) += P(16 x 16 tokens) . V_page(16 x 128)
__device__ __forceinline__ void pv_page(const uint32_t (&pa)[4], uint32_t vbase, int lane, float (&o)[16][4]) {
  const int j = lane >> 3, r = lane & 7;
  const int token = (j & 1) * 8 + r;
#pragma unroll
  for (int c = 0; c < 16; c += 2) {
    const int chunk = c + (j >> 1);
    const uint32_t addr = vbase + (chunk >> 3) * kPageHalfBytes + sw128_off(token, chunk & 7);
    uint32_t v0, v1, v2, v3;
    ldsm_x4_t(addr, v0, v1, v2, v3);
    mma_bf16_16816(o[c], pa, v0, v1);
    mma_bf16_16816(o[c + 1], pa, v2, v3);
  }
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// Load Q rows (row0 = lane/4, row1 = row0 + 8) into mma A fragments.
__device__ __forceinline__ void load_q_frags(const __nv_bfloat16* q0, const __nv_bfloat16* q1, int lane,
                                             uint32_t (&qa)[8][4]) {
  const int c = (lane & 3) * 2;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int col = kk * 16 + c;
    qa[kk][0] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + col) : 0u;
    qa[kk][1] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + col) : 0u;
    qa[kk][2] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + col + 8) : 0u;
    qa[kk][3] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + col + 8) : 0u;
  }
}

// Online-softmax update for NT n-tiles of scores already scaled to log2 units.
template <int NT>
__device__ __forceinline__ void softmax_update(float (&s)[NT][4], float (&m)[2], float (&l)[2], float (&o)[16][4]) {
  float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
    mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
  }
  mx0 = quad_max(mx0);
  mx1 = quad_max(mx1);
  const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
  const float b0 = mn0 == -CUDART_INF_F ? 0.f : mn0;
  const float b1 = mn1 == -CUDART_INF_F ? 0.f : mn1;
  const float al0 = exp2f(m[0] - b0), al1 = exp2f(m[1] - b1);
  float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    s[nt][0] = exp2f(s[nt][0] - b0);
    s[nt][1] = exp2f(s[nt][1] - b0);
    s[nt][2] = exp2f(s[nt][2] - b1);
    s[nt][3] = exp2f(s[nt][3] - b1);
    rs0 += s[nt][0] + s[nt][1];
    rs1 += s[nt][2] + s[nt][3];
  }
  l[0] = l[0] * al0 + rs0;
  l[1] = l[1] * al1 + rs1;
  m[0] = mn0;
  m[1] = mn1;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    o[c][0] *= al0;
    o[c][1] *= al0;
    o[c][2] *= al1;
    o[c][3] *= al1;
  }
}

// ------------------------------------------------------------------ decode
__global__ void __launch_bounds__(128) paged_decode_kernel(const __grid_constant__ CUtensorMap kvmap,
                                                             const PagedAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);

  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int len = a.seq_lens[seq];
  const int nblk = (len + kPageTokens - 1) / kPageTokens;
  const int per = (nblk + a.splits - 1) / a.splits;
  const int b0 = split * per;
  const int b1 = min(nblk, b0 + per);
  const int iters = b1 > b0 ? (b1 - b0 + 3) / 4 : 0;
  const int* bt = a.block_tables + static_cast<int64_t>(seq) * a.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int it) {
    const int buf = it % kStages;
    const int first = b0 + it * 4;
    const int n = min(4, b1 - first);
    int pg[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {  // all ids before the first TMA issue
      pg[b] = b < n ? bt[first + b] : 0;
      if (!in_bounds(pg[b] >= 0 && pg[b] < a.num_blocks, a.status)) pg[b] = 0;  // debug build only
    }
    mbar_expect_tx(&full[buf], n * 2 * kPageBytes);
    for (int b = 0; b < n; ++b)
      load_page(&kvmap, a, smem + buf * kStageBytes + b * 2 * kPageBytes, &full[buf], pg[b], kvh);
  };
  if (threadIdx.x == 0)
    for (int it = 0; it < min(kStages, iters); ++it) issue(it);

  const int r0 = lane >> 2, r1 = r0 + 8;
  const __nv_bfloat16* qbase = a.q + static_cast<int64_t>(seq) * a.q_stride + static_cast<int64_t>(kvh) * G * kHeadDim;
  uint32_t qa[8][4];
  load_q_frags(r0 < G ? qbase + r0 * kHeadDim : nullptr, r1 < G ? qbase + r1 * kHeadDim : nullptr, lane, qa);

  const float sl2 = a.scale * kLog2e;
  float m[2] = {-CUDART_INF_F, -CUDART_INF_F}, l[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int c = 0; c < 16; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[c][e] = 0.f;

  bool ok = true;
  for (int it = 0; it < iters; ++it) {
    const int buf = it % kStages;
    if (ok && !mbar_wait(&full[buf], (it / kStages) & 1, nullptr, a.status)) ok = false;
    const int blk = b0 + it * 4 + warp;
    if (ok && blk < b1) {
      const uint32_t kb = smem_u32(smem + buf * kStageBytes + warp * 2 * kPageBytes);
      float s[2][4];
      qk_page(qa, kb, lane, s);
      const int tok0 = blk * kPageTokens + (lane & 3) * 2;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] = (tok0 + nt * 8 + (e & 1) < len) ? s[nt][e] * sl2 : -CUDART_INF_F;
      softmax_update<2>(s, m, l, o);
      uint32_t pa[4] = {pack_bf16x2(s[0][0], s[0][1]), pack_bf16x2(s[0][2], s[0][3]), pack_bf16x2(s[1][0], s[1][1]),
                        pack_bf16x2(s[1][2], s[1][3])};
      pv_page(pa, kb + kPageBytes, lane, o);
    }
    __syncthreads();
    if (threadIdx.x == 0 && ok && it + kStages < iters) issue(it + kStages);
  }

  l[0] = quad_sum(l[0]);
  l[1] = quad_sum(l[1]);
  // Cross-warp merge through shared memory (the stage buffers are idle now).
  float* so = reinterpret_cast<float*>(smem);       // [4][16][128]
  float* sm = so + 4 * 16 * kHeadDim;               // [4][16]
  float* sls = sm + 64;                             // [4][16]
  {
    const int cb = (lane & 3) * 2;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      so[(warp * 16 + r0) * kHeadDim + c * 8 + cb] = o[c][0];
      so[(warp * 16 + r0) * kHeadDim + c * 8 + cb + 1] = o[c][1];
      so[(warp * 16 + r1) * kHeadDim + c * 8 + cb] = o[c][2];
      so[(warp * 16 + r1) * kHeadDim + c * 8 + cb + 1] = o[c][3];
    }
    if ((lane & 3) == 0) {
      sm[warp * 16 + r0] = m[0];
      sm[warp * 16 + r1] = m[1];
      sls[warp * 16 + r0] = l[0];
      sls[warp * 16 + r1] = l[1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * kHeadDim; idx += blockDim.x) {
    const int g = idx / kHeadDim, d = idx % kHeadDim;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w * 16 + g]);
    float acc = 0.f, L = 0.f;
    if (M != -CUDART_INF_F) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm[w * 16 + g] - M);
        acc += so[(w * 16 + g) * kHeadDim + d] * f;
        L += sls[w * 16 + g] * f;
      }
    }
    const int qh = kvh * G + g;
    if (a.splits == 1) {
      a.out[static_cast<int64_t>(seq) * a.out_stride + qh * kHeadDim + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
    } else {
      const int64_t part = ((static_cast<int64_t>(seq) * a.n_kv_heads + kvh) * a.splits + split) * G + g;
      a.ws_o[part * kHeadDim + d] = acc;
      if (d == 0) {
        a.ws_ml[part * 2] = M;
        a.ws_ml[part * 2 + 1] = L;
      }
    }
  }
}

__global__ void __launch_bounds__(128) decode_combine_kernel(const PagedAttnArgs a) {
  const int qh = blockIdx.x, seq = blockIdx.y, d = threadIdx.x;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int kvh = qh / G, g = qh % G;
  const int64_t base = (static_cast<int64_t>(seq) * a.n_kv_heads + kvh) * a.splits;
  float M = -CUDART_INF_F;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.ws_ml[((base + s) * G + g) * 2]);
  float acc = 0.f, L = 0.f;
  if (M != -CUDART_INF_F) {
    for (int s = 0; s < a.splits; ++s) {
      const int64_t part = (base + s) * G + g;
      const float f = exp2f(a.ws_ml[part * 2] - M);
      acc += a.ws_o[part * kHeadDim + d] * f;
      L += a.ws_ml[part * 2 + 1] * f;
    }
  }
  a.out[static_cast<int64_t>(seq) * a.out_stride + qh * kHeadDim + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
}

// ------------------------------------------------------------------ prefill
__global__ void __launch_bounds__(128) paged_prefill_kernel(const __grid_constant__ CUtensorMap kvmap,
                                                              const PagedAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);

  const int4 tile = a.tiles[blockIdx.x];
  const int seq = tile.x, qrow0 = tile.y, nq = tile.z, pos0 = tile.w;
  const int qh = blockIdx.y;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int kvh = qh / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = a.seq_lens[seq];
  const int nblk = (len + kPageTokens - 1) / kPageTokens;
  const int max_pos = min(pos0 + nq - 1, len - 1);
  const int n_tiles = min((len + 63) / 64, max_pos / 64 + 1);
  const int* bt = a.block_tables + static_cast<int64_t>(seq) * a.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int j) {
    const int buf = j % kStages;
    int pg[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      pg[b] = bt[min(j * 4 + b, nblk - 1)];  // past-the-end: last page (masked)
      if (!in_bounds(pg[b] >= 0 && pg[b] < a.num_blocks, a.status)) pg[b] = 0;  // debug build only
    }
    mbar_expect_tx(&full[buf], kStageBytes);
    for (int b = 0; b < 4; ++b)
      load_page(&kvmap, a, smem + buf * kStageBytes + b * 2 * kPageBytes, &full[buf], pg[b], kvh);
  };
  if (threadIdx.x == 0)
    for (int j = 0; j < min(kStages, n_tiles); ++j) issue(j);

  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
  const int qp0 = pos0 + r0, qp1 = pos0 + r1;
  const __nv_bfloat16* q0 = r0 < nq ? a.q + static_cast<int64_t>(qrow0 + r0) * a.q_stride + qh * kHeadDim : nullptr;
  const __nv_bfloat16* q1 = r1 < nq ? a.q + static_cast<int64_t>(qrow0 + r1) * a.q_stride + qh * kHeadDim : nullptr;
  uint32_t qa[8][4];
  load_q_frags(q0, q1, lane, qa);

  const float sl2 = a.scale * kLog2e;
  float m[2] = {-CUDART_INF_F, -CUDART_INF_F}, l[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int c = 0; c < 16; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[c][e] = 0.f;

  const int warp_max_pos = pos0 + warp * 16 + 15;
  bool ok = true;
  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j % kStages;
    if (ok && !mbar_wait(&full[buf], (j / kStages) & 1, nullptr, a.status)) ok = false;
    if (ok && j * 64 <= warp_max_pos) {
      const uint32_t sbase = smem_u32(smem + buf * kStageBytes);
      float s[8][4];
#pragma unroll
      for (int pg = 0; pg < 4; ++pg) {
        float sp[2][4];
        qk_page(qa, sbase + pg * 2 * kPageBytes, lane, sp);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[2 * pg][e] = sp[0][e];
          s[2 * pg + 1][e] = sp[1][e];
        }
      }
      const bool need_mask = (j * 64 + 63 > pos0 + warp * 16) || (j * 64 + 63 >= len);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kp = j * 64 + nt * 8 + (lane & 3) * 2 + (e & 1);
          const int qp = (e < 2) ? qp0 : qp1;
          const bool valid = !need_mask || (kp <= qp && kp < len);
          s[nt][e] = valid ? s[nt][e] * sl2 : -CUDART_INF_F;
        }
      softmax_update<8>(s, m, l, o);
#pragma unroll
      for (int pg = 0; pg < 4; ++pg) {
        uint32_t pa[4] = {pack_bf16x2(s[2 * pg][0], s[2 * pg][1]), pack_bf16x2(s[2 * pg][2], s[2 * pg][3]),
                          pack_bf16x2(s[2 * pg + 1][0], s[2 * pg + 1][1]),
                          pack_bf16x2(s[2 * pg + 1][2], s[2 * pg + 1][3])};
        pv_page(pa, sbase + pg * 2 * kPageBytes + kPageBytes, lane, o);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && ok && j + kStages < n_tiles) issue(j + kStages);
  }

  l[0] = quad_sum(l[0]);
  l[1] = quad_sum(l[1]);
  const float inv0 = l[0] > 0.f ? 1.f / l[0] : 0.f;
  const float inv1 = l[1] > 0.f ? 1.f / l[1] : 0.f;
  const int cb = (lane & 3) * 2;
  if (r0 < nq) {
    __nv_bfloat16* dst = a.out + static_cast<int64_t>(qrow0 + r0) * a.out_stride + qh * kHeadDim;
#pragma unroll
    for (int c = 0; c < 16; ++c)
      *reinterpret_cast<uint32_t*>(dst + c * 8 + cb) = pack_bf16x2(o[c][0] * inv0, o[c][1] * inv0);
  }
  if (r1 < nq) {
    __nv_bfloat16* dst = a.out + static_cast<int64_t>(qrow0 + r1) * a.out_stride + qh * kHeadDim;
#pragma unroll
    for (int c = 0; c < 16; ++c)
      *reinterpret_cast<uint32_t*>(dst + c * 8 + cb) = pack_bf16x2(o[c][2] * inv1, o[c][3] * inv1);
  }
}

bool arena_map(CUtensorMap* map, const PagedAttnArgs& a) {
  const int64_t rows = a.num_blocks * a.num_layers * 2 * a.n_kv_heads * kPageTokens;
  if (rows >= (int64_t(1) << 31)) return false;
  return make_bf16_map(map, a.arena, rows, kHeadDim, kHeadDim, kPageTokens, 64);
}

}  // namespace

// Split-KV count: the grid is seqs x kv_heads x splits CTAs, two resident per SM (97 KB of
// shared memory each). Default (mode 0, fill): just enough splits for two CTAs per SM. Mode 1
// picks the split count with the best last-wave fill (80 x 8 CTAs on 296 slots is 2.16 waves),
// moving to more splits only for a >3% gain, with >= 8 pages per split; on B200 at 80 x 2196
// it measured 0.3 ms per step slower (more, shorter CTAs plus the combine kernel).
static int g_split_mode = 0;
void set_decode_split_mode(int mode) { g_split_mode = mode; }

int paged_decode_splits(int num_seqs, int n_kv_heads, int max_blocks_per_seq) {
  const long long ctas = static_cast<long long>(num_seqs) * n_kv_heads;
  if (ctas <= 0) return 1;
  if (g_split_mode == 0) {
    const long long target = 2LL * num_sms();
    if (ctas >= target) return 1;
    int s = static_cast<int>((target + ctas - 1) / ctas);
    int cap = max_blocks_per_seq / 8;
    if (cap < 1) cap = 1;
    if (s > cap) s = cap;
    return s > 32 ? 32 : s;
  }
  const long long slots = 2LL * num_sms();
  int cap = max_blocks_per_seq / 8;
  if (cap < 1) cap = 1;
  if (cap > 32) cap = 32;
  auto eff = [&](int s) {
    const long long n = ctas * s;
    return static_cast<double>(n) / static_cast<double>(((n + slots - 1) / slots) * slots);
  };
  int best = 1;
  double best_eff = eff(1);
  for (int s = 2; s <= cap; ++s) {
    const double e = eff(s);
    if (e > best_eff + 0.03) {
      best = s;
      best_eff = e;
    }
  }
  return best;
}

int paged_decode(const PagedAttnArgs& a, cudaStream_t stream) {
  if (a.num_seqs <= 0) return 0;
  if (a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads || a.n_q_heads / a.n_kv_heads > 16) return -1;
  if (a.splits > 1 && (!a.ws_o || !a.ws_ml)) return -2;
  CUtensorMap map;
  if (!arena_map(&map, a)) return -3;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(paged_decode_kernel), kSmemBytes)) return e;
  dim3 grid(a.splits, a.n_kv_heads, a.num_seqs);
  paged_decode_kernel<<<grid, 128, kSmemBytes, stream>>>(map, a);
  if (a.splits > 1) decode_combine_kernel<<<dim3(a.n_q_heads, a.num_seqs), kHeadDim, 0, stream>>>(a);
  return cudaGetLastError();
}

int paged_decode_with_map(const PagedAttnArgs& a, const CUtensorMap& map, cudaStream_t stream) {
  if (a.num_seqs <= 0) return 0;
  if (a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads || a.n_q_heads / a.n_kv_heads > 16) return -1;
  if (a.splits > 1 && (!a.ws_o || !a.ws_ml)) return -2;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(paged_decode_kernel), kSmemBytes)) return e;
  dim3 grid(a.splits, a.n_kv_heads, a.num_seqs);
  paged_decode_kernel<<<grid, 128, kSmemBytes, stream>>>(map, a);
  if (a.splits > 1) decode_combine_kernel<<<dim3(a.n_q_heads, a.num_seqs), kHeadDim, 0, stream>>>(a);
  return cudaGetLastError();
}

int paged_prefill(const PagedAttnArgs& a, cudaStream_t stream) {
  if (a.num_tiles <= 0) return 0;
  if (a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads) return -1;
  CUtensorMap map;
  if (!arena_map(&map, a)) return -3;
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(paged_prefill_kernel), kSmemBytes)) return e;
  dim3 grid(a.num_tiles, a.n_q_heads);
  paged_prefill_kernel<<<grid, 128, kSmemBytes, stream>>>(map, a);
  return cudaGetLastError();
}

}  // namespace lakeb
