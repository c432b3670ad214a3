// Causal prefill attention, two query heads per CTA in ping-pong (sm_100a).
//
// A CTA owns one tile of up to 128 query rows for two query heads A and B of the
// same KV group, so every K/V tile it stages serves both heads. Per 128-key tile j:
//   S_h   = Q_h K_j^T          tcgen05.mma (M=128, N=128, K=128), fp32 in TMEM
//   P_h   = exp2(S_h*scale - m_h)   softmax warpgroup h: thread = query row, the whole
//                                   row in registers; P written back as bf16 over the
//                                   first 64 TMEM columns of S_h
//   O_h  += P_h V_j            tcgen05.mma with A = P_h read from TMEM, B = V_j from
//                              shared memory (MN-major), fp32 accumulator in TMEM
// The MMA warp issues PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), ... so the tensor core
// works on one head while the other head's softmax runs. O is rescaled in TMEM only
// when a row's running max grows by more than 2^8 (lazy rescale): below that the
// stale max keeps P <= 256, which bf16 P and the fp32 sums absorb.
//
// Warp roles: 0 = TMA producer (Q once, K/V pages through the block table into a
// two-stage ring), 1 = TMEM allocator + MMA issuer, 2-5 = softmax/epilogue of head A,
// 6-9 = head B. Every wait is bounded (common.cuh): a stalled role records an error
// in the status word and the CTA winds down instead of hanging.
//
// Reference parity: python/lake/kernels/attn_ref.py:13-56 (causal and residual-query
// attention over a cached prefix).
#include <math_constants.h>

#include "common.cuh"
#include "lakeb_kernels.h"
#include "tma_host.h"

namespace lakeb {
namespace {

constexpr int kTile = 128;                      // query rows per CTA, keys per K/V tile
constexpr int kHalf = 128 * 128;                // 128 rows x 64 dims x 2 B = 16 KB
constexpr int kOperand = 2 * kHalf;             // 32 KB: both 64-dim halves
constexpr int kQA = 0, kQB = kOperand;          // Q of head A and B
constexpr int kK = 2 * kOperand;                // K ring, 2 stages
constexpr int kV = kK + 2 * kOperand;           // V ring, 2 stages
constexpr int kBars = kV + 2 * kOperand;        // 192 KB
constexpr int kSmem = kBars + 256 + 1024;       // + barriers, + 1 KB for the 1024-byte alignment
constexpr int kThreads = 320;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;            // rescale O when the row max grows by more than 2^8

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two-lane fp32 arithmetic (sm_100a f32x2): one issue slot for two results.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^x for two lanes on the FMA pipe instead of the transcendental unit: x = n + f with n
// an integer (rounded through the 1.5 * 2^23 trick) and f in [-0.5, 0.5]; 2^f from a degree-3
// polynomial fitted here to 2^f on [-0.5, 0.5] by iteratively reweighted least squares on the
// relative error (max relative error 7.5e-5, below bf16's 2^-9); 2^n is added to the exponent
// bits. x is clamped at -125 so the result stays a normal float (~2e-38 where the exact value
// underflows, which no softmax sum can tell from 0).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = add2(x, make_float2(kRound, kRound));
  const float2 n = add2(t, make_float2(-kRound, -kRound));
  const float2 f = add2(x, make_float2(-n.x, -n.y));
  float2 p = fma2(make_float2(0.05517167f, 0.05517167f), f, make_float2(0.24261114f, 0.24261114f));
  p = fma2(p, f, make_float2(0.69326097f, 0.69326097f));
  p = fma2(p, f, make_float2(0.99992806f, 0.99992806f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// bf16x2 from two floats by integer rounding (round half up on the dropped 16 bits) and one
// byte permute: ALU work instead of the conversion unit.
__device__ __forceinline__ uint32_t pack_bf16x2_int(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}

// MN-major shared-memory operand with the 128-byte swizzle: 64-element MN chunks `lbo`
// bytes apart, 8-row K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// bf16 x bf16 -> fp32; A K-major, B MN-major (bit 16).
__host__ __device__ constexpr uint32_t idesc_b_mn(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A is 128 rows (lanes) x 16 bf16 packed in 8 columns.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ int64_t page_row(const PagedAttnArgs& a, int64_t phys, int kv, int head) {
  return (((phys * a.num_layers + a.layer) * 2 + kv) * a.n_kv_heads + head) * 16;
}

// Timeline of one CTA (the first launched: the heaviest query tile of head pair 0), recorded
// while g_pp_trace_on is set (prefill_trace_enable) in SM clock cycles: slot [j * 16 + e] holds
// event e of K/V tile j (see kTr* below), slot [1023] the CTA's start. Read back with
// prefill_trace_read().
constexpr int kTraceSlots = 1024;
__device__ long long g_pp_trace[kTraceSlots];
__device__ int g_pp_trace_on;
enum : int {
  kTrMmaP0 = 0,      // MMA issuer: P of head A ready (before PV_A(j))
  kTrMmaP1 = 1,      // MMA issuer: P of head B ready (before PV_B(j))
  kTrMmaK = 2,       // MMA issuer: K tile j+1 landed (before S_A(j+1))
  kTrSmWake = 3,     // softmax head h (+4 for B): S(j) ready
  kTrSmLoaded = 4,   // scores in registers
  kTrSmExp = 5,      // P computed, TMEM stores issued
  kTrSmArrive = 6,   // P handed to the MMA issuer
  kTrLoadK = 11,     // producer: K stage free for tile j
  kTrLoadV = 12,     // producer: V stage free for tile j
};

// EMUL: every EMUL-th pair of probabilities is computed by exp2_poly2 (0: none); INTPACK:
// pack P to bf16 with integer ops instead of the converter.
template <int EMUL, bool INTPACK>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_pingpong_kernel(const __grid_constant__ CUtensorMap kvmap, const __grid_constant__ CUtensorMap qmap,
                            const PagedAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2 stages]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2 heads]
  uint64_t* p_full = bars + 11;  // [2 heads]
  uint64_t* o_done = bars + 13;  // [2 heads]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 16);

  // heavy (late) query tiles first: the grid runs in reverse tile order
  const int tile_idx = a.num_tiles - 1 - static_cast<int>(blockIdx.x);
  const int4 tile = a.tiles[tile_idx];
  const int seq = tile.x, qrow0 = tile.y, nq = tile.z, pos0 = tile.w;
  const bool traced = blockIdx.x == 0 && blockIdx.y == 0 && (threadIdx.x & 31) == 0 && g_pp_trace_on;
  auto tr = [&](int j, int e) {
    if (traced && j >= 0 && j < kTraceSlots / 16 - 1) g_pp_trace[j * 16 + e] = clock64();
  };
  if (traced && threadIdx.x == 0) g_pp_trace[kTraceSlots - 1] = clock64();
  const int qh0 = 2 * static_cast<int>(blockIdx.y);  // heads qh0 (A) and qh0 + 1 (B)
  const int kvh = qh0 / (a.n_q_heads / a.n_kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = a.seq_lens[seq];
  const int nblk = (len + 15) >> 4;
  const int max_pos = min(pos0 + nq - 1, len - 1);
  const int n_tiles = max_pos < 0 ? 0 : max_pos / kTile + 1;
  const int* bt = a.block_tables + static_cast<int64_t>(seq) * a.bt_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s[2] = {tmem, tmem + 128};        // S of head A, B (P overwrites its first 64 columns)
  const uint32_t t_o[2] = {tmem + 256, tmem + 384};  // O of head A, B

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      // ------------------------------------------------------------ TMA producer
      mbar_expect_tx(q_full, 2 * kOperand);
      for (int h = 0; h < 2; ++h) {
        uint8_t* dst = smem + (h ? kQB : kQA);
        tma_load_2d(dst, &qmap, q_full, (qh0 + h) * 128, qrow0);
        tma_load_2d(dst + kHalf, &qmap, q_full, (qh0 + h) * 128 + 64, qrow0);
      }
      bool ok = true;
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
          tr(j, kv ? kTrLoadV : kTrLoadK);
          uint8_t* dst = smem + (kv ? kV : kK) + s * kOperand;
          mbar_expect_tx(full, kOperand);
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int y = static_cast<int>(page_row(a, pg[p], kv, kvh));
            tma_load_2d(dst + p * 2048, &kvmap, full, 0, y);
            tma_load_2d(dst + kHalf + p * 2048, &kvmap, full, 64, y);
          }
        }
      }
      // the release arrivals of the last two tiles must land before the CTA exits
      for (int j = max(0, n_tiles - 2); j < n_tiles && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait(&k_empty[s], (j >> 1) & 1, abort_flag, a.status) &&
             mbar_wait(&v_empty[s], (j >> 1) & 1, abort_flag, a.status);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128);
      constexpr uint32_t idesc_o = idesc_b_mn(128, 128);
      const uint32_t q_base[2] = {smem_u32(smem + kQA), smem_u32(smem + kQB)};
      auto issue_s = [&](int h, int j) {
        const uint32_t k_base = smem_u32(smem + kK + (j & 1) * kOperand);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16(t_s[h], umma_desc_sw128(q_base[h] + off), umma_desc_sw128(k_base + off), idesc_s, k > 0);
        }
        umma_commit(&s_full[h]);
      };
      auto issue_pv = [&](int h, int j) {
        const uint32_t v_base = smem_u32(smem + kV + (j & 1) * kOperand);
#pragma unroll
        for (int k = 0; k < 8; ++k)  // 16 keys per step: P columns 8k..8k+7, V rows 16k..16k+15
          umma_f16_ts(t_o[h], t_s[h] + 8 * k, desc_sw128_mn(v_base + k * 2048, kHalf), idesc_o, (j > 0) || (k > 0));
        umma_commit(&o_done[h]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, a.status) && mbar_wait(&k_full[0], 0, abort_flag, a.status);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j & 1, sn = (j + 1) & 1;
        const bool more = j + 1 < n_tiles;
        ok = mbar_wait(&v_full[s], (j >> 1) & 1, abort_flag, a.status);
        for (int h = 0; h < 2 && ok; ++h) {
          if (!mbar_wait(&p_full[h], j & 1, abort_flag, a.status)) {
            ok = false;
            break;
          }
          tr(j, h ? kTrMmaP1 : kTrMmaP0);
          tc_fence_after();
          issue_pv(h, j);
          if (h == 1) umma_commit(&v_empty[s]);
          if (more) {
            if (h == 0) {
              if (!mbar_wait(&k_full[sn], ((j + 1) >> 1) & 1, abort_flag, a.status)) {
                ok = false;
                break;
              }
              tr(j, kTrMmaK);
              tc_fence_after();
            }
            issue_s(h, j + 1);  // after PV(h, j) in issue order: P's columns are read before S overwrites them
          }
        }
        if (ok && more) umma_commit(&k_empty[sn]);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax + epilogue
    const int h = (warp - 2) >> 2;  // 0 = head A (warps 2-5), 1 = head B (warps 6-9)
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row in the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const int qpos = pos0 + r;
    const int kmax = min(qpos, len - 1);  // last key this row may see
    const float sl2 = a.scale * kLog2e;
    const bool tw = (warp & 3) == 2;  // warps 2 and 6 record the softmax timeline
    const int te = h ? 4 : 0;
    float m = -CUDART_INF_F;  // running max in log2 units (the base of P; may trail the true max by < 8)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[h], j & 1, abort_flag, a.status))) {
        ok = false;
        break;
      }
      if (tw) tr(j, kTrSmWake + te);
      tc_fence_after();
      // the row's 128 scores: four loads in flight, one wait
      const int k0 = j * kTile;
      uint32_t sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld32(t_s[h] + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32 * c));
      tmem_ld_wait();
      if (tw) tr(j, kTrSmLoaded + te);
      if (k0 + kTile - 1 > kmax) {  // the diagonal or the sequence end: keys past this row's last
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (k0 + i > kmax) sv[i] = __float_as_uint(-CUDART_INF_F);
      }
      // row max: eight independent three-input chains, then a short tree
      float mv[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mv[c] = max3f(__uint_as_float(sv[c]), __uint_as_float(sv[8 + c]), -CUDART_INF_F);
#pragma unroll
      for (int i = 16; i < 128; i += 16)
#pragma unroll
        for (int c = 0; c < 8; ++c) mv[c] = max3f(mv[c], __uint_as_float(sv[i + c]), __uint_as_float(sv[i + 8 + c]));
      float mx = max3f(max3f(mv[0], mv[1], mv[2]), max3f(mv[3], mv[4], mv[5]), fmaxf(mv[6], mv[7])) * sl2;
      const bool grow = mx > m + kRescaleLog2;
      const float m_old = m;
      if (grow) m = mx;
      const float base = m == -CUDART_INF_F ? 0.f : m;
      float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 sl2v = make_float2(sl2, sl2), nbase = make_float2(-base, -base);
#pragma unroll
      for (int k = 0; k < 64; ++k) {  // key pair k -> packed column k (written over consumed scores)
        const float2 z = fma2(make_float2(__uint_as_float(sv[2 * k]), __uint_as_float(sv[2 * k + 1])), sl2v, nbase);
        float2 p;
        if (EMUL > 0 && k % EMUL == EMUL - 1) {
          p = exp2_poly2(z);
        } else {
          p.x = ex2(z.x);
          p.y = ex2(z.y);
        }
        rs[k & 3] = add2(rs[k & 3], p);
        sv[k] = INTPACK ? pack_bf16x2_int(p.x, p.y) : pack_bf16x2(p.x, p.y);
        if (k == 31) tmem_st32(t_s[h] + lane_off, *reinterpret_cast<uint32_t(*)[32]>(sv));
      }
      tmem_st32(t_s[h] + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
      if (tw) tr(j, kTrSmExp + te);
      rs[0] = add2(add2(rs[0], rs[1]), add2(rs[2], rs[3]));
      // O and l still hold sums against the old base: bring them to m (after P, so the 128 scores
      // are no longer live). tcgen05.ld/st are warp-collective: the whole warp rescales when any
      // of its rows needs it (rows that do not keep alpha = 1).
      float alpha = 1.f;
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&o_done[h], (j - 1) & 1, abort_flag, a.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        alpha = (grow && m_old != -CUDART_INF_F) ? ex2(m_old - m) : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(t_o[h] + lane_off + c * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(t_o[h] + lane_off + c * 32, ov);
        }
      }
      l = fmaf(l, alpha, rs[0].x + rs[0].y);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[h]);
      if (tw) tr(j, kTrSmArrive + te);
    }
    if (ok && n_tiles > 0 &&
        __all_sync(0xffffffffu, mbar_wait(&o_done[h], (n_tiles - 1) & 1, abort_flag, a.status))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = a.out + static_cast<int64_t>(qrow0 + r) * a.out_stride + (qh0 + h) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        tmem_ld32(t_o[h] + lane_off + c * 32, ov);
        tmem_ld_wait();
        if (r < nq) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(pack_bf16x2(__uint_as_float(ov[8 * v]) * inv, __uint_as_float(ov[8 * v + 1]) * inv),
                                pack_bf16x2(__uint_as_float(ov[8 * v + 2]) * inv, __uint_as_float(ov[8 * v + 3]) * inv),
                                pack_bf16x2(__uint_as_float(ov[8 * v + 4]) * inv, __uint_as_float(ov[8 * v + 5]) * inv),
                                pack_bf16x2(__uint_as_float(ov[8 * v + 6]) * inv, __uint_as_float(ov[8 * v + 7]) * inv));
        }
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

bool prefill_pingpong_ok(const PagedAttnArgs& a) {
  const int G = a.n_kv_heads > 0 ? a.n_q_heads / a.n_kv_heads : 0;
  return G > 0 && G % 2 == 0 && a.n_q_heads % 2 == 0;
}

namespace {
// Softmax variants (exp on the FMA pipe, integer bf16 packing), picked with set_prefill_kernel:
// mode 1 = the default variant, 10 + i = variant i of this table.
using PrefillKernel = void (*)(CUtensorMap, CUtensorMap, PagedAttnArgs);
const PrefillKernel kVariants[] = {
    prefill_pingpong_kernel<0, false>, prefill_pingpong_kernel<0, true>, prefill_pingpong_kernel<4, false>,
    prefill_pingpong_kernel<4, true>,  prefill_pingpong_kernel<3, true>, prefill_pingpong_kernel<2, true>,
};
constexpr int kDefaultVariant = 0;  // measured fastest overall: MUFU exp, converter packing
int g_variant = kDefaultVariant;
}  // namespace

void set_prefill_variant(int v) {
  g_variant = (v >= 0 && v < static_cast<int>(sizeof(kVariants) / sizeof(kVariants[0]))) ? v : kDefaultVariant;
}

int prefill_trace_enable(int on) { return cudaMemcpyToSymbol(g_pp_trace_on, &on, sizeof(int)); }

int prefill_trace_read(long long* host, int n) {
  if (n > kTraceSlots) n = kTraceSlots;
  return cudaMemcpyFromSymbol(host, g_pp_trace, n * sizeof(long long));
}

int paged_prefill_pingpong(const PagedAttnArgs& a, int64_t q_rows, cudaStream_t stream) {
  if (a.num_tiles <= 0) return 0;
  if (!prefill_pingpong_ok(a)) return -1;
  if (a.q_stride % 8 || (reinterpret_cast<uintptr_t>(a.q) & 15)) return -2;
  if (a.out_stride % 8 || (reinterpret_cast<uintptr_t>(a.out) & 15)) return -2;
  CUtensorMap kvmap, qmap;
  const int64_t rows = a.num_blocks * a.num_layers * 2 * a.n_kv_heads * 16;
  if (rows >= (int64_t(1) << 31)) return -3;
  if (!make_bf16_map(&kvmap, a.arena, rows, 128, 128, 16, 64)) return -4;
  if (!make_bf16_map(&qmap, a.q, q_rows, static_cast<int64_t>(a.n_q_heads) * 128, a.q_stride, 128, 64)) return -5;
  const PrefillKernel kern = kVariants[g_variant];
  if (int e = ensure_smem_attr(reinterpret_cast<const void*>(kern), kSmem)) return e;
  dim3 grid(a.num_tiles, a.n_q_heads / 2);
  kern<<<grid, kThreads, kSmem, stream>>>(kvmap, qmap, a);
  return cudaGetLastError();
}

}  // namespace lakeb
