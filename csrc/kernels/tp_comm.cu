// Tensor-parallel collectives fused into the kernels around them.
//
// The residual stream of a tensor-parallel group is split by rows. Between a
// row-parallel GEMM (o_proj / down_proj, whose epilogue already pushed each
// partial row to the row's owner over NVLink, see kEpiRSPush) and the next
// column-parallel GEMM (qkv / gate_up / lm_head, which waits per row shard
// before its TMA loads), one kernel per rank does, for every owned row:
//
//   reduce-scatter completion  h += sum over ranks of the pushed partials
//   residual + RMSNorm         y = rmsnorm(h) * w
//   all-gather push            y -> every rank's GEMM input (P2P stores)
//
// so each NVLink byte crosses once and no separate collective runs.
// tp_argmax_combine closes a vocab-parallel lm_head: every rank's argmax
// epilogue leaves 64-bit (score, index) keys; the max over ranks is the token.
//
// All waits are bounded (2 s); on time-out the status word records
// kErrTimeoutFlag and the kernel returns without signalling.
#include "common.cuh"
#include "lakeb_kernels.h"

namespace lakeb {
namespace {

constexpr int kNormThreads = 128;

template <int EPT>
struct Vec {  // EPT bf16 values per thread, loaded as 16-byte (or smaller) chunks
  static constexpr int kChunk = EPT >= 8 ? 8 : EPT;
  static constexpr int kChunks = EPT / kChunk;
};

template <int N>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* src, float* v) {
  if constexpr (N == 8) {
    uint4 u = *reinterpret_cast<const uint4*>(src);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else if constexpr (N == 4) {
    uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
    float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src));
    v[0] = f.x;
    v[1] = f.y;
  }
}

template <int N>
__device__ __forceinline__ void store_bf16(__nv_bfloat16* dst, const float* v) {
  if constexpr (N == 8) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(dst) = u;
  } else if constexpr (N == 4) {
    uint2 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    *reinterpret_cast<uint2*>(dst) = u;
  } else {
    *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(v[0], v[1]);
  }
}

__device__ __forceinline__ float block_sum(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) red[w] = x;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

template <int EPT>
__global__ void __launch_bounds__(kNormThreads, 8) tp_norm_push_kernel(const TPNormArgs a) {
  using V = Vec<EPT>;
  __shared__ float red[kNormThreads / 32];
  __shared__ int ok_s;
  const int tid = threadIdx.x;

  if (blockIdx.x == 0 && a.reset_ptr) {
    for (int i = tid; i < a.reset_n; i += kNormThreads) a.reset_ptr[i] = 0ull;
  }
  if (tid == 0) {
    bool ok = true;
    if (a.recv) {
      const unsigned long long target = (a.rs_base ? *a.rs_base : 0ull) + a.rs_off;
      for (int s = 0; s < a.world && ok; ++s) ok = wait_counter(a.rs_cnt + s, target, nullptr, a.status);
    }
    ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;

  const int col0 = tid * EPT;

  for (int row = blockIdx.x; row < a.rows_per_rank; row += gridDim.x) {
    float v[EPT];
    __nv_bfloat16* hrow = a.h + static_cast<int64_t>(row) * a.dim + col0;
#pragma unroll
    for (int c = 0; c < V::kChunks; ++c) load_bf16<V::kChunk>(hrow + c * V::kChunk, v + c * V::kChunk);
    if (a.recv) {
#pragma unroll 2
      for (int s = 0; s < a.world; ++s) {
        const __nv_bfloat16* prow =
            a.recv + (static_cast<int64_t>(s) * a.rows_per_rank + row) * a.dim + col0;
        float pv[EPT];
#pragma unroll
        for (int c = 0; c < V::kChunks; ++c) load_bf16<V::kChunk>(prow + c * V::kChunk, pv + c * V::kChunk);
#pragma unroll
        for (int j = 0; j < EPT; ++j) v[j] += pv[j];
      }
      // the residual stream is bf16, as in the unsplit model's residual epilogue
#pragma unroll
      for (int j = 0; j < EPT; ++j) v[j] = __bfloat162float(__float2bfloat16(v[j]));
      if (a.store_h) {
#pragma unroll
        for (int c = 0; c < V::kChunks; ++c) store_bf16<V::kChunk>(hrow + c * V::kChunk, v + c * V::kChunk);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) ss += v[j] * v[j];
    const float inv = rsqrtf(block_sum(ss, red) / a.dim + a.eps);
    float y[EPT];
#pragma unroll
    for (int c = 0; c < V::kChunks; ++c) load_bf16<V::kChunk>(a.w + col0 + c * V::kChunk, y + c * V::kChunk);
#pragma unroll
    for (int j = 0; j < EPT; ++j) y[j] *= v[j] * inv;
    const int g = a.rank * a.rows_per_rank + row;
    const int drow = a.row_map ? a.row_map[g] : g;
    if (drow >= 0) {
      for (int d = 0; d < a.world; ++d) {
        __nv_bfloat16* out = a.dst[d] + static_cast<int64_t>(drow) * a.dst_ld + col0;
#pragma unroll
        for (int c = 0; c < V::kChunks; ++c) store_bf16<V::kChunk>(out + c * V::kChunk, y + c * V::kChunk);
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    for (int d = 0; d < a.world; ++d)
      if (a.ag_cnt[d]) red_add_release_sys(a.ag_cnt[d] + a.rank, 1ull);
  }
}

__global__ void tp_argmax_combine_kernel(const TPPtrs amax, int world,
                                         const unsigned long long* done_cnt, const unsigned long long* base,
                                         unsigned long long off, int* out, int n, int* status) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    const unsigned long long target = (base ? *base : 0ull) + off;
    bool ok = true;
    for (int s = 0; s < world && ok; ++s) ok = wait_counter(done_cnt + s, target, nullptr, status);
    ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
    unsigned long long best = 0ull;
    for (int d = 0; d < world; ++d) {
      const unsigned long long k = ld_acquire_sys(amax.p[d] + r);
      best = k > best ? k : best;
    }
    out[r] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  }
}

}  // namespace

// Up to eight CTAs per SM, so a whole prefill shard's rows are in flight at once (each row is a
// chain of dependent loads, a block reduction and the pushes: latency-, not bandwidth-bound).
int tp_norm_grid(int rows_per_rank) {
  const int g = 8 * 148;
  return rows_per_rank < g ? (rows_per_rank > 0 ? rows_per_rank : 1) : g;
}

int tp_norm_push(const TPNormArgs& a, cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxTP || a.rows_per_rank <= 0 || !a.h || !a.w) return -1;
  if (a.dim % kNormThreads) return -2;
  const int ept = a.dim / kNormThreads;
  const int grid = tp_norm_grid(a.rows_per_rank);
  switch (ept) {
    case 2: tp_norm_push_kernel<2><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 4: tp_norm_push_kernel<4><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 8: tp_norm_push_kernel<8><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 16: tp_norm_push_kernel<16><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 32: tp_norm_push_kernel<32><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 64: tp_norm_push_kernel<64><<<grid, kNormThreads, 0, stream>>>(a); break;
    default: return -3;
  }
  return cudaGetLastError();
}

int tp_argmax_combine(const TPPtrs& amax, int world, const unsigned long long* done_cnt,
                      const unsigned long long* base, unsigned long long off, int* out, int n, int* status,
                      cudaStream_t stream) {
  if (n <= 0) return 0;
  const int threads = 256;
  int blocks = (n + threads - 1) / threads;
  if (blocks > 64) blocks = 64;
  tp_argmax_combine_kernel<<<blocks, threads, 0, stream>>>(amax, world, done_cnt, base, off, out, n, status);
  return cudaGetLastError();
}

// Step epilogue of a tensor-parallel group: base[i] += delta[i]. Waits compare counters with
// base + a within-step offset, so a captured step replays with fresh targets.
namespace {
__global__ void tp_advance_kernel(unsigned long long* base, TPDeltas d) {
  const int i = threadIdx.x;
  if (i < d.n) base[i] += d.v[i];
}
}  // namespace

int tp_advance(unsigned long long* base, const TPDeltas& d, cudaStream_t stream) {
  if (d.n <= 0) return 0;
  if (d.n > kMaxTPDeltas) return -1;
  tp_advance_kernel<<<1, 32, 0, stream>>>(base, d);
  return cudaGetLastError();
}

}  // namespace lakeb
