// Memory-bound helper kernels: RMSNorm, embedding gather, logits argmax /
// grammar bitmask, chain-reject verification for speculative decoding, and the
// KV page mover used for tier promotion/demotion and peer (NVLink) transfers.
//
// Reference parity:
//   RMSNorm / q-k norm   python/lake/engine/model_executor/models/qwen/qwen3.py:34-43,120-121
//   embedding            qwen3.py:166-172
//   greedy / bitmask     python/lake/engine/sample/greedy.py:8-15, sample/grammar.py:13-20
//   chain reject         python/lake/engine/sample/reject.py:12-33
//   page moves           docs/architecture/kv-cache-pool.md:245-247 (layout transform, design only)
#include <math_constants.h>

#include "common.cuh"
#include "lakeb_kernels.h"

namespace lakeb {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row; each lane handles 8-element vectors strided by 256 elements.
__global__ void rmsnorm_warp_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, const __nv_bfloat16* __restrict__ w,
                                    __nv_bfloat16* __restrict__ out, int64_t so, int rows, int dim, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + row * sx;
  __nv_bfloat16* orow = out + row * so;
  constexpr int kMaxVec = 8;  // dim <= 8 * 256 = 2048 kept in registers
  uint4 buf[kMaxVec];
  float ss = 0.f;
  const int nvec = dim / 8;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = lane + i * 32;
    if (v < nvec) {
      buf[i] = reinterpret_cast<const uint4*>(xr)[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&buf[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / dim + eps);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = lane + i * 32;
    if (v < nvec) {
      const uint4 wv = reinterpret_cast<const uint4*>(w)[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&buf[i]);
      const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&wv);
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        float2 g = __bfloat1622float2(hw[j]);
        op[j] = pack_bf16x2(f.x * inv * g.x, f.y * inv * g.y);
      }
      reinterpret_cast<uint4*>(orow)[v] = o;
    }
  }
}

// One CTA (256 threads) per row for wide rows (dim > 2048), two passes over x.
__global__ void rmsnorm_cta_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ out, int64_t so, int dim, float eps) {
  __shared__ float red[8];
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * sx;
  __nv_bfloat16* orow = out + row * so;
  const int nvec = dim / 8;
  float ss = 0.f;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(xr)[v];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / dim + eps);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(xr)[v];
    const uint4 wv = reinterpret_cast<const uint4*>(w)[v];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      float2 g = __bfloat1622float2(hw[j]);
      op[j] = pack_bf16x2(f.x * inv * g.x, f.y * inv * g.y);
    }
    reinterpret_cast<uint4*>(orow)[v] = o;
  }
}

__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int n, int dim, int vocab, int* status) {
  const int row = blockIdx.x;
  if (row >= n) return;
  int id = ids[row];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) record_error(status, kErrBounds);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<int64_t>(id) * dim);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * dim);
  for (int v = threadIdx.x; v < dim / 8; v += blockDim.x) dst[v] = src[v];
}

// Argmax over fp32 logits rows (optionally bitmask-filtered). One CTA per row.
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t stride, int vocab,
                              const uint32_t* __restrict__ bitmask, int words, int* __restrict__ out) {
  __shared__ unsigned long long red[32];
  const int row = blockIdx.x;
  const float* lr = logits + row * stride;
  unsigned long long best = 0ull;
  for (int c = threadIdx.x; c < vocab; c += blockDim.x) {
    if (bitmask && !((bitmask[static_cast<int64_t>(row) * words + (c >> 5)] >> (c & 31)) & 1u)) continue;
    const unsigned long long key = (static_cast<unsigned long long>(float_order_key(lr[c])) << 32) |
                                   static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(c));
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (threadIdx.x == 0) out[row] = best ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull)) : -1;
  }
}

__global__ void unpack_argmax_kernel(const unsigned long long* __restrict__ keys, int* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const unsigned long long k = keys[i];
    out[i] = k ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull)) : -1;
  }
}

__global__ void apply_bitmask_kernel(float* __restrict__ logits, int64_t stride, int vocab,
                                     const uint32_t* __restrict__ bitmask, int words) {
  const int row = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= vocab) return;
  if (!((bitmask[static_cast<int64_t>(row) * words + (c >> 5)] >> (c & 31)) & 1u))
    logits[row * stride + c] = -CUDART_INF_F;
}

// Greedy chain verification: for each request, accept draft tokens while they
// match the target argmax, then emit the target token at the first mismatch
// (or the bonus token after a fully accepted chain).
__global__ void chain_reject_kernel(const int* __restrict__ draft, const int* __restrict__ draft_off,
                                    const int* __restrict__ target, const int* __restrict__ target_off,
                                    int* __restrict__ out, int* __restrict__ out_len, int out_stride, int nreq) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nreq) return;
  const int d0 = draft_off[r], d1 = draft_off[r + 1];
  const int t0 = target_off[r];
  int n = 0;
  for (int i = 0; i < d1 - d0; ++i) {
    const int t = target[t0 + i];
    out[r * out_stride + n++] = t;
    if (t != draft[d0 + i]) {
      out_len[r] = n;
      return;
    }
  }
  out[r * out_stride + n++] = target[t0 + (d1 - d0)];
  out_len[r] = n;
}

// Copy whole pages: dst_base[dst_ids[i]] <- src_base[src_ids[i]], page_bytes each.
// Either side may be a peer GPU's memory mapped into this context.
__global__ void page_copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, const int64_t* __restrict__ src_ids,
                                 const int64_t* __restrict__ dst_ids, int64_t page_bytes, int64_t sub_off, int64_t sub_bytes,
                                 int64_t src_pages, int64_t dst_pages, int* status) {
  const int64_t p = blockIdx.y;
  const int64_t si = src_ids[p], di = dst_ids[p];
  if (!in_bounds(si >= 0 && di >= 0 && (src_pages <= 0 || si < src_pages) && (dst_pages <= 0 || di < dst_pages),
                 status))
    return;
  const uint4* s = reinterpret_cast<const uint4*>(src + si * page_bytes + sub_off);
  uint4* d = reinterpret_cast<uint4*>(dst + di * page_bytes + sub_off);
  const int64_t nvec = sub_bytes / 16;
  for (int64_t v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += static_cast<int64_t>(gridDim.x) * blockDim.x)
    d[v] = s[v];
}

// Overlapped scheduling: a token id < 0 names a token the previous step sampled on the device
// (-1 - its sample index); resolve it from that step's output before the embedding reads it.
__global__ void resolve_tokens_kernel(int* __restrict__ ids, const int* __restrict__ prev, int n, int n_prev) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int v = ids[i];
    if (v < 0) {
      const int j = -1 - v;
      ids[i] = j < n_prev ? prev[j] : 0;
    }
  }
}

}  // namespace

int rmsnorm_bf16(const __nv_bfloat16* x, int64_t sx, const __nv_bfloat16* w, __nv_bfloat16* out, int64_t so, int rows,
                 int dim, float eps, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (dim % 8 || sx % 8 || so % 8) return -1;
  if (dim <= 2048) {
    const int warps = 4;
    rmsnorm_warp_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>(x, sx, w, out, so, rows, dim, eps);
  } else {
    rmsnorm_cta_kernel<<<rows, 256, 0, stream>>>(x, sx, w, out, so, dim, eps);
  }
  return cudaGetLastError();
}

int embedding_bf16(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int n, int dim, int vocab,
                   int* status, cudaStream_t stream) {
  if (n <= 0) return 0;
  if (dim % 8) return -1;
  embedding_kernel<<<n, 128, 0, stream>>>(ids, table, out, n, dim, vocab, status);
  return cudaGetLastError();
}

int argmax_f32(const float* logits, int64_t stride, int rows, int vocab, const uint32_t* bitmask, int words, int* out,
               cudaStream_t stream) {
  if (rows <= 0) return 0;
  argmax_kernel<<<rows, 512, 0, stream>>>(logits, stride, vocab, bitmask, words, out);
  return cudaGetLastError();
}

int unpack_argmax(const unsigned long long* keys, int* out, int n, cudaStream_t stream) {
  if (n <= 0) return 0;
  unpack_argmax_kernel<<<(n + 255) / 256, 256, 0, stream>>>(keys, out, n);
  return cudaGetLastError();
}

int apply_bitmask_f32(float* logits, int64_t stride, int rows, int vocab, const uint32_t* bitmask, int words,
                      cudaStream_t stream) {
  if (rows <= 0) return 0;
  apply_bitmask_kernel<<<dim3((vocab + 255) / 256, rows), 256, 0, stream>>>(logits, stride, vocab, bitmask, words);
  return cudaGetLastError();
}

int chain_reject(const int* draft, const int* draft_off, const int* target, const int* target_off, int* out,
                 int* out_len, int out_stride, int nreq, cudaStream_t stream) {
  if (nreq <= 0) return 0;
  chain_reject_kernel<<<(nreq + 127) / 128, 128, 0, stream>>>(draft, draft_off, target, target_off, out, out_len,
                                                               out_stride, nreq);
  return cudaGetLastError();
}

int page_copy(const void* src, void* dst, const int64_t* src_ids, const int64_t* dst_ids, int n, int64_t page_bytes,
              int64_t sub_off, int64_t sub_bytes, cudaStream_t stream, int64_t src_pages, int64_t dst_pages,
              int* status) {
  if (n <= 0) return 0;
  if (page_bytes % 16 || sub_off % 16 || sub_bytes % 16) return -1;
  const int64_t nvec = sub_bytes / 16;
  int gx = static_cast<int>((nvec + 255) / 256);
  if (gx > 64) gx = 64;
  page_copy_kernel<<<dim3(gx, n), 256, 0, stream>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst),
                                                    src_ids, dst_ids, page_bytes, sub_off, sub_bytes, src_pages,
                                                    dst_pages, status);
  return cudaGetLastError();
}

bool debug_checks_enabled() {
#ifdef LAKEB_DEBUG_CHECKS
  return true;
#else
  return false;
#endif
}

int resolve_tokens(int* ids, const int* prev, int n, int n_prev, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int threads = 256;
  int blocks = (n + threads - 1) / threads;
  if (blocks > 64) blocks = 64;
  resolve_tokens_kernel<<<blocks, threads, 0, stream>>>(ids, prev, n, n_prev);
  return cudaGetLastError();
}

}  // namespace lakeb
