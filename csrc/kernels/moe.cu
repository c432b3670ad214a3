// Mixture-of-experts routing, dispatch and combine for sm_100a.
//
// moe_dispatch: per token, top-k of the router logits (softmax over the k
// chosen logits gives the combine weights), then the token's hidden row is
// copied into the segment of each chosen expert: gathered[e_local*cap + pos]
// with pos from an atomic counter of that expert. With expert parallelism the
// expert lives on another GPU: the counter is that GPU's (a system-scope
// atomic over NVLink), the row is stored straight into its gathered buffer
// (P2P stores) together with the slot it must come back to, and every CTA
// finishes by adding 1 to the destination's dispatch counter. One kernel is
// both the router's top-k and the all-to-all dispatch.
//
// The grouped expert GEMMs (gemm_tcgen05.cu, groups = experts on this GPU)
// run over the gathered rows; the down projection's scatter epilogue stores
// each result row back into its token's slot at the token's GPU.
// moe_combine then adds the weighted expert outputs to the residual stream.
//
// Reference parity: the reference has no MoE execution; its model registry
// names Qwen3 MoE shells only (python/lake/engine/model_executor/models/qwen/).
#include "common.cuh"
#include "lakeb_kernels.h"

namespace lakeb {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxTopK = 4;

__global__ void __launch_bounds__(kThreads) moe_dispatch_kernel(const MoEDispatchArgs a) {
  __shared__ int dst_rank[kMaxTopK], dst_row[kMaxTopK];
  const int tid = threadIdx.x;
  const int vecs = a.dim / 8;  // 16-byte vectors per row
  for (int t = blockIdx.x; t < a.M; t += gridDim.x) {
    if (tid == 0) {
      const float* lg = a.logits + static_cast<int64_t>(t) * a.ld_logits;
      float val[kMaxTopK];
      int idx[kMaxTopK];
      uint32_t taken = 0;
      for (int j = 0; j < a.top_k; ++j) {
        float best = -INFINITY;
        int bi = 0;
        for (int e = 0; e < a.n_experts; ++e) {
          const float v = lg[e];
          if (!((taken >> e) & 1u) && v > best) {
            best = v;
            bi = e;
          }
        }
        taken |= 1u << bi;
        val[j] = best;
        idx[j] = bi;
      }
      float sum = 0.f, w[kMaxTopK];
      for (int j = 0; j < a.top_k; ++j) {
        w[j] = __expf(val[j] - val[0]);
        sum += w[j];
      }
      for (int j = 0; j < a.top_k; ++j) {
        a.weights[static_cast<int64_t>(t) * a.top_k + j] = w[j] / sum;
        const int d = idx[j] / a.experts_per_rank;
        const int le = idx[j] - d * a.experts_per_rank;
        const int pos = atomicAdd_system(a.count[d] + le, 1);
        if (pos >= a.cap) {
          record_error(a.status, kErrBounds);
          dst_rank[j] = -1;
          continue;
        }
        const int row = le * a.cap + pos;
        dst_rank[j] = d;
        dst_row[j] = row;
        a.row_slot[d][row] = t * a.top_k + j;
        if (a.row_rank[d]) a.row_rank[d][row] = a.rank;
      }
    }
    __syncthreads();
    const uint4* src = reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(t) * a.dim);
    for (int j = 0; j < a.top_k; ++j) {
      const int d = dst_rank[j];
      if (d < 0) continue;
      uint4* dst = reinterpret_cast<uint4*>(a.gathered[d] + static_cast<int64_t>(dst_row[j]) * a.dim);
      for (int v = tid; v < vecs; v += kThreads) dst[v] = src[v];
    }
    __syncthreads();
  }
  if (a.done_cnt[0]) {
    __threadfence_system();
    __syncthreads();
    if (tid == 0)
      for (int d = 0; d < a.world; ++d) red_add_release_sys(a.done_cnt[d] + a.rank, 1ull);
  }
}

__global__ void __launch_bounds__(kThreads)
    moe_combine_kernel(__nv_bfloat16* h, const __nv_bfloat16* comb, const float* weights, int M, int dim, int top_k,
                       const unsigned long long* wait_cnt, int wait_n, unsigned long long target, int* status,
                       const unsigned long long* wait_base) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    const unsigned long long goal = (wait_base ? *wait_base : 0ull) + target;
    for (int s = 0; s < wait_n && ok; ++s) ok = wait_counter(wait_cnt + s, goal, nullptr, status);
    ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;
  const int pairs = dim / 2;
  for (int t = blockIdx.x; t < M; t += gridDim.x) {
    __nv_bfloat162* hr = reinterpret_cast<__nv_bfloat162*>(h + static_cast<int64_t>(t) * dim);
    for (int c = threadIdx.x; c < pairs; c += kThreads) {
      float2 acc = __bfloat1622float2(hr[c]);
      for (int j = 0; j < top_k; ++j) {
        const float w = weights[static_cast<int64_t>(t) * top_k + j];
        const __nv_bfloat162* cr =
            reinterpret_cast<const __nv_bfloat162*>(comb + (static_cast<int64_t>(t) * top_k + j) * dim);
        const float2 v = __bfloat1622float2(cr[c]);
        acc.x += w * v.x;
        acc.y += w * v.y;
      }
      hr[c] = __floats2bfloat162_rn(acc.x, acc.y);
    }
  }
}

__global__ void wait_counters_kernel(const unsigned long long* cnt, int n, unsigned long long target, int* status,
                                     unsigned long long limit_ns, const unsigned long long* base) {
  const unsigned long long goal = (base ? *base : 0ull) + target;
  for (int s = 0; s < n; ++s)
    if (!wait_counter(cnt + s, goal, nullptr, status, limit_ns)) return;
}

}  // namespace

int moe_dispatch(const MoEDispatchArgs& a, cudaStream_t stream) {
  if (a.M < 0 || a.top_k < 1 || a.top_k > kMaxTopK || a.n_experts < a.top_k || a.n_experts > 32) return -1;
  if (a.dim % 8 || a.world < 1 || a.world > kMaxTP || a.experts_per_rank * a.world != a.n_experts) return -2;
  for (int d = 0; d < a.world; ++d)
    if (!a.gathered[d] || !a.row_slot[d] || !a.count[d]) return -3;
  moe_dispatch_kernel<<<kMoEDispatchGrid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

int moe_combine(__nv_bfloat16* h, const __nv_bfloat16* comb, const float* weights, int M, int dim, int top_k,
                const unsigned long long* wait_cnt, int wait_n, unsigned long long wait_target, int* status,
                cudaStream_t stream, const unsigned long long* wait_base) {
  if (M <= 0) return 0;
  if (dim % 2) return -1;
  const int grid = M < 1184 ? M : 1184;
  moe_combine_kernel<<<grid, kThreads, 0, stream>>>(h, comb, weights, M, dim, top_k, wait_cnt, wait_n, wait_target,
                                                    status, wait_base);
  return cudaGetLastError();
}

int wait_counters(const unsigned long long* cnt, int n, unsigned long long target, int* status,
                  cudaStream_t stream, unsigned long long limit_ns, const unsigned long long* base) {
  wait_counters_kernel<<<1, 1, 0, stream>>>(cnt, n, target, status, limit_ns ? limit_ns : kWaitLimitNs, base);
  return cudaGetLastError();
}

}  // namespace lakeb
