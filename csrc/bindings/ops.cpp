// Python bindings for the sm_100a kernels (module lake_b200._C).
// Every op runs on the caller's current CUDA stream and raises on a launch or
// argument error, so a missing or failing kernel is never silently replaced.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "../kernels/lakeb_kernels.h"

namespace {

using lakeb::GemmArgs;
using lakeb::KVArenaView;
using lakeb::PagedAttnArgs;

#define LAKEB_CHECK_RC(rc, what) TORCH_CHECK((rc) == 0, what, " failed with code ", (rc))

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

const __nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bfm(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

void check_aligned(const at::Tensor& t, const char* name, int64_t bytes = 16) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % bytes == 0, name, " must be ", bytes, "-byte aligned");
}

// Kernels move rows with 16-byte vectors: base 16-byte aligned, row stride a multiple of 8 elements.
void check_bf16_2d(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit inner stride");
  check_aligned(t, name);
  TORCH_CHECK(t.size(0) <= 1 || t.stride(0) % 8 == 0, name, " row stride must be a multiple of 8 elements");
}

int* status_ptr(const c10::optional<at::Tensor>& st) {
  if (!st.has_value()) return nullptr;
  TORCH_CHECK(st->scalar_type() == at::kInt && st->is_cuda(), "status must be an int32 CUDA tensor");
  return st->data_ptr<int>();
}

// w is bf16 [N, K], or fp8 e4m3 bytes (uint8 [N, K]) with w_scale fp32 [ceil(N/128), ceil(K/128)].
GemmArgs base_args(const at::Tensor& a, const at::Tensor& w, const c10::optional<at::Tensor>& w_scale = {}) {
  check_bf16_2d(a, "A");
  TORCH_CHECK(a.size(1) == w.size(1), "K mismatch: ", a.size(1), " vs ", w.size(1));
  GemmArgs g;
  g.A = bf(a);
  g.lda = a.stride(0);
  if (w.scalar_type() == at::kByte) {
    TORCH_CHECK(w.is_cuda() && w.dim() == 2 && w.stride(1) == 1, "fp8 weight must be a 2-D uint8 CUDA tensor");
    check_aligned(w, "W8");
    TORCH_CHECK(w_scale.has_value() && w_scale->scalar_type() == at::kFloat && w_scale->dim() == 2 &&
                    w_scale->is_contiguous() && w_scale->size(0) == (w.size(0) + 127) / 128 &&
                    w_scale->size(1) == (w.size(1) + 127) / 128,
                "fp8 weight needs fp32 block scales [ceil(N/128), ceil(K/128)]");
    g.B8 = w.data_ptr<uint8_t>();
    g.ldb8 = w.stride(0);
    g.b_scale = w_scale->data_ptr<float>();
    g.b_scale_ld = static_cast<int>(w_scale->size(1));
  } else {
    check_bf16_2d(w, "W");
    g.B = bf(w);
    g.ldb = w.stride(0);
  }
  g.M = static_cast<int>(a.size(0));
  g.N = static_cast<int>(w.size(0));
  g.K = static_cast<int>(a.size(1));
  return g;
}

// Pinned host ranges registered as KV arenas (register_host_arena). The pinned check runs once,
// at registration: under CUDA-graph capture the runtime's pointer query is not available, so a
// per-call is_pinned() would reject the arena inside a captured step.
std::mutex g_host_mu;
std::vector<std::pair<uintptr_t, size_t>> g_host_arenas;

void register_host_arena(const at::Tensor& t) {
  TORCH_CHECK(!t.is_cuda() && t.is_pinned() && t.is_contiguous(), "a host KV arena must be contiguous pinned memory");
  std::lock_guard<std::mutex> lk(g_host_mu);
  g_host_arenas.emplace_back(reinterpret_cast<uintptr_t>(t.data_ptr()), t.nbytes());
}

void unregister_host_arena(const at::Tensor& t) {
  std::lock_guard<std::mutex> lk(g_host_mu);
  const auto p = reinterpret_cast<uintptr_t>(t.data_ptr());
  for (auto it = g_host_arenas.begin(); it != g_host_arenas.end(); ++it)
    if (it->first == p) {
      g_host_arenas.erase(it);
      return;
    }
}

bool is_registered_host(const at::Tensor& t) {
  const auto p = reinterpret_cast<uintptr_t>(t.data_ptr());
  const size_t n = t.nbytes();
  std::lock_guard<std::mutex> lk(g_host_mu);
  for (const auto& r : g_host_arenas)
    if (p >= r.first && p + n <= r.first + r.second) return true;
  return false;
}

// `host_ok`: the arena may be registered pinned host memory, which the GPU reaches through its
// unified address (the kernel-side write-behind of decode K/V into the host tier).
KVArenaView arena_view(const at::Tensor& arena, int64_t layer, bool host_ok = false) {
  TORCH_CHECK(arena.is_cuda() || (host_ok && is_registered_host(arena)),
              "arena must be device memory (or, as a second K/V target, pinned host memory registered with "
              "register_host_arena)");
  TORCH_CHECK(arena.scalar_type() == at::kBFloat16 && arena.dim() == 6 && arena.is_contiguous(),
              "arena must be a contiguous bf16 [blocks, layers, 2, kv_heads, block, 128] tensor");
  TORCH_CHECK(arena.size(5) == 128, "head_dim must be 128");
  check_aligned(arena, "arena");
  KVArenaView v;
  v.base = bfm(arena);
  v.block_stride = arena.stride(0);
  v.layer_offset = layer * arena.stride(1);
  v.kv_stride = arena.stride(2);
  v.head_stride = arena.stride(3);
  v.block_size = static_cast<int>(arena.size(4));
  v.num_slots = arena.size(0) * arena.size(4);
  return v;
}

template <class T>
T* ptr_of(const py::handle& o) {
  return reinterpret_cast<T*>(static_cast<uintptr_t>(o.cast<int64_t>()));
}

// Tensor-parallel fusion arguments (lake_b200.parallel.tp builds the dict):
// world, rank, rows_per_rank, m_rot, ag_cnt, ag_off, rs_recv[], rs_cnt[], done_cnt[], col_offset.
void apply_tp(GemmArgs& g, const c10::optional<py::dict>& tp) {
  if (!tp.has_value()) return;
  const py::dict& d = *tp;
  auto& t = g.tp;
  t.world = d["world"].cast<int>();
  TORCH_CHECK(t.world >= 1 && t.world <= lakeb::kMaxTP, "tp world out of range");
  t.rank = d["rank"].cast<int>();
  t.rows_per_rank = d["rows_per_rank"].cast<int>();
  if (d.contains("m_rot")) t.m_rot = d["m_rot"].cast<int>();
  if (d.contains("ag_cnt")) {
    t.ag_cnt = ptr_of<const unsigned long long>(d["ag_cnt"]);
    t.ag_off = d["ag_off"].cast<unsigned long long>();
    if (d.contains("ag_all")) t.ag_all = d["ag_all"].cast<int>();
    if (d.contains("ag_base") && !d["ag_base"].is_none()) t.ag_base = ptr_of<const unsigned long long>(d["ag_base"]);
  }
  auto fill = [&](const char* key, auto* arr) {
    if (!d.contains(key)) return;
    py::list l = d[key];
    TORCH_CHECK(static_cast<int>(l.size()) == t.world, key, " needs one pointer per rank");
    using P = std::remove_reference_t<decltype(arr[0])>;  // element pointer type
    for (int i = 0; i < t.world; ++i) arr[i] = reinterpret_cast<P>(static_cast<uintptr_t>(l[i].cast<int64_t>()));
  };
  fill("rs_recv", t.rs_recv);
  fill("rs_cnt", t.rs_cnt);
  fill("done_cnt", t.done_cnt);
  if (d.contains("col_offset")) t.col_offset = d["col_offset"].cast<int>();
}

// out = a @ w.T  (bf16 out) or fp32 out
void linear(const at::Tensor& a, const at::Tensor& w, at::Tensor& out, c10::optional<at::Tensor> status,
            int64_t max_ctas, c10::optional<at::Tensor> w_scale) {
  GemmArgs g = base_args(a, w, w_scale);
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(0) == a.size(0) && out.size(1) == w.size(0), "out shape");
  check_aligned(out, "out");
  TORCH_CHECK(out.size(0) <= 1 || out.stride(0) % 8 == 0, "out row stride must be a multiple of 8 elements");
  g.C = out.data_ptr();
  g.ldc = out.stride(0);
  g.status = status_ptr(status);
  g.max_ctas = static_cast<int>(max_ctas);
  int epi = out.scalar_type() == at::kFloat ? lakeb::kEpiStoreF32 : lakeb::kEpiStoreBf16;
  TORCH_CHECK(out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16, "out dtype");
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, epi, cur_stream()), "linear");
}

// out = residual + a @ w.T   (residual may be out itself)
void linear_residual(const at::Tensor& a, const at::Tensor& w, const at::Tensor& residual, at::Tensor& out,
                     c10::optional<at::Tensor> status, c10::optional<at::Tensor> w_scale) {
  GemmArgs g = base_args(a, w, w_scale);
  check_bf16_2d(out, "out");
  check_bf16_2d(residual, "residual");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == w.size(0) && residual.sizes() == out.sizes(), "shapes");
  g.C = out.data_ptr();
  g.ldc = out.stride(0);
  g.R = bf(residual);
  g.ldr = residual.stride(0);
  g.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, lakeb::kEpiResidual, cur_stream()), "linear_residual");
}

// out[:, j] = silu(gate_j) * up_j with w rows interleaved per 256-row tile: [gate 128 | up 128]
void linear_swiglu(const at::Tensor& a, const at::Tensor& w, at::Tensor& out, c10::optional<at::Tensor> status,
                   c10::optional<py::dict> tp, c10::optional<at::Tensor> w_scale) {
  GemmArgs g = base_args(a, w, w_scale);
  apply_tp(g, tp);
  check_bf16_2d(out, "out");
  TORCH_CHECK(w.size(0) % 256 == 0, "gate_up rows must be a multiple of 256");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) * 2 == w.size(0), "out shape");
  g.C = out.data_ptr();
  g.ldc = out.stride(0);
  g.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, lakeb::kEpiSwiGLU, cur_stream()), "linear_swiglu");
}

// q_out = RoPE(q); K (RoPE) and V written into the paged arena at `slots` (and
// the peer arena at `peer_slots` when given).
void linear_qkv(const at::Tensor& a, const at::Tensor& w, at::Tensor& q_out, const at::Tensor& rope_cs,
                const at::Tensor& positions, const at::Tensor& slots, const at::Tensor& arena, int64_t layer,
                int64_t n_q_heads, int64_t n_kv_heads, c10::optional<at::Tensor> peer_arena,
                c10::optional<at::Tensor> peer_slots, c10::optional<at::Tensor> status, c10::optional<py::dict> tp,
                c10::optional<at::Tensor> q_norm, c10::optional<at::Tensor> k_norm, double qk_eps, c10::optional<at::Tensor> w_scale) {
  GemmArgs g = base_args(a, w, w_scale);
  apply_tp(g, tp);
  if (q_norm.has_value() && k_norm.has_value()) {
    TORCH_CHECK(q_norm->numel() == 128 && k_norm->numel() == 128 && q_norm->scalar_type() == at::kBFloat16 &&
                    k_norm->scalar_type() == at::kBFloat16 && q_norm->is_contiguous() && k_norm->is_contiguous(),
                "q_norm / k_norm must be bf16 [128]");
    g.q_norm_w = bf(*q_norm);
    g.k_norm_w = bf(*k_norm);
    g.qk_eps = static_cast<float>(qk_eps);
  }
  check_bf16_2d(q_out, "q_out");
  TORCH_CHECK(q_out.size(0) == a.size(0) && q_out.size(1) == n_q_heads * 128, "q_out shape");
  TORCH_CHECK(rope_cs.scalar_type() == at::kFloat && rope_cs.is_contiguous() && rope_cs.dim() == 3 &&
                  rope_cs.size(1) == 64 && rope_cs.size(2) == 2,
              "rope_cs must be fp32 [max_pos, 64, 2]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.numel() >= a.size(0), "positions int32");
  TORCH_CHECK(slots.scalar_type() == at::kLong && slots.numel() >= a.size(0), "slots int64");
  g.C = q_out.data_ptr();
  g.ldc = q_out.stride(0);
  g.rope_cs = reinterpret_cast<const float2*>(rope_cs.data_ptr<float>());
  g.positions = positions.data_ptr<int>();
  g.slots = slots.data_ptr<int64_t>();
  g.kv = arena_view(arena, layer);
  g.n_q_heads = static_cast<int>(n_q_heads);
  g.n_kv_heads = static_cast<int>(n_kv_heads);
  if (peer_arena.has_value() && peer_slots.has_value()) {
    g.peer_kv = arena_view(*peer_arena, layer, /*host_ok=*/true);
    TORCH_CHECK(peer_slots->scalar_type() == at::kLong, "peer_slots int64");
    g.peer_slots = peer_slots->data_ptr<int64_t>();
  }
  g.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, lakeb::kEpiQKV, cur_stream()), "linear_qkv");
}

// amax[row] = packed (value, index) of the row's argmax of a @ w.T (bitmask-filtered).
void linear_argmax(const at::Tensor& a, const at::Tensor& w, at::Tensor& amax, c10::optional<at::Tensor> bitmask,
                   c10::optional<at::Tensor> status, c10::optional<py::dict> tp, c10::optional<at::Tensor> w_scale) {
  GemmArgs g = base_args(a, w, w_scale);
  apply_tp(g, tp);
  TORCH_CHECK(amax.scalar_type() == at::kLong && amax.numel() >= a.size(0) && amax.is_contiguous(), "amax int64");
  check_aligned(amax, "amax", 8);
  amax.zero_();
  g.amax = reinterpret_cast<unsigned long long*>(amax.data_ptr<int64_t>());
  if (bitmask.has_value()) {
    TORCH_CHECK(bitmask->scalar_type() == at::kInt && bitmask->dim() == 2 && bitmask->is_contiguous(), "bitmask");
    g.bitmask = reinterpret_cast<const uint32_t*>(bitmask->data_ptr<int>());
    g.bitmask_words = static_cast<int>(bitmask->size(1));
  }
  g.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, lakeb::kEpiArgmax, cur_stream()), "linear_argmax");
}

// GEMM -> reduce-scatter: each partial row of a @ w.T goes to its owner rank's receive buffer.
void linear_rs(const at::Tensor& a, const at::Tensor& w, const py::dict& tp, c10::optional<at::Tensor> status, c10::optional<at::Tensor> w_scale) {
  GemmArgs g = base_args(a, w, w_scale);
  apply_tp(g, tp);
  g.ldc = w.size(0);  // receive rows are dense [world][rows_per_rank][N]
  g.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, lakeb::kEpiRSPush, cur_stream()), "linear_rs");
}

// Reduce-scatter completion + residual + RMSNorm + all-gather push (see tp_comm.cu).
void tp_norm_push(at::Tensor& h, const at::Tensor& w, double eps, const py::dict& d, c10::optional<at::Tensor> status) {
  check_bf16_2d(h, "h");
  TORCH_CHECK(h.is_contiguous() && w.is_contiguous() && w.numel() == h.size(1), "h / w layout");
  lakeb::TPNormArgs a;
  a.world = d["world"].cast<int>();
  a.rank = d["rank"].cast<int>();
  a.rows_per_rank = d["rows_per_rank"].cast<int>();
  TORCH_CHECK(h.size(0) >= a.rows_per_rank, "h has fewer rows than rows_per_rank");
  a.dim = static_cast<int>(h.size(1));
  a.h = bfm(h);
  a.w = bf(w);
  a.eps = static_cast<float>(eps);
  if (d.contains("recv") && !d["recv"].is_none()) {
    a.recv = ptr_of<const __nv_bfloat16>(d["recv"]);
    a.rs_cnt = ptr_of<const unsigned long long>(d["rs_cnt"]);
    a.rs_off = d["rs_off"].cast<unsigned long long>();
    if (d.contains("rs_base") && !d["rs_base"].is_none()) a.rs_base = ptr_of<const unsigned long long>(d["rs_base"]);
  }
  if (d.contains("store_h")) a.store_h = d["store_h"].cast<int>();
  py::list dst = d["dst"];
  py::list cnt = d["ag_cnt"];
  TORCH_CHECK(static_cast<int>(dst.size()) == a.world && static_cast<int>(cnt.size()) == a.world, "per-rank lists");
  for (int i = 0; i < a.world; ++i) {
    a.dst[i] = ptr_of<__nv_bfloat16>(dst[i]);
    a.ag_cnt[i] = ptr_of<unsigned long long>(cnt[i]);
  }
  a.dst_ld = d["dst_ld"].cast<int64_t>();
  if (d.contains("row_map") && !d["row_map"].is_none()) a.row_map = ptr_of<const int>(d["row_map"]);
  if (d.contains("reset_ptr") && !d["reset_ptr"].is_none()) {
    a.reset_ptr = ptr_of<unsigned long long>(d["reset_ptr"]);
    a.reset_n = d["reset_n"].cast<int>();
  }
  a.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::tp_norm_push(a, cur_stream()), "tp_norm_push");
}

void tp_argmax_combine(const std::vector<int64_t>& amax_ptrs, int64_t done_cnt, int64_t off, at::Tensor& out,
                       int64_t n, c10::optional<at::Tensor> status, int64_t base) {
  TORCH_CHECK(out.scalar_type() == at::kInt && out.is_cuda() && out.numel() >= n, "out int32");
  lakeb::TPPtrs p;
  TORCH_CHECK(amax_ptrs.size() >= 1 && amax_ptrs.size() <= static_cast<size_t>(lakeb::kMaxTP), "world");
  for (size_t i = 0; i < amax_ptrs.size(); ++i)
    p.p[i] = reinterpret_cast<const unsigned long long*>(static_cast<uintptr_t>(amax_ptrs[i]));
  LAKEB_CHECK_RC(lakeb::tp_argmax_combine(p, static_cast<int>(amax_ptrs.size()),
                                           reinterpret_cast<const unsigned long long*>(done_cnt),
                                           reinterpret_cast<const unsigned long long*>(base),
                                           static_cast<unsigned long long>(off), out.data_ptr<int>(),
                                           static_cast<int>(n), status_ptr(status), cur_stream()),
                 "tp_argmax_combine");
}

// base[i] += deltas[i] on the current stream (captured into a graph with the deltas as constants).
void tp_advance(int64_t base, const std::vector<int64_t>& deltas) {
  lakeb::TPDeltas d;
  TORCH_CHECK(base != 0 && deltas.size() <= static_cast<size_t>(lakeb::kMaxTPDeltas), "tp_advance arguments");
  d.n = static_cast<int>(deltas.size());
  for (size_t i = 0; i < deltas.size(); ++i) d.v[i] = static_cast<unsigned long long>(deltas[i]);
  LAKEB_CHECK_RC(lakeb::tp_advance(reinterpret_cast<unsigned long long*>(base), d, cur_stream()), "tp_advance");
}

// Grouped expert GEMM over gathered rows: w is [groups, N, K]; rows of group g are
// a[g*group_rows, g*group_rows + group_count[g]). epi: swiglu (out [groups*group_rows, N/2])
// or scatter (each row to dst_ptrs[row_rank[row] or 0] + row_slot[row]*N).
void gemm_grouped(const at::Tensor& a, const at::Tensor& w, c10::optional<at::Tensor> out, int64_t epi,
                  const at::Tensor& group_count, int64_t group_rows, c10::optional<at::Tensor> row_slot,
                  c10::optional<at::Tensor> row_rank, std::vector<int64_t> dst_ptrs, c10::optional<py::dict> tp,
                  c10::optional<at::Tensor> status) {
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w.scalar_type() == at::kBFloat16, "w must be [G, N, K] bf16");
  const int64_t G = w.size(0), N = w.size(1), K = w.size(2);
  at::Tensor w2 = w.view({G * N, K});
  GemmArgs g = base_args(a, w2);
  g.N = static_cast<int>(N);
  g.groups = static_cast<int>(G);
  g.group_rows = static_cast<int>(group_rows);
  TORCH_CHECK(group_count.scalar_type() == at::kInt && group_count.numel() >= G, "group_count int32 [G]");
  g.group_count = group_count.data_ptr<int>();
  TORCH_CHECK(a.size(0) == G * group_rows, "a must have groups*group_rows rows");
  apply_tp(g, tp);
  if (epi == lakeb::kEpiSwiGLU) {
    TORCH_CHECK(out.has_value(), "out required");
    check_bf16_2d(*out, "out");
    TORCH_CHECK(out->size(0) == a.size(0) && out->size(1) * 2 == N && N % 256 == 0, "out shape");
    g.C = out->data_ptr();
    g.ldc = out->stride(0);
  } else if (epi == lakeb::kEpiScatter) {
    TORCH_CHECK(row_slot.has_value() && row_slot->scalar_type() == at::kInt, "row_slot int32");
    g.row_slot = row_slot->data_ptr<int>();
    if (row_rank.has_value()) g.row_rank = row_rank->data_ptr<int>();
    TORCH_CHECK(!dst_ptrs.empty() && dst_ptrs.size() <= static_cast<size_t>(lakeb::kMaxTP), "dst_ptrs");
    for (size_t i = 0; i < dst_ptrs.size(); ++i)
      g.tp.rs_recv[i] = reinterpret_cast<__nv_bfloat16*>(static_cast<uintptr_t>(dst_ptrs[i]));
    g.ldc = N;
  } else {
    TORCH_CHECK(false, "gemm_grouped: epi must be swiglu or scatter");
  }
  g.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::gemm_bf16(g, static_cast<int>(epi), cur_stream()), "gemm_grouped");
}

// Router top-k + gather into expert segments (+ all-to-all dispatch over NVLink when world > 1).
void moe_dispatch(const at::Tensor& logits, const at::Tensor& x, at::Tensor& weights, int64_t n_experts,
                  int64_t top_k, int64_t cap, int64_t world, int64_t rank, std::vector<int64_t> gathered,
                  std::vector<int64_t> row_slot, std::vector<int64_t> row_rank, std::vector<int64_t> count,
                  std::vector<int64_t> done_cnt, c10::optional<at::Tensor> status) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "logits fp32 2-D");
  check_bf16_2d(x, "x");
  TORCH_CHECK(x.is_contiguous() && weights.scalar_type() == at::kFloat && weights.is_contiguous(), "x / weights");
  lakeb::MoEDispatchArgs a;
  a.logits = logits.data_ptr<float>();
  a.ld_logits = static_cast<int>(logits.stride(0));
  a.x = bf(x);
  a.M = static_cast<int>(x.size(0));
  a.dim = static_cast<int>(x.size(1));
  a.n_experts = static_cast<int>(n_experts);
  a.top_k = static_cast<int>(top_k);
  a.cap = static_cast<int>(cap);
  a.weights = weights.data_ptr<float>();
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.experts_per_rank = static_cast<int>(n_experts / world);
  auto P = [](int64_t v) { return static_cast<uintptr_t>(v); };
  TORCH_CHECK(static_cast<int64_t>(gathered.size()) == world && static_cast<int64_t>(count.size()) == world &&
                  static_cast<int64_t>(row_slot.size()) == world, "per-rank pointer lists");
  for (int i = 0; i < world; ++i) {
    a.gathered[i] = reinterpret_cast<__nv_bfloat16*>(P(gathered[i]));
    a.row_slot[i] = reinterpret_cast<int*>(P(row_slot[i]));
    a.row_rank[i] = row_rank.empty() ? nullptr : reinterpret_cast<int*>(P(row_rank[i]));
    a.count[i] = reinterpret_cast<int*>(P(count[i]));
    a.done_cnt[i] = done_cnt.empty() ? nullptr : reinterpret_cast<unsigned long long*>(P(done_cnt[i]));
  }
  a.status = status_ptr(status);
  LAKEB_CHECK_RC(lakeb::moe_dispatch(a, cur_stream()), "moe_dispatch");
}

void moe_combine(at::Tensor& h, const at::Tensor& comb, const at::Tensor& weights, int64_t top_k, int64_t wait_cnt,
                 int64_t wait_n, int64_t target, c10::optional<at::Tensor> status, int64_t wait_base) {
  check_bf16_2d(h, "h");
  TORCH_CHECK(h.is_contiguous() && comb.is_contiguous() && comb.scalar_type() == at::kBFloat16, "layouts");
  LAKEB_CHECK_RC(lakeb::moe_combine(bfm(h), bf(comb), weights.data_ptr<float>(), static_cast<int>(h.size(0)),
                                     static_cast<int>(h.size(1)), static_cast<int>(top_k),
                                     reinterpret_cast<const unsigned long long*>(static_cast<uintptr_t>(wait_cnt)),
                                     static_cast<int>(wait_n), static_cast<unsigned long long>(target),
                                     status_ptr(status), cur_stream(),
                                     reinterpret_cast<const unsigned long long*>(static_cast<uintptr_t>(wait_base))),
                 "moe_combine");
}

void wait_counters(int64_t cnt, int64_t n, int64_t target, c10::optional<at::Tensor> status, int64_t limit_ns,
                   int64_t base) {
  LAKEB_CHECK_RC(lakeb::wait_counters(reinterpret_cast<const unsigned long long*>(static_cast<uintptr_t>(cnt)),
                                       static_cast<int>(n), static_cast<unsigned long long>(target),
                                       status_ptr(status), cur_stream(), static_cast<unsigned long long>(limit_ns),
                                       reinterpret_cast<const unsigned long long*>(static_cast<uintptr_t>(base))),
                 "wait_counters");
}

PagedAttnArgs attn_args(const at::Tensor& q, at::Tensor& out, const at::Tensor& arena, int64_t layer,
                        const at::Tensor& block_tables, const at::Tensor& seq_lens, int64_t n_q_heads,
                        int64_t n_kv_heads, double scale, c10::optional<at::Tensor> status) {
  check_bf16_2d(q, "q");
  check_bf16_2d(out, "out");
  TORCH_CHECK(arena.dim() == 6 && arena.is_contiguous() && arena.size(5) == 128 && arena.size(4) == 16,
              "arena layout");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.stride(1) == 1,
              "block_tables int32 [seqs, max_blocks]");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt, "seq_lens int32");
  PagedAttnArgs p;
  p.q = bf(q);
  p.q_stride = q.stride(0);
  p.out = bfm(out);
  p.out_stride = out.stride(0);
  p.arena = bf(arena);
  p.num_blocks = arena.size(0);
  p.num_layers = static_cast<int>(arena.size(1));
  p.layer = static_cast<int>(layer);
  TORCH_CHECK(arena.size(3) == n_kv_heads, "kv heads mismatch");
  p.n_q_heads = static_cast<int>(n_q_heads);
  p.n_kv_heads = static_cast<int>(n_kv_heads);
  p.block_tables = block_tables.data_ptr<int>();
  p.bt_stride = static_cast<int>(block_tables.stride(0));
  p.seq_lens = seq_lens.data_ptr<int>();
  p.num_seqs = static_cast<int>(seq_lens.numel());
  p.scale = static_cast<float>(scale);
  p.status = status_ptr(status);
  return p;
}

void paged_decode(const at::Tensor& q, at::Tensor& out, const at::Tensor& arena, int64_t layer,
                  const at::Tensor& block_tables, const at::Tensor& seq_lens, int64_t n_q_heads, int64_t n_kv_heads,
                  double scale, int64_t splits, c10::optional<at::Tensor> ws_o, c10::optional<at::Tensor> ws_ml,
                  c10::optional<at::Tensor> status) {
  PagedAttnArgs p = attn_args(q, out, arena, layer, block_tables, seq_lens, n_q_heads, n_kv_heads, scale, status);
  TORCH_CHECK(q.size(0) >= p.num_seqs, "one query row per sequence");
  p.splits = static_cast<int>(splits);
  if (splits > 1) {
    TORCH_CHECK(ws_o.has_value() && ws_ml.has_value(), "split-KV needs workspaces");
    const int64_t G = n_q_heads / n_kv_heads;
    TORCH_CHECK(ws_o->scalar_type() == at::kFloat && ws_o->numel() >= p.num_seqs * n_kv_heads * splits * G * 128,
                "ws_o too small");
    TORCH_CHECK(ws_ml->scalar_type() == at::kFloat && ws_ml->numel() >= p.num_seqs * n_kv_heads * splits * G * 2,
                "ws_ml too small");
    p.ws_o = ws_o->data_ptr<float>();
    p.ws_ml = ws_ml->data_ptr<float>();
  }
  LAKEB_CHECK_RC(lakeb::paged_decode(p, cur_stream()), "paged_decode");
}

int64_t decode_splits(int64_t num_seqs, int64_t n_kv_heads, int64_t max_blocks) {
  return lakeb::paged_decode_splits(static_cast<int>(num_seqs), static_cast<int>(n_kv_heads),
                                    static_cast<int>(max_blocks));
}

void paged_prefill(const at::Tensor& q, at::Tensor& out, const at::Tensor& arena, int64_t layer,
                   const at::Tensor& block_tables, const at::Tensor& seq_lens, const at::Tensor& tiles,
                   int64_t n_q_heads, int64_t n_kv_heads, double scale, c10::optional<at::Tensor> status,
                   bool tensor_core) {
  PagedAttnArgs p = attn_args(q, out, arena, layer, block_tables, seq_lens, n_q_heads, n_kv_heads, scale, status);
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 4 && tiles.is_contiguous(),
              "tiles int32 [n, 4]");
  check_aligned(tiles, "tiles");
  p.tiles = reinterpret_cast<const int4*>(tiles.data_ptr<int>());
  p.num_tiles = static_cast<int>(tiles.size(0));
  if (tensor_core) {
    LAKEB_CHECK_RC(lakeb::paged_prefill_tc(p, q.size(0), cur_stream()), "paged_prefill_tc");
  } else {
    LAKEB_CHECK_RC(lakeb::paged_prefill(p, cur_stream()), "paged_prefill");
  }
}

void rmsnorm(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, double eps) {
  check_bf16_2d(x, "x");
  check_bf16_2d(out, "out");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.numel() == x.size(1), "w");
  check_aligned(w, "w");
  LAKEB_CHECK_RC(lakeb::rmsnorm_bf16(bf(x), x.stride(0), bf(w), bfm(out), out.stride(0), static_cast<int>(x.size(0)),
                                     static_cast<int>(x.size(1)), static_cast<float>(eps), cur_stream()),
                 "rmsnorm");
}

void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, c10::optional<at::Tensor> status) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids int32");
  check_bf16_2d(table, "table");
  check_bf16_2d(out, "out");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && out.size(1) == table.size(1), "shapes");
  LAKEB_CHECK_RC(lakeb::embedding_bf16(ids.data_ptr<int>(), bf(table), bfm(out), static_cast<int>(ids.numel()),
                                       static_cast<int>(table.size(1)), static_cast<int>(table.size(0)),
                                       status_ptr(status), cur_stream()),
                 "embedding");
}

void argmax(const at::Tensor& logits, c10::optional<at::Tensor> bitmask, at::Tensor& out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "logits fp32 2-D");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() >= logits.size(0), "out int32");
  const uint32_t* bm = nullptr;
  int words = 0;
  if (bitmask.has_value()) {
    bm = reinterpret_cast<const uint32_t*>(bitmask->data_ptr<int>());
    words = static_cast<int>(bitmask->size(1));
  }
  LAKEB_CHECK_RC(lakeb::argmax_f32(logits.data_ptr<float>(), logits.stride(0), static_cast<int>(logits.size(0)),
                                   static_cast<int>(logits.size(1)), bm, words, out.data_ptr<int>(), cur_stream()),
                 "argmax");
}

void unpack_argmax(const at::Tensor& keys, at::Tensor& out, int64_t n) {
  TORCH_CHECK(keys.scalar_type() == at::kLong && out.scalar_type() == at::kInt, "dtypes");
  LAKEB_CHECK_RC(lakeb::unpack_argmax(reinterpret_cast<const unsigned long long*>(keys.data_ptr<int64_t>()),
                                      out.data_ptr<int>(), static_cast<int>(n), cur_stream()),
                 "unpack_argmax");
}

void apply_bitmask(at::Tensor& logits, const at::Tensor& bitmask) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "logits");
  TORCH_CHECK(bitmask.scalar_type() == at::kInt && bitmask.dim() == 2, "bitmask");
  LAKEB_CHECK_RC(lakeb::apply_bitmask_f32(logits.data_ptr<float>(), logits.stride(0), static_cast<int>(logits.size(0)),
                                          static_cast<int>(logits.size(1)),
                                          reinterpret_cast<const uint32_t*>(bitmask.data_ptr<int>()),
                                          static_cast<int>(bitmask.size(1)), cur_stream()),
                 "apply_bitmask");
}

void chain_reject(const at::Tensor& draft, const at::Tensor& draft_off, const at::Tensor& target,
                  const at::Tensor& target_off, at::Tensor& out, at::Tensor& out_len) {
  for (auto* t : {&draft, &draft_off, &target, &target_off})
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous(), "int32 inputs");
  const int nreq = static_cast<int>(draft_off.numel() - 1);
  LAKEB_CHECK_RC(lakeb::chain_reject(draft.data_ptr<int>(), draft_off.data_ptr<int>(), target.data_ptr<int>(),
                                     target_off.data_ptr<int>(), out.data_ptr<int>(), out_len.data_ptr<int>(),
                                     static_cast<int>(out.stride(0)), nreq, cur_stream()),
                 "chain_reject");
}

// Copy pages between two page-major buffers (either may be a peer GPU's buffer).
void resolve_tokens(at::Tensor& ids, const at::Tensor& prev) {
  TORCH_CHECK(ids.is_cuda() && prev.is_cuda() && ids.scalar_type() == at::kInt && prev.scalar_type() == at::kInt &&
                  ids.is_contiguous() && prev.is_contiguous(),
              "ids / prev: contiguous int32 CUDA tensors");
  LAKEB_CHECK_RC(lakeb::resolve_tokens(ids.data_ptr<int>(), prev.data_ptr<int>(), static_cast<int>(ids.numel()),
                                       static_cast<int>(prev.numel()), cur_stream()),
                 "resolve_tokens");
}

void page_copy(const at::Tensor& src, at::Tensor& dst, const at::Tensor& src_ids, const at::Tensor& dst_ids,
               int64_t page_bytes, int64_t sub_off, int64_t sub_bytes, c10::optional<at::Tensor> status) {
  TORCH_CHECK(src_ids.scalar_type() == at::kLong && dst_ids.scalar_type() == at::kLong, "ids int64");
  TORCH_CHECK(src_ids.numel() == dst_ids.numel(), "id count mismatch");
  TORCH_CHECK(page_bytes > 0, "page_bytes must be positive");
  check_aligned(src, "src");
  check_aligned(dst, "dst");
  const int64_t src_pages = static_cast<int64_t>(src.numel()) * src.element_size() / page_bytes;
  const int64_t dst_pages = static_cast<int64_t>(dst.numel()) * dst.element_size() / page_bytes;
  LAKEB_CHECK_RC(lakeb::page_copy(src.data_ptr(), dst.data_ptr(), src_ids.data_ptr<int64_t>(),
                                  dst_ids.data_ptr<int64_t>(), static_cast<int>(src_ids.numel()), page_bytes,
                                  sub_off, sub_bytes, cur_stream(), src_pages, dst_pages, status_ptr(status)),
                 "page_copy");
}

// Same as page_copy but the destination is given as a raw device address
// (an IPC-mapped peer buffer that has no tensor of its own in this process).
void page_copy_to_ptr(const at::Tensor& src, int64_t dst_ptr, const at::Tensor& src_ids, const at::Tensor& dst_ids,
                      int64_t page_bytes, int64_t sub_off, int64_t sub_bytes) {
  TORCH_CHECK(src_ids.scalar_type() == at::kLong && dst_ids.scalar_type() == at::kLong, "ids int64");
  check_aligned(src, "src");
  TORCH_CHECK(dst_ptr % 16 == 0, "dst_ptr must be 16-byte aligned");
  LAKEB_CHECK_RC(lakeb::page_copy(src.data_ptr(), reinterpret_cast<void*>(dst_ptr), src_ids.data_ptr<int64_t>(),
                                  dst_ids.data_ptr<int64_t>(), static_cast<int>(src_ids.numel()), page_bytes,
                                  sub_off, sub_bytes, cur_stream()),
                 "page_copy_to_ptr");
}

// Let kernels on the current device address memory that lives on `peer_device`
// (e.g. an arena mapped from another process through CUDA IPC). Returns true if
// access is (now) enabled.
bool enable_peer_access(int64_t peer_device) {
  int cur = 0;
  TORCH_CHECK(cudaGetDevice(&cur) == cudaSuccess, "cudaGetDevice failed");
  if (cur == peer_device) return true;
  int can = 0;
  TORCH_CHECK(cudaDeviceCanAccessPeer(&can, cur, static_cast<int>(peer_device)) == cudaSuccess,
              "cudaDeviceCanAccessPeer failed");
  if (!can) return false;
  cudaError_t e = cudaDeviceEnablePeerAccess(static_cast<int>(peer_device), 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return true;
  }
  TORCH_CHECK(e == cudaSuccess, "cudaDeviceEnablePeerAccess failed: ", cudaGetErrorString(e));
  return true;
}

// ---------------------------------------------------------------- IPC-shared buffers
// A buffer other processes can map: its own cudaMalloc allocation (so the IPC
// handle covers exactly this tensor), zero-filled, freed with the tensor.
at::Tensor alloc_ipc_tensor(std::vector<int64_t> sizes, at::ScalarType dtype) {
  int64_t n = 1;
  for (auto s : sizes) n *= s;
  const size_t bytes = static_cast<size_t>(n) * c10::elementSize(dtype);
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes);
  TORCH_CHECK(e == cudaSuccess, "cudaMalloc(", bytes, ") failed: ", cudaGetErrorString(e));
  e = cudaMemset(ptr, 0, bytes);
  TORCH_CHECK(e == cudaSuccess, "cudaMemset failed: ", cudaGetErrorString(e));
  int dev = 0;
  cudaGetDevice(&dev);
  auto opts = at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, dev));
  return torch::from_blob(ptr, sizes, [](void* p) { cudaFree(p); }, opts);
}

// IPC handle (64 bytes) of a tensor made by alloc_ipc_tensor.
py::bytes ipc_export(const at::Tensor& t) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, t.data_ptr());
  TORCH_CHECK(e == cudaSuccess, "cudaIpcGetMemHandle failed: ", cudaGetErrorString(e));
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

// Map another process's buffer into the *current* device's context (peer access
// from this device to the owner is enabled by the driver as needed). The tensor
// reports the current device; its memory may physically live on a peer GPU.
at::Tensor ipc_import(const py::bytes& handle, std::vector<int64_t> sizes, at::ScalarType dtype) {
  std::string hs(handle);
  TORCH_CHECK(hs.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, hs.data(), sizeof(h));
  void* ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  int dev = 0;
  cudaGetDevice(&dev);
  auto opts = at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, dev));
  return torch::from_blob(ptr, sizes, [](void* p) { cudaIpcCloseMemHandle(p); }, opts);
}

}  // namespace

#ifndef LAKEB_MODULE
#define LAKEB_MODULE _C
#endif
PYBIND11_MODULE(LAKEB_MODULE, m) {
  m.def("enable_peer_access", &enable_peer_access);
  m.def("alloc_ipc_tensor", &alloc_ipc_tensor);
  m.def("ipc_export", &ipc_export);
  m.def("ipc_import", &ipc_import);
  m.doc() = "lake_b200 sm_100a kernels";
  namespace py = pybind11;
  m.def("linear", &linear, py::arg("a"), py::arg("w"), py::arg("out"), py::arg("status") = py::none(),
        py::arg("max_ctas") = 0, py::arg("w_scale") = py::none());
  m.def("linear_residual", &linear_residual, py::arg("a"), py::arg("w"), py::arg("residual"), py::arg("out"),
        py::arg("status") = py::none(), py::arg("w_scale") = py::none());
  m.def("linear_swiglu", &linear_swiglu, py::arg("a"), py::arg("w"), py::arg("out"), py::arg("status") = py::none(),
        py::arg("tp") = py::none(), py::arg("w_scale") = py::none());
  m.def("linear_rs", &linear_rs, py::arg("a"), py::arg("w"), py::arg("tp"), py::arg("status") = py::none(), py::arg("w_scale") = py::none());
  m.def("tp_norm_push", &tp_norm_push, py::arg("h"), py::arg("w"), py::arg("eps"), py::arg("tp"),
        py::arg("status") = py::none());
  m.def("tp_argmax_combine", &tp_argmax_combine, py::arg("amax_ptrs"), py::arg("done_cnt"), py::arg("off"),
        py::arg("out"), py::arg("n"), py::arg("status") = py::none(), py::arg("base") = 0);
  m.def("tp_advance", &tp_advance, py::arg("base"), py::arg("deltas"));
  m.def("resolve_tokens", &resolve_tokens, py::arg("ids"), py::arg("prev"));
  m.def("gemm_grouped", &gemm_grouped, py::arg("a"), py::arg("w"), py::arg("out"), py::arg("epi"),
        py::arg("group_count"), py::arg("group_rows"), py::arg("row_slot") = py::none(),
        py::arg("row_rank") = py::none(), py::arg("dst_ptrs") = std::vector<int64_t>{}, py::arg("tp") = py::none(),
        py::arg("status") = py::none());
  m.def("moe_dispatch", &moe_dispatch, py::arg("logits"), py::arg("x"), py::arg("weights"), py::arg("n_experts"),
        py::arg("top_k"), py::arg("cap"), py::arg("world"), py::arg("rank"), py::arg("gathered"), py::arg("row_slot"),
        py::arg("row_rank"), py::arg("count"), py::arg("done_cnt"), py::arg("status") = py::none());
  m.def("moe_combine", &moe_combine, py::arg("h"), py::arg("comb"), py::arg("weights"), py::arg("top_k"),
        py::arg("wait_cnt") = 0, py::arg("wait_n") = 0, py::arg("target") = 0, py::arg("status") = py::none(),
        py::arg("wait_base") = 0);
  m.def("wait_counters", &wait_counters, py::arg("cnt"), py::arg("n"), py::arg("target"),
        py::arg("status") = py::none(), py::arg("limit_ns") = 0, py::arg("base") = 0);
  m.def("moe_dispatch_grid", []() { return lakeb::kMoEDispatchGrid; });
  m.def("set_gemm_pair_mode", [](int64_t mode) { lakeb::set_gemm_pair_mode(static_cast<int>(mode)); });
  m.def("gemm_pair_mode", []() { return lakeb::gemm_pair_mode(); });
  m.def("set_gemm_streamk_mode", [](int64_t mode) { lakeb::set_gemm_streamk_mode(static_cast<int>(mode)); });
  m.def("set_decode_split_mode", [](int64_t mode) { lakeb::set_decode_split_mode(static_cast<int>(mode)); });
  m.def("set_prefill_kernel", [](int64_t mode) { lakeb::set_prefill_kernel(static_cast<int>(mode)); });
  m.def("set_gemm_w8a8_min_m", [](int64_t m) { lakeb::set_gemm_w8a8_min_m(static_cast<int>(m)); });
  m.def("gemm_w8a8_reserve", [](int64_t m, int64_t k) { return lakeb::gemm_w8a8_reserve(m, k); },
        "reserve the current device's W8A8 activation workspace for M x K (outside graph capture)");
  m.def("quantize_fp8_rows", [](const at::Tensor& x, at::Tensor& q, at::Tensor& s) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x bf16 [M, K]");
    TORCH_CHECK(q.scalar_type() == at::kByte && q.sizes() == x.sizes() && q.is_contiguous(), "q uint8 [M, K]");
    TORCH_CHECK(s.scalar_type() == at::kFloat && s.dim() == 2 && s.size(0) == x.size(0) &&
                    s.size(1) == x.size(1) / 128 && s.is_contiguous(), "s fp32 [M, K/128]");
    LAKEB_CHECK_RC(lakeb::quantize_fp8_rows(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                                            static_cast<int>(x.size(0)), static_cast<int>(x.size(1)),
                                            q.data_ptr<uint8_t>(), q.size(1), s.data_ptr<float>(),
                                            static_cast<int>(s.size(1)), cur_stream()),
                   "quantize_fp8_rows");
  });
  m.def("prefill_trace_enable", [](bool on) {
    LAKEB_CHECK_RC(lakeb::prefill_trace_enable(on ? 1 : 0), "prefill_trace_enable");
  });
  m.def("prefill_trace", []() {
    auto t = at::zeros({1024}, at::TensorOptions().dtype(at::kLong));
    LAKEB_CHECK_RC(lakeb::prefill_trace_read(reinterpret_cast<long long*>(t.data_ptr<int64_t>()), 1024), "prefill_trace_read");
    return t;
  });
  m.def("register_host_arena", &register_host_arena, "accept this pinned host tensor as a second K/V target");
  m.def("unregister_host_arena", &unregister_host_arena);
  m.def("gemm_grid", [](int64_t M, int64_t N, int64_t K, int64_t epi, bool w8) {
    return lakeb::gemm_grid(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), static_cast<int>(epi), 0,
                            w8);
  }, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"), py::arg("w8") = false);
  m.def("gemm_workspace_init", &lakeb::gemm_workspace_init,
        "allocate the current device's stream-K workspace (outside any graph capture)");
  m.def("tp_norm_grid", [](int64_t rows) { return lakeb::tp_norm_grid(static_cast<int>(rows)); });
  m.def("linear_qkv", &linear_qkv, py::arg("a"), py::arg("w"), py::arg("q_out"), py::arg("rope_cs"),
        py::arg("positions"), py::arg("slots"), py::arg("arena"), py::arg("layer"), py::arg("n_q_heads"),
        py::arg("n_kv_heads"), py::arg("peer_arena") = py::none(), py::arg("peer_slots") = py::none(),
        py::arg("status") = py::none(), py::arg("tp") = py::none(), py::arg("q_norm") = py::none(),
        py::arg("k_norm") = py::none(), py::arg("qk_eps") = 1e-6, py::arg("w_scale") = py::none());
  m.def("linear_argmax", &linear_argmax, py::arg("a"), py::arg("w"), py::arg("amax"), py::arg("bitmask") = py::none(),
        py::arg("status") = py::none(), py::arg("tp") = py::none(), py::arg("w_scale") = py::none());
  m.def("paged_decode", &paged_decode, py::arg("q"), py::arg("out"), py::arg("arena"), py::arg("layer"),
        py::arg("block_tables"), py::arg("seq_lens"), py::arg("n_q_heads"), py::arg("n_kv_heads"), py::arg("scale"),
        py::arg("splits") = 1, py::arg("ws_o") = py::none(), py::arg("ws_ml") = py::none(),
        py::arg("status") = py::none());
  m.def("decode_splits", &decode_splits);
  m.def("paged_prefill", &paged_prefill, py::arg("q"), py::arg("out"), py::arg("arena"), py::arg("layer"),
        py::arg("block_tables"), py::arg("seq_lens"), py::arg("tiles"), py::arg("n_q_heads"), py::arg("n_kv_heads"),
        py::arg("scale"), py::arg("status") = py::none(), py::arg("tensor_core") = true);
  m.def("rmsnorm", &rmsnorm);
  m.def("embedding", &embedding, py::arg("ids"), py::arg("table"), py::arg("out"), py::arg("status") = py::none());
  m.def("argmax", &argmax);
  m.def("unpack_argmax", &unpack_argmax);
  m.def("apply_bitmask", &apply_bitmask);
  m.def("chain_reject", &chain_reject);
  m.def("page_copy", &page_copy, py::arg("src"), py::arg("dst"), py::arg("src_ids"), py::arg("dst_ids"),
        py::arg("page_bytes"), py::arg("sub_off"), py::arg("sub_bytes"), py::arg("status") = py::none());
  m.def("debug_checks", &lakeb::debug_checks_enabled,
        "true in the bounds-checked debug build (lake_b200/_C_debug.so)");
  m.def("page_copy_to_ptr", &page_copy_to_ptr);
}
