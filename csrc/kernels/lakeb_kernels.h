// Host-side declarations of every CUDA launcher in csrc/kernels. The torch
// binding (csrc/bindings/ops.cpp) is the only consumer; kernels themselves are
// compiled without torch headers.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace lakeb {

// ----------------------------------------------------------------- GEMM
// C[M,N] = A[M,K] * B[N,K]^T, bf16 operands (both K-major), fp32 accumulation
// in tensor memory, fused epilogue selected by `epi`.
enum GemmEpi : int {
  kEpiStoreBf16 = 0,  // C (bf16) = acc
  kEpiResidual = 1,   // C (bf16) = acc + R   (R may alias C)
  kEpiSwiGLU = 2,     // C[:, j] = silu(acc[gate j]) * acc[up j]  (tile-interleaved weight rows)
  kEpiQKV = 3,        // q -> C with RoPE; k (RoPE) and v -> paged KV arena (+ optional peer arena)
  kEpiArgmax = 4,     // per-row argmax (optionally bitmask-filtered) via 64-bit atomicMax
  kEpiStoreF32 = 5,   // C (fp32) = acc
  kEpiRSPush = 6,     // partial rows -> owner rank's receive buffer over NVLink (GEMM + reduce-scatter)
  kEpiScatter = 7,    // row r -> rs_recv[row_rank[r] or 0] + row_slot[r] * ldc (skip if slot < 0), bf16
};

constexpr int kMaxTP = 8;

// Tensor-parallel fusion of a GEMM with the collective beside it. The residual
// stream is split by rows: rank r owns rows [r*rows_per_rank, (r+1)*rows_per_rank).
// Counters are monotonically increasing; a wait on counter c completes when
// c >= (base ? *base : 0) + off. Every CTA of a signalling kernel adds 1 to the
// counter slot of its rank at every destination rank.
struct TPGemmArgs {
  int world = 1, rank = 0;
  int rows_per_rank = 0;
  int m_rot = 0;  // m-block the tile walk starts at (own rows first for all-gather, peers' rows first for RS)
  // all-gather -> GEMM: A rows of shard s are usable once ag_cnt[s] reaches the target
  const unsigned long long* ag_cnt = nullptr;
  const unsigned long long* ag_base = nullptr;
  unsigned long long ag_off = 0;
  int ag_all = 0;  // 1: wait for every shard before the first tile (rows not laid out by shard)
  // GEMM -> reduce-scatter: partial row g goes to rank g / rows_per_rank at
  // rs_recv[dst] + (rank * rows_per_rank + g % rows_per_rank) * ldc, then rs_cnt[dst][rank] += 1 per CTA
  __nv_bfloat16* rs_recv[kMaxTP] = {};
  unsigned long long* rs_cnt[kMaxTP] = {};
  // completion signal of any epilogue (done_cnt[dst][rank] += 1 per CTA)
  unsigned long long* done_cnt[kMaxTP] = {};
  int col_offset = 0;  // global index of this rank's first output column (vocab-parallel argmax)
};

struct KVArenaView {
  __nv_bfloat16* base = nullptr;  // arena [num_blocks, layers, 2, kv_heads, block_size, head_dim]
  int64_t block_stride = 0;       // elements between consecutive blocks
  int64_t layer_offset = 0;       // elements to this layer's K half inside a block
  int64_t kv_stride = 0;          // elements from the K half to the V half
  int64_t head_stride = 0;        // elements between kv heads
  int block_size = 16;            // tokens per block
  int64_t num_slots = 0;          // blocks x block_size (index checks of the debug build)
};

struct GemmArgs {
  const __nv_bfloat16* A = nullptr;
  int64_t lda = 0;
  const __nv_bfloat16* B = nullptr;
  int64_t ldb = 0;
  int M = 0, N = 0, K = 0;
  void* C = nullptr;
  int64_t ldc = 0;
  const __nv_bfloat16* R = nullptr;
  int64_t ldr = 0;
  // QKV epilogue
  const float2* rope_cs = nullptr;  // [max_pos, head_dim/2] (cos, sin)
  const int* positions = nullptr;   // [M]
  const int64_t* slots = nullptr;   // [M] local slot (block*block_size+offset), <0 = skip
  KVArenaView kv;
  const int64_t* peer_slots = nullptr;  // [M] slot in the peer arena, <0 = skip
  KVArenaView peer_kv;                  // arena on another GPU (P2P-mapped), base==nullptr = none
  int n_q_heads = 0, n_kv_heads = 0;
  // optional per-head RMSNorm of q and k before RoPE (Qwen3): weights [128] bf16
  const __nv_bfloat16* q_norm_w = nullptr;
  const __nv_bfloat16* k_norm_w = nullptr;
  float qk_eps = 1e-6f;
  // argmax epilogue
  unsigned long long* amax = nullptr;  // [M], zero-initialised by the caller
  const uint32_t* bitmask = nullptr;   // [M, bitmask_words], bit=1 allowed
  int bitmask_words = 0;
  int* status = nullptr;               // device status word
  int max_ctas = 0;                    // 0 = number of SMs
  TPGemmArgs tp;
  // Grouped GEMM (one group per expert): group g owns A rows [g*group_rows, g*group_rows + group_count[g])
  // and B rows [g*N, (g+1)*N); output row r of the group is A row r. group_count must be final when
  // the kernel starts (written by an earlier kernel on the stream); tiles past a group's count are skipped.
  int groups = 0;
  int group_rows = 0;  // multiple of 128
  const int* group_count = nullptr;
  // fp8 weights (W8A16): B is e4m3 [N (x groups), K] bytes with one fp32 scale per 128x128 block,
  // b_scale[(n / 128) * b_scale_ld + k / 128]; converter warps dequantise each stage to bf16 in
  // shared memory and the MMA runs on bf16 (kind::f16)
  const uint8_t* B8 = nullptr;
  int64_t ldb8 = 0;  // bytes between rows of B8
  const float* b_scale = nullptr;
  int b_scale_ld = 0;
  // stream-K (set by the dispatcher): the (tile, k-block) units are cut into one contiguous range
  // per CTA; a tile cut between CTAs is summed in split_ws (fp32 [grid][128][BN], zero between
  // uses) and the last contributor to arrive (split_cnt per slot) applies the epilogue
  int streamk = 0;
  float* split_ws = nullptr;
  int* split_cnt = nullptr;
  // kEpiScatter destinations (rows indexed like A)
  const int* row_slot = nullptr;
  const int* row_rank = nullptr;
  // fp8 activations (W8A8; the dispatcher fills these for fp8 weights at prefill sizes): A8 is e4m3
  // [M, K] bytes with one fp32 scale per row and 128-column block, a_scale[m * a_scale_ld + k / 128].
  // The MMAs run kind::f8f6f4 per 128-deep k-block into a TMEM partial and the epilogue warps add
  // each partial, times a_scale x b_scale, into fp32 registers (one scale pair per k-block)
  const uint8_t* A8 = nullptr;
  int64_t lda8 = 0;
  const float* a_scale = nullptr;
  int a_scale_ld = 0;
};

// Block-scaled e4m3 quantisation of bf16 rows: q[m, k] = x[m, k] / s[m, k/128] with
// s = amax(|x[m, 128-block]|) / 448 (1 for an all-zero block). K % 128 == 0.
int quantize_fp8_rows(const __nv_bfloat16* x, int64_t ldx, int M, int K, uint8_t* q, int64_t ldq, float* s,
                      int s_ld, cudaStream_t stream);
// Smallest M at which gemm_bf16 runs fp8-weight GEMMs as W8A8 (0 = never: always W8A16).
void set_gemm_w8a8_min_m(int m);
// Runs fp8-weight GEMMs with M >= the threshold as W8A8 from now on when the device's activation
// workspace holds M x K (allocated here; call outside graph capture). Returns false on failure.
// The workspace is shared by the device's W8A8 GEMMs: issue them from one stream at a time.
bool gemm_w8a8_reserve(int64_t M, int64_t K);

// Two-SM (cta_group::2) GEMM for large M; epilogues: store bf16, residual, SwiGLU, fp32.
int gemm_bf16_pair(const GemmArgs& args, int epi, cudaStream_t stream);
int gemm_pair_grid(int M, int N);
// 0 = never use the two-SM kernel from gemm_bf16, 1 = use it for large plain GEMMs (M >= 512).
void set_gemm_pair_mode(int mode);
int gemm_pair_mode();

// Number of CTAs gemm_bf16 launches for a shape (the per-call increment of TP counters).
// CTAs a gemm_bf16 launch of this shape uses (one cross-GPU signal per CTA): the TP host code
// sizes its counter waits with it.
int gemm_grid(int M, int N, int K, int epi, int max_ctas, bool w8 = false);
bool gemm_workspace_init();  // current device's stream-K workspace (call outside graph capture)

// Returns 0 on success, otherwise a cudaError_t or negative argument error.
int gemm_bf16(const GemmArgs& args, int epi, cudaStream_t stream);

// ----------------------------------------------------------------- attention
// Paged attention over the KV arena [num_blocks, layers, 2, kv_heads, block_size=16, head_dim=128].
struct PagedAttnArgs {
  const __nv_bfloat16* q = nullptr;  // [tokens, n_q_heads*128]
  int64_t q_stride = 0;              // elements between tokens
  __nv_bfloat16* out = nullptr;      // [tokens, n_q_heads*128]
  int64_t out_stride = 0;
  const __nv_bfloat16* arena = nullptr;
  int64_t num_blocks = 0;
  int num_layers = 0, layer = 0;
  int n_q_heads = 0, n_kv_heads = 0;
  const int* block_tables = nullptr;  // [num_seqs, bt_stride]
  int bt_stride = 0;
  const int* seq_lens = nullptr;      // [num_seqs] context length (keys) per sequence
  int num_seqs = 0;
  float scale = 0.f;
  // decode: split-KV partials (scratch). ws_o [num_seqs, kv_heads, splits, G, 128], ws_ml [.., G, 2]
  int splits = 1;
  float* ws_o = nullptr;
  float* ws_ml = nullptr;
  // prefill: query tiles (seq, first query row, number of queries <= 64, position of first query)
  const int4* tiles = nullptr;
  int num_tiles = 0;
  int* status = nullptr;
};

// One query token per sequence (decode). Query row s belongs to sequence s.
int paged_decode(const PagedAttnArgs& a, cudaStream_t stream);
// paged_decode with a caller-encoded tensor map of the arena (no tensor-map cache use).
int paged_decode_with_map(const PagedAttnArgs& a, const CUtensorMap& arena_map, cudaStream_t stream);
// Number of split-KV partitions paged_decode will use for a batch shape.
int paged_decode_splits(int num_seqs, int n_kv_heads, int max_blocks_per_seq);
void set_decode_split_mode(int mode);  // 0: fill 2 CTAs per SM (default), 1: best wave efficiency
void set_gemm_streamk_mode(int mode);  // 1: stream-K where it balances SMs (default), 0: data-parallel only
// Causal prefill / chunked prefill over query tiles of <= 64 rows (warp-level MMA).
int paged_prefill(const PagedAttnArgs& a, cudaStream_t stream);
// Same on tcgen05 tensor cores over query tiles of <= 128 rows; q has q_rows rows.
int paged_prefill_tc(const PagedAttnArgs& a, int64_t q_rows, cudaStream_t stream);
// Two query heads of one KV group per CTA (ping-pong softmax/MMA, P and O in TMEM); needs an
// even number of query heads per KV head. paged_prefill_tc dispatches to it when it applies
// (set_prefill_kernel(0) keeps the one-head kernel).
bool prefill_pingpong_ok(const PagedAttnArgs& a);
int paged_prefill_pingpong(const PagedAttnArgs& a, int64_t q_rows, cudaStream_t stream);
void set_prefill_kernel(int mode);  // 1: ping-pong where it applies (default), 0: one head per CTA, 10+i: variant i
void set_prefill_variant(int v);    // softmax variant of the ping-pong kernel (-1: default)
// Timeline of the ping-pong kernel's first CTA (SM clock cycles): recording on/off, read back.
int prefill_trace_enable(int on);
int prefill_trace_read(long long* host, int n);

// ----------------------------------------------------------------- misc
int rmsnorm_bf16(const __nv_bfloat16* x, int64_t sx, const __nv_bfloat16* w, __nv_bfloat16* out, int64_t so, int rows,
                 int dim, float eps, cudaStream_t stream);
int embedding_bf16(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int n, int dim, int vocab,
                   int* status, cudaStream_t stream);
int argmax_f32(const float* logits, int64_t stride, int rows, int vocab, const uint32_t* bitmask, int words, int* out,
               cudaStream_t stream);
int unpack_argmax(const unsigned long long* keys, int* out, int n, cudaStream_t stream);
int apply_bitmask_f32(float* logits, int64_t stride, int rows, int vocab, const uint32_t* bitmask, int words,
                      cudaStream_t stream);
int chain_reject(const int* draft, const int* draft_off, const int* target, const int* target_off, int* out,
                 int* out_len, int out_stride, int nreq, cudaStream_t stream);
// ----------------------------------------------------------------- tensor parallel
// Reduce-scatter completion + residual + RMSNorm + all-gather push, per owned row:
//   h = h + sum_src recv[src][row]          (when recv != nullptr, after rs_cnt waits)
//   y = rmsnorm(h) * w                      -> dst[d][row_map(global row)] for every rank d
// then ag_cnt[d][rank] += 1 per CTA. rows_per_rank rows are owned; global row = rank*rows_per_rank + row.
struct TPNormArgs {
  int world = 1, rank = 0, rows_per_rank = 0, dim = 0;
  const __nv_bfloat16* recv = nullptr;  // local [world][rows_per_rank][dim]
  const unsigned long long* rs_cnt = nullptr;
  const unsigned long long* rs_base = nullptr;
  unsigned long long rs_off = 0;
  __nv_bfloat16* h = nullptr;  // local [rows_per_rank][dim]
  int store_h = 1;
  const __nv_bfloat16* w = nullptr;
  float eps = 1e-5f;
  __nv_bfloat16* dst[kMaxTP] = {};
  int64_t dst_ld = 0;
  const int* row_map = nullptr;  // [world*rows_per_rank] destination row or -1; null = identity
  unsigned long long* ag_cnt[kMaxTP] = {};
  unsigned long long* reset_ptr = nullptr;  // zeroed by block 0 before signalling (local array)
  int reset_n = 0;
  int* status = nullptr;
};
int tp_norm_push(const TPNormArgs& a, cudaStream_t stream);
int tp_norm_grid(int rows_per_rank);

// Vocab-parallel argmax combine: waits done_cnt[src] targets, token[r] = argmax over ranks of amax[d][r].
struct TPPtrs {
  const unsigned long long* p[kMaxTP] = {};
};
constexpr int kMaxTPDeltas = 16;
struct TPDeltas {
  int n = 0;
  unsigned long long v[kMaxTPDeltas] = {};
};
int tp_advance(unsigned long long* base, const TPDeltas& d, cudaStream_t stream);
int tp_argmax_combine(const TPPtrs& amax, int world, const unsigned long long* done_cnt,
                      const unsigned long long* base, unsigned long long off, int* out, int n, int* status,
                      cudaStream_t stream);

// ----------------------------------------------------------------- mixture of experts
// Top-k routing + gather of token rows into per-expert segments (and, across GPUs, the
// all-to-all dispatch over NVLink). Local form: logits [M, ld_logits] fp32 (first E used),
// x [M, dim] bf16 -> gathered [E*cap, dim], row_slot[E*cap] = token*top_k + j, weights [M, top_k],
// count[E] (zeroed by the caller). Expert e lives on rank e / experts_per_rank.
struct MoEDispatchArgs {
  const float* logits = nullptr;
  int ld_logits = 0;
  const __nv_bfloat16* x = nullptr;
  int M = 0, dim = 0, n_experts = 0, top_k = 2, cap = 0;
  float* weights = nullptr;  // [M, top_k]
  int world = 1, rank = 0, experts_per_rank = 0;
  // per destination rank: its gathered rows, row_slot, row_rank, count arrays (peer pointers for EP)
  __nv_bfloat16* gathered[kMaxTP] = {};
  int* row_slot[kMaxTP] = {};
  int* row_rank[kMaxTP] = {};
  int* count[kMaxTP] = {};
  unsigned long long* done_cnt[kMaxTP] = {};  // EP: +1 per CTA at every destination after the writes
  int* status = nullptr;
};
int moe_dispatch(const MoEDispatchArgs& a, cudaStream_t stream);
constexpr int kMoEDispatchGrid = 64;  // fixed, so every rank adds the same count per call

// h[t] += sum_j weights[t, j] * comb[t*top_k + j]   (after waiting for EP combine counters)
int moe_combine(__nv_bfloat16* h, const __nv_bfloat16* comb, const float* weights, int M, int dim, int top_k,
                const unsigned long long* wait_cnt, int wait_n, unsigned long long wait_target, int* status,
                cudaStream_t stream, const unsigned long long* wait_base = nullptr);
// Waits until wait_cnt[0..n) >= target (EP: all sources dispatched) - a launch-ordering point.
// Wait until every cnt[i] >= (*base, when given) + target; a wait that runs past limit_ns (0: the
// default 2 s) records kErrTimeoutFlag in *status and the kernel returns. A device-resident base
// keeps the target valid when the launch is replayed from a CUDA graph.
int wait_counters(const unsigned long long* cnt, int n, unsigned long long target, int* status,
                  cudaStream_t stream, unsigned long long limit_ns = 0, const unsigned long long* base = nullptr);

// ids[i] < 0 -> prev[-1 - ids[i]] (tokens sampled by the previous, still in-flight step)
int resolve_tokens(int* ids, const int* prev, int n, int n_prev, cudaStream_t stream);
// src_pages / dst_pages bound the page ids in the debug build (0 = unknown)
int page_copy(const void* src, void* dst, const int64_t* src_ids, const int64_t* dst_ids, int n, int64_t page_bytes,
              int64_t sub_off, int64_t sub_bytes, cudaStream_t stream, int64_t src_pages = 0, int64_t dst_pages = 0,
              int* status = nullptr);
bool debug_checks_enabled();  // true in the bounds-checked debug build

}  // namespace lakeb
