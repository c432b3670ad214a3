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
};

struct KVArenaView {
  __nv_bfloat16* base = nullptr;  // arena [num_blocks, layers, 2, kv_heads, block_size, head_dim]
  int64_t block_stride = 0;       // elements between consecutive blocks
  int64_t layer_offset = 0;       // elements to this layer's K half inside a block
  int64_t kv_stride = 0;          // elements from the K half to the V half
  int64_t head_stride = 0;        // elements between kv heads
  int block_size = 16;            // tokens per block
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
  // argmax epilogue
  unsigned long long* amax = nullptr;  // [M], zero-initialised by the caller
  const uint32_t* bitmask = nullptr;   // [M, bitmask_words], bit=1 allowed
  int bitmask_words = 0;
  int* status = nullptr;               // device status word
  int max_ctas = 0;                    // 0 = number of SMs
};

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
// Causal prefill / chunked prefill over query tiles of <= 64 rows (warp-level MMA).
int paged_prefill(const PagedAttnArgs& a, cudaStream_t stream);
// Same on tcgen05 tensor cores over query tiles of <= 128 rows; q has q_rows rows.
int paged_prefill_tc(const PagedAttnArgs& a, int64_t q_rows, cudaStream_t stream);

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
int page_copy(const void* src, void* dst, const int64_t* src_ids, const int64_t* dst_ids, int n, int64_t page_bytes,
              int64_t sub_off, int64_t sub_bytes, cudaStream_t stream);

}  // namespace lakeb
