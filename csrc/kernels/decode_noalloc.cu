// Allocation-free entry point for paged decode attention (see decode_noalloc.h
// for who needs it and the contract). This entry point has no counterpart in
// the reference implementation.
//
// The split-KV partial results (per sequence, KV head, split and query head:
// 128 fp32 values plus a running max and sum) go to a fixed device array in
// this translation unit instead of caller-provided workspaces.
#include <cuda.h>
#include <cuda_runtime.h>

#include "decode_noalloc.h"
#include "lakeb_kernels.h"
#include "tma_host.h"

namespace {

// Scratch shared by every call on a device; see the header for sizing and races.
static __device__ __align__(256) unsigned char g_decode_scratch[LAKEB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
// Device address of g_decode_scratch per device, looked up once with that device current.
void* g_scratch_ptr[kMaxDevices] = {nullptr};

int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return LAKEB_NOALLOC_ESETUP;
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || !p) return e != cudaSuccess ? static_cast<int>(e) : LAKEB_NOALLOC_ESETUP;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int64_t lakeb_paged_decode_noalloc_scratch_bytes(int num_seqs, int n_q_heads, int n_kv_heads, int splits) {
  if (splits <= 1 || n_kv_heads <= 0) return 0;
  const int64_t G = n_q_heads / n_kv_heads;
  const int64_t parts = static_cast<int64_t>(num_seqs) * n_kv_heads * splits * G;
  const int64_t o_bytes = parts * 128 * 4;
  const int64_t ml_bytes = parts * 2 * 4;
  return ((o_bytes + 255) / 256) * 256 + ml_bytes;
}

extern "C" int lakeb_paged_decode_noalloc(const void* q, int64_t q_stride, void* out, int64_t out_stride,
                                          const void* arena, int64_t num_blocks, int num_layers, int layer,
                                          int n_q_heads, int n_kv_heads, const int* block_tables, int bt_stride,
                                          const int* seq_lens, int num_seqs, float scale, int splits, void* stream) {
  if (num_seqs <= 0) return 0;
  if (!q || !out || !arena || !block_tables || !seq_lens || n_kv_heads <= 0 || n_q_heads % n_kv_heads ||
      n_q_heads / n_kv_heads > 16 || q_stride % 8 || out_stride % 8 || (reinterpret_cast<uintptr_t>(q) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(arena) & 15))
    return LAKEB_NOALLOC_EARG;
  // A layer outside the arena would still be inside the tensor map (rows of another block), so
  // nothing would fault and the result would be silently wrong: refuse it here.
  if (num_blocks <= 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || bt_stride < 1)
    return LAKEB_NOALLOC_EARG;
  if (splits <= 0) splits = lakeb::paged_decode_splits(num_seqs, n_kv_heads, bt_stride);
  const int64_t need = lakeb_paged_decode_noalloc_scratch_bytes(num_seqs, n_q_heads, n_kv_heads, splits);
  if (need > static_cast<int64_t>(LAKEB_NOALLOC_SCRATCH_BYTES)) return LAKEB_NOALLOC_ETOO_LARGE;

  lakeb::PagedAttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.arena = static_cast<const __nv_bfloat16*>(arena);
  a.num_blocks = num_blocks;
  a.num_layers = num_layers;
  a.layer = layer;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.seq_lens = seq_lens;
  a.num_seqs = num_seqs;
  a.scale = scale;
  a.splits = splits;
  if (splits > 1) {
    void* base = nullptr;
    int rc = scratch_for_current_device(&base);
    if (rc) return rc;
    const int64_t G = n_q_heads / n_kv_heads;
    const int64_t o_bytes = static_cast<int64_t>(num_seqs) * n_kv_heads * splits * G * 128 * 4;
    a.ws_o = static_cast<float*>(base);
    a.ws_ml = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + ((o_bytes + 255) / 256) * 256);
  }
  const int64_t rows = num_blocks * num_layers * 2 * n_kv_heads * 16;
  if (rows >= (int64_t(1) << 31)) return LAKEB_NOALLOC_EARG;
  CUtensorMap map;
  if (!lakeb::encode_bf16_map(&map, arena, rows, 128, 128, 16, 64)) return LAKEB_NOALLOC_EARG;
  return lakeb::paged_decode_with_map(a, map, static_cast<cudaStream_t>(stream));
}
