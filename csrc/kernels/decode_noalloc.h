// Allocation-free entry point for paged decode attention.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this library.
//
// Who it is for: callers that must not allocate device memory while serving.
// Typical cases are a serving process that partitions HBM once at start-up
// (weights, KV arena, activations) and treats any later cudaMalloc as a
// budget violation; code embedded in another framework whose caching
// allocator owns the device memory, so a private cudaMalloc would fragment or
// exceed that allocator's pool; and latency-critical paths where
// cudaMalloc/cudaFree would add an implicit device synchronisation. Such
// callers cannot hand the split-KV decode kernel the scratch buffers it needs
// for its partial results, so this entry point keeps that scratch in a
// fixed-size array compiled into the library.
//
// Contract:
//  * The caller passes inputs and outputs only (device pointers, all of the
//    same device, which must be current). Layouts are those of
//    lakeb::paged_decode: q and out are [num_seqs, n_q_heads*128] bf16 rows
//    with the given row strides (elements, multiples of 8, 16-byte aligned);
//    arena is [num_blocks, num_layers, 2, n_kv_heads, 16, 128] bf16;
//    block_tables is [num_seqs, bt_stride] int32; seq_lens is [num_seqs]
//    int32.
//  * Scratch lives in a file-scope device array of LAKEB_NOALLOC_SCRATCH_BYTES
//    (8 MiB). Every GPU that loads the library holds those 8 MiB until the
//    process exits. A batch whose split-KV partials need more returns
//    LAKEB_NOALLOC_ETOO_LARGE and launches nothing.
//  * The first call on a device looks up the scratch array's device address
//    (cudaGetSymbolAddress) with that device current. With CUDA's lazy module
//    loading (the default), that first call is also what loads this library's
//    GPU module on the device, which creates the 8 MiB array (the driver's
//    memory, not cudaMalloc) and can synchronise the device. Make that first
//    call before any stream capture on the device, and outside
//    latency-critical paths; every later call allocates nothing.
//  * No call allocates or frees device memory through cudaMalloc/cudaFree or
//    an allocating library routine (torch's included).
//  * The bounds-checked debug build records index errors in a status word;
//    this entry point passes none, so those checks are not reported through
//    it (out-of-range page ids are skipped silently in that build). Argument
//    errors (layer outside [0, num_layers), num_blocks <= 0, bt_stride < 1,
//    misaligned pointers or strides) return LAKEB_NOALLOC_EARG before any
//    launch.
//  * Every call shares the one scratch array, which keeps the previous call's
//    contents. The kernels overwrite every partial result they later read, so
//    nothing has to start at zero. Calls whose kernels overlap on the GPU
//    (different streams without ordering between them) race on the scratch:
//    serialise them on one stream or with events.
#pragma once
#include <stdint.h>

#define LAKEB_NOALLOC_SCRATCH_BYTES (8u << 20)
#define LAKEB_NOALLOC_ETOO_LARGE (-100)
#define LAKEB_NOALLOC_ESETUP (-101)
#define LAKEB_NOALLOC_EARG (-102)

#ifdef __cplusplus
extern "C" {
#endif

// Returns 0 on success, a negative LAKEB_NOALLOC_* code, or a cudaError_t.
// splits <= 0 picks the split count paged_decode would use for this shape.
int lakeb_paged_decode_noalloc(const void* q, int64_t q_stride, void* out, int64_t out_stride, const void* arena,
                               int64_t num_blocks, int num_layers, int layer, int n_q_heads, int n_kv_heads,
                               const int* block_tables, int bt_stride, const int* seq_lens, int num_seqs, float scale,
                               int splits, void* stream);

// Bytes of scratch the call above needs for this shape (0 when no split is used).
int64_t lakeb_paged_decode_noalloc_scratch_bytes(int num_seqs, int n_q_heads, int n_kv_heads, int splits);

#ifdef __cplusplus
}
#endif
