#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lakeb {

// Tensor map for a row-major bf16 matrix [rows, cols] (leading dimension `ld`
// elements) with boxes of box_rows x box_cols, 128-byte swizzle, zero fill
// outside the bounds. Cached per (pointer, shape, device).
bool make_bf16_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                   int box_cols = 64);

// Same encoding without the cache: fills `out` only (no heap use).
bool encode_bf16_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                     int box_cols = 64);

// Byte-element 2-D map without swizzle (fp8 operands staged for conversion).
bool make_u8_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                 int box_cols);
// e4m3 operand map for tcgen05 (kind::f8f6f4): byte elements, boxes of box_rows x 128 bytes with the
// 128-byte swizzle (one swizzle row = one 128-deep k-block), zero fill outside the bounds.
bool make_fp8_sw128_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);
int num_sms();

// Raises a kernel's dynamic shared-memory limit to `bytes` on the CURRENT device.
// cudaFuncSetAttribute is per device, so the call is remembered per (kernel, device):
// a process that launches on several GPUs sets it once on each of them. Thread-safe.
// Returns 0 or the cudaError_t of the failed call.
int ensure_smem_attr(const void* kernel, int bytes);

}  // namespace lakeb
