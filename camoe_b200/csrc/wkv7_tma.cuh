// TMA (cp.async.bulk.tensor) helpers: host-side tensor-map encoding for the
// [B, T, H, N] operand arrays and the device-side tile load.
//
// Each operand is described to the TMA unit as a 4-D tensor (N, H, T, B)
// with N innermost, so one 16-step chunk of one head is a {64, 1, 16, 1} box:
// 16 rows of 128 bytes.  Rows past T are out of bounds in the T dimension and
// arrive zero-filled.  The box lands in shared memory with the 128-byte
// swizzle: the 16-byte piece k of row r is stored at piece k ^ (r & 7), which
// keeps row-parallel shared-memory reads free of bank conflicts.  Loads start
// at x = 0 or, for column-range boxes, at a column offset whose byte offset is
// a multiple of 16; no load writes global memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace camoe {
namespace tma {

constexpr int kRowBytes = 128;             // 64 bf16
constexpr int kTileBytes = 16 * kRowBytes;  // one 16-step chunk of one head

// element offset of (row r, column c) inside a swizzled 16 x 64 bf16 tile
__host__ __device__ __forceinline__ int swz(int r, int c) {
  return r * 64 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7);
}

// Make the calling thread's current device's primary context current for the
// driver before tensor maps are encoded (cuTensorMapEncodeTiled is a driver
// call and fails on a thread with no current context, e.g. a framework's
// backward worker thread that has launched nothing yet).  Returns false when
// the runtime has no usable device.
bool bind_context();

// Encode the (N, H, T, B) map of a bf16 [B, T, H, 64] array; returns false on failure.
bool encode_bhtn(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H);
// Same for an fp32 array, without swizzle: a chunk lands as a plain [16][64] fp32 tile.
bool encode_bhtn_f32(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H);

// Map of a bf16 (or, with f32, fp32) [B, T, H, 64] array with a
// {n_box, 1, 16, 1} box and no swizzle (rows of n_box columns, row-major in
// shared memory), for stores of a column range of one chunk.
bool encode_bhtn_cols(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H,
                      int n_box, bool f32);

// Map of a row-major bf16 [rows, inner] matrix with a {64, box_rows} box and
// the 128-byte swizzle (each box lands as box_rows rows of 128 bytes, 16-byte
// pieces XOR-swizzled by row % 8); boxes past either extent read zeros.
// inner x 2 bytes must be a multiple of 16.
bool encode_2d_sw128(CUtensorMap* map, const void* base, int64_t inner, int64_t rows,
                     int box_rows);

// Load the box at (x, y) of a 2-D map, completing on `bar`.
__device__ __forceinline__ void load_2d(void* dst_smem, const CUtensorMap* map, int x, int y,
                                        uint64_t* bar) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  const uint32_t mb = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mb)
      : "memory");
}

__device__ __forceinline__ void load_tile(void* dst_smem, const CUtensorMap* map, int h,
                                          int t0, int b, uint64_t* bar) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  const uint32_t mb = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(h), "r"(t0), "r"(b), "r"(mb)
      : "memory");
}

// Same with the box starting at column n0 (n0 x element size a multiple of 16 bytes).
__device__ __forceinline__ void load_tile_at(void* dst_smem, const CUtensorMap* map, int n0, int h,
                                             int t0, int b, uint64_t* bar) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  const uint32_t mb = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(n0), "r"(h), "r"(t0), "r"(b), "r"(mb)
      : "memory");
}

// Store one chunk box from shared memory at columns n0.. of head h, steps
// t0.., batch b (bulk-group completion; rows past T are not written).
__device__ __forceinline__ void store_tile(const CUtensorMap* map, const void* src_smem, int n0,
                                           int h, int t0, int b) {
  const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(src_smem));
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];\n" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(n0), "r"(h), "r"(t0), "r"(b), "r"(src)
      : "memory");
}

}  // namespace tma
}  // namespace camoe
