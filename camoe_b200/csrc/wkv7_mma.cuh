// Warp-level bf16 tensor-core helpers (mma.sync m16n8k16, fp32 accumulate)
// and fragment conventions used by the chunked WKV-7 kernels.
//
// Fragment layout of mma.m16n8k16.row.col (g = lane / 4, q = lane % 4):
//   A (16x16, M x K):  a0 = (g, 2q..2q+1)   a1 = (g+8, 2q..2q+1)
//                      a2 = (g, 2q+8..+9)   a3 = (g+8, 2q+8..+9)
//   B (16x8,  K x N):  b0 = (2q..2q+1, g)   b1 = (2q+8..+9, g)
//   C (16x8,  M x N):  c0,c1 = (g, 2q..2q+1)  c2,c3 = (g+8, 2q..2q+1)
// so the accumulators of two adjacent n8 tiles are exactly the A fragment of
// one k16 step (acc_to_a), which keeps chained products in registers.
//
// Shared-memory tiles are bf16, row-major with a padded row stride, read with
// ldmatrix:  A from [m][k] storage (lda_rowmajor) or [k][m] storage
// (lda_colmajor, .trans);  B from [n][k] storage (ldb_nk) or [k][n] storage
// (ldb_kn, .trans).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace camoe {
namespace mma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void stsm_x4(void* p, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(smem_u32(p)),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void stsm_x4_t(void* p, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(smem_u32(p)),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// A fragment (16 x 16 at rows m0.., cols k0..) from a row-major [m][k] tile.
__device__ __forceinline__ void lda_rowmajor(uint32_t (&a)[4], const __nv_bfloat16* tile,
                                             int ld, int m0, int k0, int lane) {
  const int r = m0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = k0 + (lane >> 4) * 8;
  ldsm_x4(a, tile + r * ld + c);
}

// A fragment (16 x 16, A[m][k] = tile[k][m]) from a [k][m] tile.
__device__ __forceinline__ void lda_colmajor(uint32_t (&a)[4], const __nv_bfloat16* tile,
                                             int ld, int m0, int k0, int lane) {
  const int k = k0 + (lane & 7) + (lane >> 4) * 8;
  const int m = m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(a, tile + k * ld + m);
}

// B fragments of two n8 tiles (n0..n0+7 -> b[0],b[1]; n0+8..n0+15 -> b[2],b[3])
// for k0..k0+15, from an [n][k] tile (B[k][n] = tile[n][k]).
__device__ __forceinline__ void ldb_nk(uint32_t (&b)[4], const __nv_bfloat16* tile, int ld,
                                       int n0, int k0, int lane) {
  const int n = n0 + (lane & 7) + (lane >> 4) * 8;
  const int k = k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(b, tile + n * ld + k);
}

// Same from a [k][n] tile (B[k][n] = tile[k][n]).
__device__ __forceinline__ void ldb_kn(uint32_t (&b)[4], const __nv_bfloat16* tile, int ld,
                                       int n0, int k0, int lane) {
  const int k = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int n = n0 + (lane >> 4) * 8;
  ldsm_x4_t(b, tile + k * ld + n);
}

// Accumulators of n8 tiles (2kk, 2kk+1) -> bf16 A fragment of k-step kk.
__device__ __forceinline__ void acc_to_a(uint32_t (&a)[4], const float (&c0)[4],
                                         const float (&c1)[4]) {
  a[0] = pack_bf16(c0[0], c0[1]);
  a[1] = pack_bf16(c0[2], c0[3]);
  a[2] = pack_bf16(c1[0], c1[1]);
  a[3] = pack_bf16(c1[2], c1[3]);
}

// Store an accumulator tile (16 x 8 at rows m0, cols n0) as bf16 into a [m][n] tile.
__device__ __forceinline__ void store_acc_bf16(__nv_bfloat16* tile, int ld, int m0, int n0,
                                               const float (&c)[4], int lane) {
  const int g = lane >> 2, q = lane & 3;
  *reinterpret_cast<__nv_bfloat162*>(tile + (m0 + g) * ld + n0 + 2 * q) =
      __floats2bfloat162_rn(c[0], c[1]);
  *reinterpret_cast<__nv_bfloat162*>(tile + (m0 + g + 8) * ld + n0 + 2 * q) =
      __floats2bfloat162_rn(c[2], c[3]);
}

// Store an accumulator tile transposed: tile[n][m] (bf16).
__device__ __forceinline__ void store_acc_bf16_t(__nv_bfloat16* tile, int ld, int m0, int n0,
                                                 const float (&c)[4], int lane) {
  const int g = lane >> 2, q = lane & 3;
  tile[(n0 + 2 * q) * ld + m0 + g] = __float2bfloat16_rn(c[0]);
  tile[(n0 + 2 * q + 1) * ld + m0 + g] = __float2bfloat16_rn(c[1]);
  tile[(n0 + 2 * q) * ld + m0 + g + 8] = __float2bfloat16_rn(c[2]);
  tile[(n0 + 2 * q + 1) * ld + m0 + g + 8] = __float2bfloat16_rn(c[3]);
}

// Store an accumulator tile as fp32 into a [m][n] tile.
__device__ __forceinline__ void store_acc_f32(float* tile, int ld, int m0, int n0,
                                              const float (&c)[4], int lane) {
  const int g = lane >> 2, q = lane & 3;
  tile[(m0 + g) * ld + n0 + 2 * q] = c[0];
  tile[(m0 + g) * ld + n0 + 2 * q + 1] = c[1];
  tile[(m0 + g + 8) * ld + n0 + 2 * q] = c[2];
  tile[(m0 + g + 8) * ld + n0 + 2 * q + 1] = c[3];
}

// ---- layout-generic loaders --------------------------------------------------
// A layout maps (row, column) of a bf16 tile to an element offset; row starts
// of 8-column (16-byte) pieces must be 16-byte aligned.
struct Padded {  // row-major with padded row stride
  int ld;
  __device__ __forceinline__ int operator()(int r, int c) const { return r * ld + c; }
};
struct Swz64 {  // 64 columns, 128-byte rows, 16-byte pieces XOR-swizzled by (row & 7)
  __device__ __forceinline__ int operator()(int r, int c) const {
    return r * 64 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7);
  }
};
struct Swz16 {  // 16 columns, 32-byte rows, the two pieces swizzled by bit 2 of the row
  __device__ __forceinline__ int operator()(int r, int c) const {
    return r * 16 + ((((c >> 3) ^ ((r >> 2) & 1))) << 3) + (c & 7);
  }
};

template <typename Lay>
__device__ __forceinline__ void lda_rm(uint32_t (&a)[4], const __nv_bfloat16* tile, Lay lay,
                                       int m0, int k0, int lane) {
  ldsm_x4(a, tile + lay(m0 + (lane & 7) + ((lane >> 3) & 1) * 8, k0 + (lane >> 4) * 8));
}
template <typename Lay>
__device__ __forceinline__ void lda_cm(uint32_t (&a)[4], const __nv_bfloat16* tile, Lay lay,
                                       int m0, int k0, int lane) {
  ldsm_x4_t(a, tile + lay(k0 + (lane & 7) + (lane >> 4) * 8, m0 + ((lane >> 3) & 1) * 8));
}
template <typename Lay>
__device__ __forceinline__ void ldb_nk(uint32_t (&b)[4], const __nv_bfloat16* tile, Lay lay,
                                       int n0, int k0, int lane) {
  ldsm_x4(b, tile + lay(n0 + (lane & 7) + (lane >> 4) * 8, k0 + ((lane >> 3) & 1) * 8));
}
template <typename Lay>
__device__ __forceinline__ void ldb_kn(uint32_t (&b)[4], const __nv_bfloat16* tile, Lay lay,
                                       int n0, int k0, int lane) {
  ldsm_x4_t(b, tile + lay(k0 + (lane & 7) + ((lane >> 3) & 1) * 8, n0 + (lane >> 4) * 8));
}

// Store an accumulator tile (16 x 8 at rows m0, cols n0) as bf16 through a layout
// (shared or global memory).
template <typename Lay>
__device__ __forceinline__ void store_acc_lay(__nv_bfloat16* tile, Lay lay, int m0, int n0,
                                              const float (&c)[4], int lane) {
  const int g = lane >> 2, q = lane & 3;
  *reinterpret_cast<__nv_bfloat162*>(tile + lay(m0 + g, n0 + 2 * q)) =
      __floats2bfloat162_rn(c[0], c[1]);
  *reinterpret_cast<__nv_bfloat162*>(tile + lay(m0 + g + 8, n0 + 2 * q)) =
      __floats2bfloat162_rn(c[2], c[3]);
}

// Store a bf16 A fragment (16 x 16 at rows m0, cols k0) through a layout.
template <typename Lay>
__device__ __forceinline__ void store_a_lay(__nv_bfloat16* tile, Lay lay, int m0, int k0,
                                            const uint32_t (&a)[4], int lane) {
  const int g = lane >> 2, q = lane & 3;
  *reinterpret_cast<uint32_t*>(tile + lay(m0 + g, k0 + 2 * q)) = a[0];
  *reinterpret_cast<uint32_t*>(tile + lay(m0 + g + 8, k0 + 2 * q)) = a[1];
  *reinterpret_cast<uint32_t*>(tile + lay(m0 + g, k0 + 8 + 2 * q)) = a[2];
  *reinterpret_cast<uint32_t*>(tile + lay(m0 + g + 8, k0 + 8 + 2 * q)) = a[3];
}

// Inverses of lda_rm / lda_cm: store a bf16 A fragment (16 x 16 at rows m0,
// cols k0) into a [m][k] tile, or transposed into a [k][m] tile (stmatrix).
template <typename Lay>
__device__ __forceinline__ void sta_rm(__nv_bfloat16* tile, Lay lay, int m0, int k0,
                                       const uint32_t (&a)[4], int lane) {
  stsm_x4(tile + lay(m0 + (lane & 7) + ((lane >> 3) & 1) * 8, k0 + (lane >> 4) * 8), a);
}
template <typename Lay>
__device__ __forceinline__ void sta_cm(__nv_bfloat16* tile, Lay lay, int m0, int k0,
                                       const uint32_t (&a)[4], int lane) {
  stsm_x4_t(tile + lay(k0 + (lane & 7) + (lane >> 4) * 8, m0 + ((lane >> 3) & 1) * 8), a);
}

// acc (16 x 16) = A (16 x 64, four k-step fragments) M + V (16 x 16) N, with
// M and N given as B fragments.  Even and odd k-steps accumulate separately
// (two dependent chains of depth 3 instead of one of depth 5) and are summed.
__device__ __forceinline__ void mma_k64_k16(float (&acc)[2][4], const uint32_t (&a)[4][4],
                                            const uint32_t (&v)[4], const uint32_t (&bM)[4][4],
                                            const uint32_t (&bN)[4]) {
  float o[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = o[nt][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 4; kk += 2) {
    mma16816(acc[0], a[kk], bM[kk][0], bM[kk][1]);
    mma16816(acc[1], a[kk], bM[kk][2], bM[kk][3]);
    mma16816(o[0], a[kk + 1], bM[kk + 1][0], bM[kk + 1][1]);
    mma16816(o[1], a[kk + 1], bM[kk + 1][2], bM[kk + 1][3]);
  }
  mma16816(o[0], v, bN[0], bN[1]);
  mma16816(o[1], v, bN[2], bN[3]);
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] += o[nt][e];
}

// acc (16 x 16 output at columns n0) += A (16 x 16*KS) B;
// AT: A stored [k][m] (else [m][k]); BT: B stored [k][n] (else [n][k]).
template <bool AT, bool BT, int KS, typename LA, typename LB>
__device__ __forceinline__ void mm16(float (&acc)[2][4], const __nv_bfloat16* A, LA la,
                                     const __nv_bfloat16* B, LB lb, int n0, int lane) {
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    uint32_t a[4], b[4];
    if (AT) lda_cm(a, A, la, 0, 16 * kk, lane); else lda_rm(a, A, la, 0, 16 * kk, lane);
    if (BT) ldb_kn(b, B, lb, n0, 16 * kk, lane); else ldb_nk(b, B, lb, n0, 16 * kk, lane);
    mma16816(acc[0], a, b[0], b[1]);
    mma16816(acc[1], a, b[2], b[3]);
  }
}

}  // namespace mma
}  // namespace camoe
