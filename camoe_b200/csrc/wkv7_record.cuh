// Per-chunk records that the chunked kernels exchange through global memory,
// and the state checkpoint, all inside the caller's checkpoint buffer or the
// backward workspace.
//
// Checkpoint buffer (written by the forward, read by the backward), for
// `chains` chains of `nchunk` 16-step chunks:
//   [chains][nchunk] KeyRec      key-side matrices of every chunk
//   [chains][nchunk] TriRec      the chunk's triangular inverse and two Gram
//                                blocks, for the key-side backward
//   [chains][nstate] state       bf16 64x64 state at the start of chunks
//                                2, 4, 6, ... (rows of 128 bytes, 16-byte
//                                pieces swizzled by row & 7)
// nstate = (nchunk - 1) / 2; the state at the start of odd chunks is
// recomputed from the preceding even one, chunk 0 starts from zero.  Per
// chunk this is 9472 + 2624 + 4096 bytes, below the 16 KiB per chunk of the
// reference's [B, H, T/16, 64, 64] fp32 checkpoint tensor.
//
// Backward workspace: [chains][nchunk] XRec.
#pragma once

#include "wkv7_common.cuh"

namespace camoe {
namespace rec {

// 16 x 64 bf16 tiles are stored Swz64, 16 x 16 tiles Swz16 (see wkv7_mma.cuh),
// so a bulk copy lands them in shared memory ready for conflict-free ldmatrix.
struct KeyRec {
  bf16 W[16 * 64], Qy[16 * 64], Bb[16 * 64], Kb[16 * 64];
  bf16 Q[16 * 16], P[16 * 16];
  float lam[64];
};
static_assert(sizeof(KeyRec) == 9472, "KeyRec layout");

// Ti = (I - A)^{-1} in fp32 (upper triangle zero), Bm = strict(At Kb^T) and
// Cm = lower(Rt Bb^T) in bf16, in the padded shared-memory layouts of the
// key-side kernels ([16][17] fp32, [16][24] bf16), so a bulk copy lands them
// ready for use.
struct TriRec {
  float Tf[16][17];
  bf16 Bm[16][24], Cm[16][24];
};
static_assert(sizeof(TriRec) == 2624, "TriRec layout");

// What the value-side backward hands to the key-side backward for one chunk:
// bf16 copies of the chunk's start state S, of G'' = dL/dS' diag(lam), of SA^T
// and dSA^T (rows = state row i).  S is written only for chunks 0, 1 and the
// odd chunks; for even chunks from 2 on the space stays unwritten and the
// reader takes the start state from the forward's state checkpoint instead.
struct XRec {
  bf16 S[64 * 64];     // Swz64 layout over 64 rows
  bf16 G[64 * 64];     // Swz64
  bf16 SAT[64 * 16];   // Swz16 layout over 64 rows
  bf16 dSAT[64 * 16];  // Swz16
};
static_assert(sizeof(XRec) % 16 == 0, "XRec size");

constexpr int64_t kStateBytes = 64 * 64 * 2;

__host__ __device__ __forceinline__ int64_t nstate(int64_t nchunk) {
  return nchunk > 0 ? (nchunk - 1) / 2 : 0;
}
__host__ __device__ __forceinline__ size_t ckpt_bytes(int64_t chains, int64_t nchunk) {
  return static_cast<size_t>(chains * nchunk) * (sizeof(KeyRec) + sizeof(TriRec)) +
         static_cast<size_t>(chains * nstate(nchunk)) * kStateBytes;
}
// inference forward through the two-kernel path: the KeyRecs only
__host__ __device__ __forceinline__ size_t infer_bytes(int64_t chains, int64_t nchunk) {
  return static_cast<size_t>(chains * nchunk) * sizeof(KeyRec);
}
__host__ __device__ __forceinline__ size_t work_bytes(int64_t chains, int64_t nchunk) {
  return static_cast<size_t>(chains * nchunk) * sizeof(XRec);
}
__device__ __forceinline__ KeyRec* keyrec(void* ckpt, int64_t ch, int64_t nchunk, int64_t c) {
  return reinterpret_cast<KeyRec*>(ckpt) + (ch * nchunk + c);
}
__device__ __forceinline__ TriRec* trirec(void* ckpt, int64_t chains, int64_t ch, int64_t nchunk,
                                          int64_t c) {
  char* base = reinterpret_cast<char*>(ckpt) + chains * nchunk * sizeof(KeyRec);
  return reinterpret_cast<TriRec*>(base) + (ch * nchunk + c);
}
// state at the start of even chunk c >= 2
__device__ __forceinline__ char* state_ptr(void* ckpt, int64_t chains, int64_t ch,
                                           int64_t nchunk, int64_t c) {
  char* base = reinterpret_cast<char*>(ckpt) + chains * nchunk * (sizeof(KeyRec) + sizeof(TriRec));
  return base + (ch * nstate(nchunk) + (c / 2 - 1)) * kStateBytes;
}
__device__ __forceinline__ XRec* xrec(void* work, int64_t ch, int64_t nchunk, int64_t c) {
  return reinterpret_cast<XRec*>(work) + (ch * nchunk + c);
}

}  // namespace rec

// The sequential value kernels split a chain's 64 state rows (independent in
// the recurrence) over 4 / RB CTAs of RB 16-row blocks: as many CTAs as the
// SMs hold at once, at most 4 per chain.
// Role index of hardware warp w in the value kernels, whose roles are laid
// out as [3 RB compute warps][producer][store].  Warp w runs on SMSP w % 4;
// with RB == 2 the producer and store roles move to warps 4 and 5, so the two
// recurrence warps (0, 1) share their SMSPs only with those light warps.
template <int RB>
__device__ __forceinline__ int role_warp(int w) {
  if (RB != 2) return w;
  return w < 4 ? w : (w < 6 ? w + 2 : w - 2);
}

inline int rows_per_cta(int64_t chains, int sms) {
  if (chains * 4 <= sms) return 1;
  if (chains * 2 <= sms) return 2;
  return 4;
}
}  // namespace camoe
