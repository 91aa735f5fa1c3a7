// Key-side phases of one 16-step chunk, shared by the chunked forward and
// backward kernels.  "Key side" = everything that depends on r, w, k, a, b
// only (not on the state or v); see wkv7_chunked_fwd.cu for the algebra.
//
// All functions are executed by one group of 4 warps (gw = warp index within
// the group, gtid = thread index within the group); the caller separates the
// phases with a group-wide named barrier.
#pragma once

#include "wkv7_common.cuh"
#include "wkv7_mma.cuh"
#include "wkv7_tma.cuh"

namespace camoe {
namespace ks {

using namespace camoe::mma;

constexpr int L = kChunk;  // 16
constexpr int LD = 72;     // padded row stride of 16 x 64 bf16 tiles (144 B: conflict-free ldmatrix)
constexpr int LDS = 24;    // padded row stride of 16 x 16 bf16 tiles

using Tile = bf16[L][LD];
using Tile16 = bf16[L][LDS];
// row stride of the fp32 16 x 64 prefix and log-decay tiles the backward keeps:
// 72 floats put the rows t, t + 1, t + 2, t + 3 read by one half-warp's float2
// loads (rows of 8 threads apart, columns 2q) on distinct banks (64 would map
// every row to the same banks)
constexpr int LDF = kN + 8;

// Phase 1 (SIMT): per column pair (2p, 2p+1), the log-decays lw =
// log_decay(w_in, kind), their inclusive prefix cum inside the chunk,
// Lam = exp(cum), and the scaled operands At = a exp(cum - lw), Rt = r Lam,
// Kb = k / Lam, Bb = b / Lam.  lam (the decay over the whole chunk) = Lam of
// the last step.  Thread layout: p = gtid / 4, tq = gtid % 4 (the four lanes of
// a column pair adjacent); lane tq owns rows 2tq, 2tq + 1 (first half) and
// 8 + 2tq, 9 + 2tq (second half), so the four rows one instruction touches are
// 2 apart, which puts them on different banks both in the swizzled TMA tiles
// and in the padded tiles (rows 8 apart share banks in both).  The prefix is
// two interleaved scans over the four lanes, one per half, the second offset
// by the first half's total.
// With `cum_out`/`lw_out` non-null, the fp32 prefixes and log-decays are kept
// for the backward.  Steps u >= nvalid (past the end of a sequence whose
// length is not a multiple of L) get lw = 0, so lam is the decay over the
// steps that exist and a final state taken after the chunk is exact.  The input tiles are 16 x 64 bf16, either row-major with
// stride LD (SWZ = false) or as landed by a swizzled TMA load (SWZ = true).
template <bool SWZ>
__device__ __forceinline__ int raw_idx(int u, int j) {
  return SWZ ? tma::swz(u, j) : u * LD + j;
}

__device__ __forceinline__ float2 exp_pair(float2 x) { return make_float2(__expf(x.x), __expf(x.y)); }
__device__ __forceinline__ float2 ld_bf2(const bf16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

// At, Rt are written through layout lar, Kb, Bb through layout lkb (16 x 64 bf16).
// The two columns of a pair run as packed two-lane fp32 operations
// (__fmul2_rn, __fadd2_rn: each lane rounded as the scalar operation).
template <bool SWZ, typename LAR, typename LKB>
__device__ __forceinline__ void decays(const bf16* rr, const bf16* ww, const bf16* kk,
                                       const bf16* aa, const bf16* bb, bf16* At, bf16* Rt, LAR lar,
                                       bf16* Kb, bf16* Bb, LKB lkb, float* lam, float (*cum_out)[LDF],
                                       float (*lw_out)[LDF], int gtid, int kind, int nvalid = L) {
  const int p = gtid >> 2, tq = gtid & 3, j = 2 * p;
  const int lane = gtid & 31;
  // the lane's rows: e = 0, 1 first half, e = 2, 3 second half
  int rows[4];
  rows[0] = 2 * tq;
  rows[1] = 2 * tq + 1;
  rows[2] = 8 + 2 * tq;
  rows[3] = 9 + 2 * tq;
  float2 lw[4];  // log-decays of the column pair, per row
#pragma unroll
  for (int e = 0; e < 4; ++e) lw[e] = ld_bf2(ww + raw_idx<SWZ>(rows[e], j));
  if (kind == kDecayWind) {  // uniform branch: one transform per call
#pragma unroll
    for (int e = 0; e < 4; ++e) lw[e] = __fmul2_rn(exp_pair(lw[e]), make_float2(-1.f, -1.f));
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 den = __fadd2_rn(exp_pair(make_float2(-lw[e].x, -lw[e].y)), make_float2(1.f, 1.f));
      lw[e] = __fmul2_rn(make_float2(__fdividef(1.0f, den.x), __fdividef(1.0f, den.y)),
                         make_float2(kWScale, kWScale));
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (rows[e] >= nvalid) lw[e] = make_float2(0.f, 0.f);
    if (lw_out != nullptr) *reinterpret_cast<float2*>(&lw_out[rows[e]][j]) = lw[e];
  }
  // inclusive scans over the four lanes of the half totals (h: first half, g: second)
  const float2 h = __fadd2_rn(lw[0], lw[1]), gs = __fadd2_rn(lw[2], lw[3]);
  float2 sh = h, sg = gs;
#pragma unroll
  for (int d = 1; d < 4; d <<= 1) {
    const float2 a = make_float2(__shfl_up_sync(0xffffffffu, sh.x, d), __shfl_up_sync(0xffffffffu, sh.y, d));
    const float2 b = make_float2(__shfl_up_sync(0xffffffffu, sg.x, d), __shfl_up_sync(0xffffffffu, sg.y, d));
    if (tq >= d) {
      sh = __fadd2_rn(sh, a);
      sg = __fadd2_rn(sg, b);
    }
  }
  // the first half's total sits in the pair's last lane
  const int last = (lane & ~3) | 3;
  const float2 tot = make_float2(__shfl_sync(0xffffffffu, sh.x, last), __shfl_sync(0xffffffffu, sh.y, last));
  // cum before each half's first row of this lane
  float2 off[2];
  off[0] = make_float2(sh.x - h.x, sh.y - h.y);
  off[1] = make_float2(tot.x + sg.x - gs.x, tot.y + sg.y - gs.y);
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float2 cu = off[hf];
    float2 px = exp_pair(cu);  // exp(cum) before the row
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      const int e = 2 * hf + x, u = rows[e];
      cu = __fadd2_rn(cu, lw[e]);
      if (cum_out != nullptr) *reinterpret_cast<float2*>(&cum_out[u][j]) = cu;
      const float2 Lc = exp_pair(cu), ic = exp_pair(make_float2(-cu.x, -cu.y));
      const int o = raw_idx<SWZ>(u, j);
      const float2 r = ld_bf2(rr + o), k = ld_bf2(kk + o), a = ld_bf2(aa + o), b = ld_bf2(bb + o);
      const float2 at = __fmul2_rn(a, px), rt = __fmul2_rn(r, Lc), kt = __fmul2_rn(k, ic), bt = __fmul2_rn(b, ic);
      *reinterpret_cast<__nv_bfloat162*>(At + lar(u, j)) = __floats2bfloat162_rn(at.x, at.y);
      *reinterpret_cast<__nv_bfloat162*>(Rt + lar(u, j)) = __floats2bfloat162_rn(rt.x, rt.y);
      *reinterpret_cast<__nv_bfloat162*>(Kb + lkb(u, j)) = __floats2bfloat162_rn(kt.x, kt.y);
      *reinterpret_cast<__nv_bfloat162*>(Bb + lkb(u, j)) = __floats2bfloat162_rn(bt.x, bt.y);
      px = Lc;
    }
    if (hf == 1 && tq == 3) *reinterpret_cast<float2*>(&lam[j]) = px;  // row 15
  }
}

// Phase 2 (tensor cores): the four 16x16 Gram blocks, warp gw computes block gw:
//   0: Ga = strict(At Bb^T) (fp32)   1: Bm = strict(At Kb^T)
//   2: Cm = lower(Rt Bb^T)           3: Dm = lower(Rt Kb^T)
template <typename LAR, typename LKB>
__device__ __forceinline__ void grams(const bf16* At, const bf16* Rt, LAR lar, const bf16* Bb,
                                      const bf16* Kb, LKB lkb, float (*Ga)[L + 1], Tile16& Bm,
                                      Tile16& Cm, Tile16& Dm, int gw, int lane) {
  const bf16* Am = (gw >> 1) ? Rt : At;
  const bf16* Bn = (gw & 1) ? Kb : Bb;
  float acc[2][4] = {};
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4], b[4];
    lda_rm(a, Am, lar, 0, kk * 16, lane);
    ldb_nk(b, Bn, lkb, 0, kk * 16, lane);
    mma16816(acc[0], a, b[0], b[1]);
    mma16816(acc[1], a, b[2], b[3]);
  }
  const int g = lane >> 2, q = lane & 3;
  const bool strict = gw < 2;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = g + (e >= 2 ? 8 : 0), s = 8 * nt + 2 * q + (e & 1);
      const bool keep = strict ? (s < t) : (s <= t);
      acc[nt][e] = keep ? acc[nt][e] : 0.f;
    }
  if (gw == 0) {
    store_acc_f32(&Ga[0][0], L + 1, 0, 0, acc[0], lane);
    store_acc_f32(&Ga[0][0], L + 1, 0, 8, acc[1], lane);
  } else {
    bf16* dst = gw == 1 ? &Bm[0][0] : gw == 2 ? &Cm[0][0] : &Dm[0][0];
    store_acc_bf16(dst, LDS, 0, 0, acc[0], lane);
    store_acc_bf16(dst, LDS, 0, 8, acc[1], lane);
  }
}

// Phase 3 (one warp): Tf = (I - Ga)^{-1} (lower unitriangular) by 8x8 blocks
// in fp32 (forward substitution per column, then T21 = T22 A21 T11), Ti = bf16(Tf).
__device__ __forceinline__ void inverse(const float (*Ga)[L + 1], float (*Tf)[L + 1],
                                        float (*Mf)[9], Tile16& Ti, int lane) {
  if (lane < 16) {
    const int o = (lane >> 3) * 8, c = lane & 7;
    float x[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float acc = (r == c) ? 1.f : 0.f;
#pragma unroll
      for (int s = 0; s < r; ++s) acc += Ga[o + r][o + s] * x[s];
      x[r] = acc;  // x[s] == 0 for s < c: the column starts at its diagonal
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) Tf[o + r][o + c] = x[r];
  }
  __syncwarp();
#pragma unroll
  for (int e2 = 0; e2 < 2; ++e2) {  // M = A21 T11
    const int e = lane + 32 * e2, r = e >> 3, c = e & 7;
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) acc += Ga[8 + r][s] * Tf[s][c];
    Mf[r][c] = acc;
  }
  __syncwarp();
#pragma unroll
  for (int e2 = 0; e2 < 2; ++e2) {  // T21 = T22 M
    const int e = lane + 32 * e2, r = e >> 3, c = e & 7;
    float acc = 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m) acc += Tf[8 + r][8 + m] * Mf[m][c];
    Tf[8 + r][c] = acc;
  }
  __syncwarp();
#pragma unroll
  for (int e8 = 0; e8 < 8; ++e8) {
    const int e = lane + 32 * e8, r = e >> 4, c = e & 15;
    const bool upper = c > r;
    const float v = upper ? 0.f : Tf[r][c];
    if (upper) Tf[r][c] = 0.f;
    Ti[r][c] = __float2bfloat16_rn(v);
  }
}

// Phase 4a: W = Ti At (warp gw: columns 16gw..16gw+15); Q = Ti Bm (warp 3).
// At is read through lar, W written through lw, Q through lq.
template <typename LAR, typename LW, typename LQ>
__device__ __forceinline__ void w_and_q(const Tile16& Ti, const bf16* At, LAR lar, const Tile16& Bm,
                                        bf16* W, LW lw, bf16* Q, LQ lq, int gw, int lane) {
  uint32_t a[4], b[4];
  lda_rowmajor(a, &Ti[0][0], LDS, 0, 0, lane);
  ldb_kn(b, At, lar, 16 * gw, 0, lane);
  float acc[2][4] = {};
  mma16816(acc[0], a, b[0], b[1]);
  mma16816(acc[1], a, b[2], b[3]);
  store_acc_lay(W, lw, 0, 16 * gw, acc[0], lane);
  store_acc_lay(W, lw, 0, 16 * gw + 8, acc[1], lane);
  if (gw == 3) {
    float qa[2][4] = {};
    ldb_kn(b, &Bm[0][0], LDS, 0, 0, lane);
    mma16816(qa[0], a, b[0], b[1]);
    mma16816(qa[1], a, b[2], b[3]);
    store_acc_lay(Q, lq, 0, 0, qa[0], lane);
    store_acc_lay(Q, lq, 0, 8, qa[1], lane);
  }
}

// accumulator pair initialised from a bf16 tile (through layout lay) at (m0, n0)
template <typename Lay>
__device__ __forceinline__ void acc_from_bf16(float (&c)[4], const bf16* tile, Lay lay, int m0,
                                              int n0, int lane) {
  const int g = lane >> 2, q = lane & 3;
  const float2 lo = __bfloat1622float2(
      *reinterpret_cast<const __nv_bfloat162*>(tile + lay(m0 + g, n0 + 2 * q)));
  const float2 hi = __bfloat1622float2(
      *reinterpret_cast<const __nv_bfloat162*>(tile + lay(m0 + g + 8, n0 + 2 * q)));
  c[0] = lo.x; c[1] = lo.y; c[2] = hi.x; c[3] = hi.y;
}

// Phase 4b: Qy = Rt + Cm W (warp gw: columns 16gw..); P = Cm Q + Dm (warp 2).
// W is read through lw, Rt through lar, Q through lq; Qy written through lqy, P through lp.
template <typename LW, typename LAR, typename LQ, typename LQY, typename LP>
__device__ __forceinline__ void qy_and_p(const Tile16& Cm, const bf16* W, LW lw, const bf16* Rt,
                                         LAR lar, const bf16* Q, LQ lq, const Tile16& Dm, bf16* Qy,
                                         LQY lqy, bf16* P, LP lp, int gw, int lane) {
  uint32_t a[4], b[4];
  lda_rowmajor(a, &Cm[0][0], LDS, 0, 0, lane);
  ldb_kn(b, W, lw, 16 * gw, 0, lane);
  float acc[2][4];
  acc_from_bf16(acc[0], Rt, lar, 0, 16 * gw, lane);
  acc_from_bf16(acc[1], Rt, lar, 0, 16 * gw + 8, lane);
  mma16816(acc[0], a, b[0], b[1]);
  mma16816(acc[1], a, b[2], b[3]);
  store_acc_lay(Qy, lqy, 0, 16 * gw, acc[0], lane);
  store_acc_lay(Qy, lqy, 0, 16 * gw + 8, acc[1], lane);
  if (gw == 2) {
    float pa[2][4];
    acc_from_bf16(pa[0], &Dm[0][0], Padded{LDS}, 0, 0, lane);
    acc_from_bf16(pa[1], &Dm[0][0], Padded{LDS}, 0, 8, lane);
    ldb_kn(b, Q, lq, 0, 0, lane);
    mma16816(pa[0], a, b[0], b[1]);
    mma16816(pa[1], a, b[2], b[3]);
    store_acc_lay(P, lp, 0, 0, pa[0], lane);
    store_acc_lay(P, lp, 0, 8, pa[1], lane);
  }
}

}  // namespace ks
}  // namespace camoe
