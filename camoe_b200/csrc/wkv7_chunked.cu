// Chunked WKV-7 ClampW on the tensor cores (bf16 operands, fp32 accumulate
// and fp32 state), the bf16 path of the operator.
//
// Per chain (b, h), chunks of L = 16 steps are processed in order.  With the
// log-decay lw = -e^{-1/2} sigmoid(w_in) (camoe/cuda/rwkv7_clampw.cu:42),
// cum_t = sum_{s<=t} lw_s inside the chunk, Lam = exp(cum), Lamx = exp(cum - lw)
// and lam = Lam_{L-1}, the 16 steps of
//     S_t = S_{t-1} (diag w_t + a_t b_t^T) + v_t k_t^T,  y_t = S_t r_t,  sa_t = S_{t-1} a_t
// starting from the state S (rows = value index i, columns = key index j) are
//     SA = W S^T + Q V          (L x N, row t = sa_t)
//     Y  = Qy S^T + P V
//     S' = S diag(lam) + SA^T Bh + V^T Kh
// with the "key-side" matrices, which depend on r, w, k, a, b only:
//     At = a*Lamx, Rt = r*Lam, Kb = k/Lam, Bb = b/Lam, Bh = Bb*lam, Kh = Kb*lam
//     A  = strict_lower(At Bb^T), Bm = strict_lower(At Kb^T),
//     Cm = lower(Rt Bb^T),        Dm = lower(Rt Kb^T),     Ti = (I - A)^{-1}
//     W = Ti At, Q = Ti Bm, Qy = Rt + Cm W, P = Cm Q + Dm.
// (the intra-chunk solve is the WY / UT-transform form of chunked delta-rule
// recurrences, e.g. Yang et al. 2024, "Parallelizing Linear Transformers with
// the Delta Rule over Sequence Length").  ClampW bounds every decay below by
// exp(-e^{-1/2}) = 0.545, so 1/Lam <= 0.545^-16 ~ 1.6e4 and no factor over- or
// underflows in bf16/fp32.
//
// Work split: one CTA of 4 warps per chain.  The key-side matrices of a chunk
// are computed by all warps together (SIMT for the decays and the 16x16
// triangular inverse, mma.sync for the products).  Warp w owns state rows
// 16w..16w+15 for the whole sequence as mma accumulators (32 fp32 registers
// per thread); its SA, Y and state products chain in registers (accumulators
// reused as A fragments).  Inputs stream through a 3-deep cp.async ring.
#include "wkv7_common.cuh"
#include "wkv7_mma.cuh"

namespace camoe {
namespace chunked {

using namespace camoe::mma;

constexpr int L = kChunk;    // 16 steps per chunk
constexpr int LD = 72;       // padded row stride (elements) of 64-wide bf16 tiles
constexpr int LDS = 24;      // padded row stride of 16-wide bf16 tiles
constexpr int NST = 3;       // input ring depth
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kNumIn = 6;    // r, w, k, a, b, v
enum { IN_R = 0, IN_W = 1, IN_K = 2, IN_A = 3, IN_B = 4, IN_V = 5 };

// Key-side matrices of one chunk.
struct KeySide {
  bf16 At[L][LD], Rt[L][LD], Kb[L][LD], Bb[L][LD], Bh[L][LD], Kh[L][LD];
  bf16 W[L][LD], Qy[L][LD];
  bf16 Bm[L][LDS], Cm[L][LDS], Dm[L][LDS], Ti[L][LDS], Q[L][LDS], P[L][LDS];
  float Ga[L][L + 1];   // strictly lower A (fp32), input of the inverse
  float Tf[L][L + 1];   // (I - A)^{-1} in fp32
  float Mf[8][9];       // scratch of the blocked inverse
  float lam[kN];        // decay over the whole chunk
  float cum[L][kN];     // inclusive log-decay prefix (fp32), for the backward
  float sig[L][kN];     // sigmoid(w_in), for the backward
};

struct FwdSmem {
  bf16 raw[NST][kNumIn][L][LD];
  KeySide ks;
};

__device__ __forceinline__ const bf16* in_ptr(const FwdArgs& p, int t) {
  const void* v = t == IN_R ? p.r : t == IN_W ? p.w : t == IN_K ? p.k : t == IN_A ? p.a
                : t == IN_B ? p.b : p.v;
  return static_cast<const bf16*>(v);
}

// cp.async the 16 x 64 tiles of `n` tensors of chunk c into dst[n][L][LD]
template <typename GetPtr>
__device__ __forceinline__ void issue_tiles(bf16 (*dst)[L][LD], int n, GetPtr get, int64_t cbase,
                                            int64_t ts, int64_t T, int64_t c, int tid,
                                            int nthreads) {
  const int64_t t0 = c * L;
  for (int idx = tid; idx < n * L * 8; idx += nthreads) {
    const int tens = idx / (L * 8), rem = idx % (L * 8);
    const int u = rem >> 3, part = rem & 7;
    const bool ok = t0 + u < T;
    const bf16* src = get(tens) + (ok ? cbase + (t0 + u) * ts + part * 8 : 0);
    cp_async16(&dst[tens][u][part * 8], src, ok);
  }
}

// Phase K1: decays and the scaled operand tiles.  Thread -> (column j, half h).
__device__ __forceinline__ void keyside_decays(KeySide& ks, const bf16 (*raw)[L][LD], int tid) {
  const int j = tid >> 1, h = tid & 1;
  float lwv[8], cumv[8];
  float cacc = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int u = 8 * h + e;
    const float x = __bfloat162float(raw[IN_W][u][j]);
    const float sg = 1.0f / (1.0f + __expf(-x));
    ks.sig[u][j] = sg;
    const float lw = kWScale * sg;
    cacc += lw;
    lwv[e] = lw;
    cumv[e] = cacc;
  }
  const float other = __shfl_xor_sync(0xffffffffu, cacc, 1);
  const float off = h ? other : 0.f;
  const float total = h ? other + cacc : cacc + other;
  const float lamv = __expf(total);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int u = 8 * h + e;
    const float c = off + cumv[e];
    ks.cum[u][j] = c;
    const float Lam = __expf(c), Lamx = __expf(c - lwv[e]), iLam = __expf(-c);
    const float fin = lamv * iLam;
    const float r = __bfloat162float(raw[IN_R][u][j]), k = __bfloat162float(raw[IN_K][u][j]);
    const float a = __bfloat162float(raw[IN_A][u][j]), b = __bfloat162float(raw[IN_B][u][j]);
    ks.At[u][j] = __float2bfloat16_rn(a * Lamx);
    ks.Rt[u][j] = __float2bfloat16_rn(r * Lam);
    ks.Kb[u][j] = __float2bfloat16_rn(k * iLam);
    ks.Bb[u][j] = __float2bfloat16_rn(b * iLam);
    ks.Bh[u][j] = __float2bfloat16_rn(b * fin);
    ks.Kh[u][j] = __float2bfloat16_rn(k * fin);
  }
  if (h) ks.lam[j] = lamv;
}

// Phase K2: the four 16x16 Gram blocks, one per warp.
__device__ __forceinline__ void keyside_grams(KeySide& ks, int wq, int lane) {
  const bf16* Am = (wq >> 1) ? &ks.Rt[0][0] : &ks.At[0][0];
  const bf16* Bn = (wq & 1) ? &ks.Kb[0][0] : &ks.Bb[0][0];
  float acc[2][4] = {};
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4], b[4];
    lda_rowmajor(a, Am, LD, 0, kk * 16, lane);
    ldb_nk(b, Bn, LD, 0, kk * 16, lane);
    mma16816(acc[0], a, b[0], b[1]);
    mma16816(acc[1], a, b[2], b[3]);
  }
  const int g = lane >> 2, q = lane & 3;
  const bool strict = wq < 2;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = g + (e >= 2 ? 8 : 0), s = 8 * nt + 2 * q + (e & 1);
      const bool keep = strict ? (s < t) : (s <= t);
      acc[nt][e] = keep ? acc[nt][e] : 0.f;
    }
  if (wq == 0) {
    store_acc_f32(&ks.Ga[0][0], L + 1, 0, 0, acc[0], lane);
    store_acc_f32(&ks.Ga[0][0], L + 1, 0, 8, acc[1], lane);
  } else {
    bf16* dst = wq == 1 ? &ks.Bm[0][0] : wq == 2 ? &ks.Cm[0][0] : &ks.Dm[0][0];
    store_acc_bf16(dst, LDS, 0, 0, acc[0], lane);
    store_acc_bf16(dst, LDS, 0, 8, acc[1], lane);
  }
}

// Phase K3 (one warp): Tf = (I - A)^{-1} by 8x8 blocks in fp32; Ti = bf16(Tf).
__device__ __forceinline__ void keyside_inverse(KeySide& ks, int lane) {
  if (lane < 16) {
    const int o = (lane >> 3) * 8, c = lane & 7;
    float x[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      float acc = (r == c) ? 1.f : 0.f;
#pragma unroll
      for (int s = 0; s < r; ++s) acc += ks.Ga[o + r][o + s] * x[s];
      x[r] = acc;  // x[s] == 0 for s < c, so the column starts at its diagonal
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) ks.Tf[o + r][o + c] = x[r];
  }
  __syncwarp();
#pragma unroll
  for (int e2 = 0; e2 < 2; ++e2) {  // M = A21 T11
    const int e = lane + 32 * e2, r = e >> 3, c = e & 7;
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) acc += ks.Ga[8 + r][s] * ks.Tf[s][c];
    ks.Mf[r][c] = acc;
  }
  __syncwarp();
#pragma unroll
  for (int e2 = 0; e2 < 2; ++e2) {  // T21 = T22 M
    const int e = lane + 32 * e2, r = e >> 3, c = e & 7;
    float acc = 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m) acc += ks.Tf[8 + r][8 + m] * ks.Mf[m][c];
    ks.Tf[8 + r][c] = acc;
  }
  __syncwarp();
#pragma unroll
  for (int e8 = 0; e8 < 8; ++e8) {
    const int e = lane + 32 * e8, r = e >> 4, c = e & 15;
    float v = (c > r) ? 0.f : ks.Tf[r][c];
    if (c > r) ks.Tf[r][c] = 0.f;
    ks.Ti[r][c] = __float2bfloat16_rn(v);
  }
}

// Phase K4a: W = Ti At (warp w: columns 16w..16w+15); Q = Ti Bm (warp 3).
__device__ __forceinline__ void keyside_wq(KeySide& ks, int wq, int lane) {
  uint32_t a[4], b[4];
  lda_rowmajor(a, &ks.Ti[0][0], LDS, 0, 0, lane);
  ldb_kn(b, &ks.At[0][0], LD, 16 * wq, 0, lane);
  float acc[2][4] = {};
  mma16816(acc[0], a, b[0], b[1]);
  mma16816(acc[1], a, b[2], b[3]);
  store_acc_bf16(&ks.W[0][0], LD, 0, 16 * wq, acc[0], lane);
  store_acc_bf16(&ks.W[0][0], LD, 0, 16 * wq + 8, acc[1], lane);
  if (wq == 3) {
    float qa[2][4] = {};
    ldb_kn(b, &ks.Bm[0][0], LDS, 0, 0, lane);
    mma16816(qa[0], a, b[0], b[1]);
    mma16816(qa[1], a, b[2], b[3]);
    store_acc_bf16(&ks.Q[0][0], LDS, 0, 0, qa[0], lane);
    store_acc_bf16(&ks.Q[0][0], LDS, 0, 8, qa[1], lane);
  }
}

// accumulator initialised from a bf16 [m][n] tile at (m0, n0)
__device__ __forceinline__ void acc_from_bf16(float (&c)[4], const bf16* tile, int ld, int m0,
                                              int n0, int lane) {
  const int g = lane >> 2, q = lane & 3;
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(tile + (m0 + g) * ld + n0 + 2 * q));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(tile + (m0 + g + 8) * ld + n0 + 2 * q));
  c[0] = lo.x; c[1] = lo.y; c[2] = hi.x; c[3] = hi.y;
}

// Phase K4b: Qy = Rt + Cm W (warp w: columns 16w..); P = Cm Q + Dm (warp 2).
__device__ __forceinline__ void keyside_qyp(KeySide& ks, int wq, int lane) {
  uint32_t a[4], b[4];
  lda_rowmajor(a, &ks.Cm[0][0], LDS, 0, 0, lane);
  ldb_kn(b, &ks.W[0][0], LD, 16 * wq, 0, lane);
  float acc[2][4];
  acc_from_bf16(acc[0], &ks.Rt[0][0], LD, 0, 16 * wq, lane);
  acc_from_bf16(acc[1], &ks.Rt[0][0], LD, 0, 16 * wq + 8, lane);
  mma16816(acc[0], a, b[0], b[1]);
  mma16816(acc[1], a, b[2], b[3]);
  store_acc_bf16(&ks.Qy[0][0], LD, 0, 16 * wq, acc[0], lane);
  store_acc_bf16(&ks.Qy[0][0], LD, 0, 16 * wq + 8, acc[1], lane);
  if (wq == 2) {
    float pa[2][4];
    acc_from_bf16(pa[0], &ks.Dm[0][0], LDS, 0, 0, lane);
    acc_from_bf16(pa[1], &ks.Dm[0][0], LDS, 0, 8, lane);
    ldb_kn(b, &ks.Q[0][0], LDS, 0, 0, lane);
    mma16816(pa[0], a, b[0], b[1]);
    mma16816(pa[1], a, b[2], b[3]);
    store_acc_bf16(&ks.P[0][0], LDS, 0, 0, pa[0], lane);
    store_acc_bf16(&ks.P[0][0], LDS, 0, 8, pa[1], lane);
  }
}

// All key-side phases of one chunk (all 4 warps; ends synchronised).
__device__ __forceinline__ void keyside_forward(KeySide& ks, const bf16 (*raw)[L][LD], int tid,
                                                int wq, int lane) {
  keyside_decays(ks, raw, tid);
  __syncthreads();
  keyside_grams(ks, wq, lane);
  __syncthreads();
  if (wq == 0) keyside_inverse(ks, lane);
  __syncthreads();
  keyside_wq(ks, wq, lane);
  __syncthreads();
  keyside_qyp(ks, wq, lane);
  __syncthreads();
}

// checkpoint slot of chunk c (state at the chunk's start, bf16 A fragments):
// uint4 index ((warp * 4 + kstep) * 32 + lane)
__device__ __forceinline__ const uint4* ckpt_slot(const float* base, int64_t ch, int64_t nchunk,
                                                  int64_t c) {
  return reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(base) +
                                        (ch * nchunk + c) * (kN * kN * 2));
}

// ---------------------------------------------------------------------------
// Backward.  For chunk c (walked in reverse) with incoming state S (from the
// checkpoint), the gradient dS' of the state after the chunk (carried from
// chunk c+1), dY and the external dSA:
//     dSA  = dSA_ext + Bh dS'^T
//     dS   = dS' diag(lam) + dY^T Qy + dSA^T W           (carried to chunk c-1)
//     dV   = Kh dS'^T + P^T dY + Q^T dSA
// and, summed over the state rows i,
//     dW = dSA S,  dQy = dY S,  dBh = SA dS',  dKh = V dS',
//     dQ = strict(dSA V^T),  dP = lower(dY V^T),  dlam = colsum(S o dS')
// which the key-side backward turns into dr, dw, dk, da, db:
//     dW += Cm^T dQy,  dQ += Cm^T dP,  dCm = lower(dQy W^T + dP Q^T)
//     dTi = dW At^T + dQ Bm^T,  dA = strict(Ti^T dTi Ti^T),  dBm = strict(Ti^T dQ)
//     dAt = Ti^T dW + dA Bb + dBm Kb,   dRt = dQy + dCm Bb + dP Kb
//     dBb = dA^T At + dCm^T Rt + dBh lam,  dKb = dBm^T At + dP^T Rt + dKh lam
//     da = dAt Lamx, dr = dRt Lam, dk = dKb / Lam, db = dBb / Lam
//     dcum = dRt o Rt - dKb o Kb - dBb o Bb (+ dlam lam at the last step),
//     dcumx = dAt o At,  dlw_s = sum_{t>=s} dcum_t + sum_{t>s} dcumx_t,
//     dw_in = dlw * (-e^{-1/2}) sigmoid (1 - sigmoid).
// Warp w owns state rows 16w.. for the value side and key columns 16w.. for
// the column-indexed key-side gradients; the 16x16 pieces are single-warp jobs.

constexpr int NSTB = 2;
constexpr int kNumInB = 7;  // r, w, k, a, b, v, dy
enum { IN_DY = 6 };
enum { OUT_DR = 0, OUT_DW = 1, OUT_DK = 2, OUT_DA = 3, OUT_DB = 4, OUT_DV = 5 };

struct BwdSmem {
  bf16 raw[NSTB][kNumInB][L][LD];
  float dsa[NSTB][L][kN];
  KeySide ks;
  bf16 Sin[kN][LD], dSo[kN][LD];     // state at the chunk start / gradient at its end
  bf16 SAT[kN][LDS], dSAT[kN][LDS];  // [i][t]
  float dlam_part[kWarps][kN];
  float dlam[kN];
  bf16 dQy[L][LD], dW2[L][LD];
  float dQf[L][L + 1], dTf[L][L + 1], dM1[L][L + 1];
  bf16 dPb[L][LDS], dQ2b[L][LDS], dCmb[L][LDS], dAb[L][LDS], dBmb[L][LDS];
  float dcum[L][kN], dcumx[L][kN];
  float dlamx[kN];
  bf16 out[6][L][LD];
};

__device__ __forceinline__ const bf16* in_ptr_b(const BwdArgs& p, int t) {
  const void* v = t == IN_R ? p.r : t == IN_W ? p.w : t == IN_K ? p.k : t == IN_A ? p.a
                : t == IN_B ? p.b : t == IN_V ? p.v : p.dy;
  return static_cast<const bf16*>(v);
}

// acc (16 x 16 at columns n0) += A (16 x 16*KS) B;  AT: A stored [k][m]; BT: B stored [k][n]
template <bool AT, bool BT, int KS>
__device__ __forceinline__ void mm16(float (&acc)[2][4], const bf16* A, int lda, const bf16* B,
                                     int ldb, int n0, int lane) {
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    uint32_t a[4], b[4];
    if (AT) lda_colmajor(a, A, lda, 0, 16 * kk, lane); else lda_rowmajor(a, A, lda, 0, 16 * kk, lane);
    if (BT) ldb_kn(b, B, ldb, n0, 16 * kk, lane); else ldb_nk(b, B, ldb, n0, 16 * kk, lane);
    mma16816(acc[0], a, b[0], b[1]);
    mma16816(acc[1], a, b[2], b[3]);
  }
}

__device__ __forceinline__ void zero(float (&acc)[2][4]) {
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
}

// keep element (t, s) of a 16x16 accumulator pair when s < t (strict) or s <= t
__device__ __forceinline__ void mask_lower(float (&acc)[2][4], bool strict, int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = g + (e >= 2 ? 8 : 0), s = 8 * nt + 2 * q + (e & 1);
      if (strict ? (s >= t) : (s > t)) acc[nt][e] = 0.f;
    }
}

__global__ void __launch_bounds__(kThreads) chunked_bwd_kernel(BwdArgs p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>(smem_raw);
  KeySide& ks = sm.ks;
  const int tid = threadIdx.x, lane = tid & 31, wq = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int64_t ch = blockIdx.x;
  const int64_t nchunk = p.g.nchunk, T = p.g.T, ts = p.g.tstride();
  const int64_t cbase = p.g.base(ch);
  const int i0 = 16 * wq, j0 = 16 * wq;
  auto get = [&](int t) { return in_ptr_b(p, t); };

  auto issue = [&](int st, int64_t c) {
    issue_tiles(sm.raw[st], kNumInB, get, cbase, ts, T, c, tid, kThreads);
    const int64_t t0 = c * L;
    for (int idx = tid; idx < L * 16; idx += kThreads) {  // dsa: 16 rows x 16 copies
      const int u = idx >> 4, part = idx & 15;
      const bool ok = p.dsa != nullptr && t0 + u < T;
      const float* src = ok ? p.dsa + cbase + (t0 + u) * ts + part * 4 : nullptr;
      if (ok) cp_async16(&sm.dsa[st][u][part * 4], src, true);
      else *reinterpret_cast<float4*>(&sm.dsa[st][u][part * 4]) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };

  float dSo[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) dSo[nt][e] = 0.f;

  if (nchunk > 0) issue(0, nchunk - 1);
  cp_async_commit();
  for (int64_t it = 0; it < nchunk; ++it) {
    const int64_t c = nchunk - 1 - it;
    const int st = it & 1;
    if (it + 1 < nchunk) issue(st ^ 1, c - 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const bf16(*raw)[L][LD] = sm.raw[st];
    keyside_forward(ks, raw, tid, wq, lane);

    // ---------------- value side (rows i0..i0+15) ----------------
    float Sin[8][4];
    if (c > 0) {
      const uint4* src = ckpt_slot(p.ckpt, ch, nchunk, c);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint4 x = src[(wq * 4 + kk) * 32 + lane];
        const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[h]));
          float* dst = h < 2 ? Sin[2 * kk] : Sin[2 * kk + 1];
          dst[2 * (h & 1)] = f.x;
          dst[2 * (h & 1) + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) Sin[nt][e] = 0.f;
    }
    uint32_t sA[4][4], dA_[4][4], vA[4], dyA[4], b[4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      acc_to_a(sA[kk], Sin[2 * kk], Sin[2 * kk + 1]);
      acc_to_a(dA_[kk], dSo[2 * kk], dSo[2 * kk + 1]);
    }
    lda_colmajor(vA, &raw[IN_V][0][0], LD, i0, 0, lane);
    lda_colmajor(dyA, &raw[IN_DY][0][0], LD, i0, 0, lane);

    float sat[2][4] = {}, dsat[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        dsat[nt][e] = sm.dsa[st][8 * nt + 2 * q + (e & 1)][i0 + g + (e >= 2 ? 8 : 0)];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      ldb_nk(b, &ks.W[0][0], LD, 0, 16 * kk, lane);
      mma16816(sat[0], sA[kk], b[0], b[1]);
      mma16816(sat[1], sA[kk], b[2], b[3]);
      ldb_nk(b, &ks.Bh[0][0], LD, 0, 16 * kk, lane);
      mma16816(dsat[0], dA_[kk], b[0], b[1]);
      mma16816(dsat[1], dA_[kk], b[2], b[3]);
    }
    ldb_nk(b, &ks.Q[0][0], LDS, 0, 0, lane);
    mma16816(sat[0], vA, b[0], b[1]);
    mma16816(sat[1], vA, b[2], b[3]);
    uint32_t dsaA[4];
    acc_to_a(dsaA, dsat[0], dsat[1]);

    // dV^T = dS' Kh^T + dY^T P + dSA^T Q
    {
      float dvt[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ldb_nk(b, &ks.Kh[0][0], LD, 0, 16 * kk, lane);
        mma16816(dvt[0], dA_[kk], b[0], b[1]);
        mma16816(dvt[1], dA_[kk], b[2], b[3]);
      }
      ldb_kn(b, &ks.P[0][0], LDS, 0, 0, lane);
      mma16816(dvt[0], dyA, b[0], b[1]);
      mma16816(dvt[1], dyA, b[2], b[3]);
      ldb_kn(b, &ks.Q[0][0], LDS, 0, 0, lane);
      mma16816(dvt[0], dsaA, b[0], b[1]);
      mma16816(dvt[1], dsaA, b[2], b[3]);
      store_acc_bf16_t(&sm.out[OUT_DV][0][0], LD, i0, 0, dvt[0], lane);
      store_acc_bf16_t(&sm.out[OUT_DV][0][0], LD, i0, 8, dvt[1], lane);
    }

    // rows of S, dS', SA^T, dSA^T for the sums over i; dlam partial sums
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      store_acc_bf16(&sm.Sin[0][0], LD, i0, 8 * nt, Sin[nt], lane);
      store_acc_bf16(&sm.dSo[0][0], LD, i0, 8 * nt, dSo[nt], lane);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      store_acc_bf16(&sm.SAT[0][0], LDS, i0, 8 * nt, sat[nt], lane);
      store_acc_bf16(&sm.dSAT[0][0], LDS, i0, 8 * nt, dsat[nt], lane);
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float p0 = Sin[nt][0] * dSo[nt][0] + Sin[nt][2] * dSo[nt][2];
      float p1 = Sin[nt][1] * dSo[nt][1] + Sin[nt][3] * dSo[nt][3];
#pragma unroll
      for (int m = 4; m < 32; m <<= 1) {
        p0 += __shfl_xor_sync(0xffffffffu, p0, m);
        p1 += __shfl_xor_sync(0xffffffffu, p1, m);
      }
      if (g == 0) {
        sm.dlam_part[wq][8 * nt + 2 * q] = p0;
        sm.dlam_part[wq][8 * nt + 2 * q + 1] = p1;
      }
    }

    // dS = dS' diag(lam) + dY^T Qy + dSA^T W  (becomes dS' of chunk c-1)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float l0 = ks.lam[8 * nt + 2 * q], l1 = ks.lam[8 * nt + 2 * q + 1];
      dSo[nt][0] *= l0; dSo[nt][1] *= l1; dSo[nt][2] *= l0; dSo[nt][3] *= l1;
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      ldb_kn(b, &ks.Qy[0][0], LD, 16 * m, 0, lane);
      mma16816(dSo[2 * m], dyA, b[0], b[1]);
      mma16816(dSo[2 * m + 1], dyA, b[2], b[3]);
      ldb_kn(b, &ks.W[0][0], LD, 16 * m, 0, lane);
      mma16816(dSo[2 * m], dsaA, b[0], b[1]);
      mma16816(dSo[2 * m + 1], dsaA, b[2], b[3]);
    }
    __syncthreads();

    // ---------------- B1: sums over the rows (warp w: columns j0..j0+15) ----------------
    float dW[2][4], dQy[2][4], dBh[2][4], dKh[2][4];
    zero(dW); zero(dQy); zero(dBh); zero(dKh);
    mm16<true, true, 4>(dW, &sm.dSAT[0][0], LDS, &sm.Sin[0][0], LD, j0, lane);
    mm16<false, true, 4>(dQy, &raw[IN_DY][0][0], LD, &sm.Sin[0][0], LD, j0, lane);
    mm16<true, true, 4>(dBh, &sm.SAT[0][0], LDS, &sm.dSo[0][0], LD, j0, lane);
    mm16<false, true, 4>(dKh, &raw[IN_V][0][0], LD, &sm.dSo[0][0], LD, j0, lane);
    store_acc_bf16(&sm.dQy[0][0], LD, 0, j0, dQy[0], lane);
    store_acc_bf16(&sm.dQy[0][0], LD, 0, j0 + 8, dQy[1], lane);
    if (wq == 0) {  // dQ = strict(dSA V^T)
      float dq[2][4] = {};
      mm16<true, false, 4>(dq, &sm.dSAT[0][0], LDS, &raw[IN_V][0][0], LD, 0, lane);
      mask_lower(dq, true, lane);
      store_acc_f32(&sm.dQf[0][0], L + 1, 0, 0, dq[0], lane);
      store_acc_f32(&sm.dQf[0][0], L + 1, 0, 8, dq[1], lane);
    } else if (wq == 1) {  // dP = lower(dY V^T)
      float dp[2][4] = {};
      mm16<false, false, 4>(dp, &raw[IN_DY][0][0], LD, &raw[IN_V][0][0], LD, 0, lane);
      mask_lower(dp, false, lane);
      store_acc_bf16(&sm.dPb[0][0], LDS, 0, 0, dp[0], lane);
      store_acc_bf16(&sm.dPb[0][0], LDS, 0, 8, dp[1], lane);
    } else if (wq == 2) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = lane + 32 * e;
        sm.dlam[j] = sm.dlam_part[0][j] + sm.dlam_part[1][j] + sm.dlam_part[2][j] + sm.dlam_part[3][j];
      }
    }
    __syncwarp();
    // dW += Cm^T dQy (own columns)
    mm16<true, true, 1>(dW, &ks.Cm[0][0], LDS, &sm.dQy[0][0], LD, j0, lane);
    store_acc_bf16(&sm.dW2[0][0], LD, 0, j0, dW[0], lane);
    store_acc_bf16(&sm.dW2[0][0], LD, 0, j0 + 8, dW[1], lane);
    __syncthreads();

    // ---------------- B2 ----------------
    if (wq == 0) {  // dCm = lower(dQy W^T + dP Q^T)
      float dcm[2][4] = {};
      mm16<false, false, 4>(dcm, &sm.dQy[0][0], LD, &ks.W[0][0], LD, 0, lane);
      mm16<false, false, 1>(dcm, &sm.dPb[0][0], LDS, &ks.Q[0][0], LDS, 0, lane);
      mask_lower(dcm, false, lane);
      store_acc_bf16(&sm.dCmb[0][0], LDS, 0, 0, dcm[0], lane);
      store_acc_bf16(&sm.dCmb[0][0], LDS, 0, 8, dcm[1], lane);
    } else if (wq == 1) {  // dQ += Cm^T dP;  dTi = dW At^T + dQ Bm^T
      float dq[2][4];
      const int gg = lane >> 2, qq = lane & 3;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          dq[nt][e] = sm.dQf[gg + (e >= 2 ? 8 : 0)][8 * nt + 2 * qq + (e & 1)];
      mm16<true, true, 1>(dq, &ks.Cm[0][0], LDS, &sm.dPb[0][0], LDS, 0, lane);
      store_acc_bf16(&sm.dQ2b[0][0], LDS, 0, 0, dq[0], lane);
      store_acc_bf16(&sm.dQ2b[0][0], LDS, 0, 8, dq[1], lane);
      __syncwarp();
      float dti[2][4] = {};
      mm16<false, false, 4>(dti, &sm.dW2[0][0], LD, &ks.At[0][0], LD, 0, lane);
      mm16<false, false, 1>(dti, &sm.dQ2b[0][0], LDS, &ks.Bm[0][0], LDS, 0, lane);
      store_acc_f32(&sm.dTf[0][0], L + 1, 0, 0, dti[0], lane);
      store_acc_f32(&sm.dTf[0][0], L + 1, 0, 8, dti[1], lane);
    }
    float dAt[2][4] = {};  // Ti^T dW (own columns)
    mm16<true, true, 1>(dAt, &ks.Ti[0][0], LDS, &sm.dW2[0][0], LD, j0, lane);
    __syncthreads();

    // ---------------- B3 ----------------
    if (wq == 0) {  // dA = strict(Ti^T dTi Ti^T) in fp32
#pragma unroll
      for (int e8 = 0; e8 < 8; ++e8) {  // M1 = dTi Ti^T
        const int e = lane + 32 * e8, t = e >> 4, s = e & 15;
        float acc = 0.f;
#pragma unroll
        for (int u = 0; u < L; ++u) acc += sm.dTf[t][u] * ks.Tf[s][u];
        sm.dM1[t][s] = acc;
      }
      __syncwarp();
#pragma unroll
      for (int e8 = 0; e8 < 8; ++e8) {
        const int e = lane + 32 * e8, t = e >> 4, s = e & 15;
        float acc = 0.f;
#pragma unroll
        for (int u = 0; u < L; ++u) acc += ks.Tf[u][t] * sm.dM1[u][s];
        sm.dAb[t][s] = __float2bfloat16_rn(s < t ? acc : 0.f);
      }
    } else if (wq == 1) {  // dBm = strict(Ti^T dQ)
      float dbm[2][4] = {};
      mm16<true, true, 1>(dbm, &ks.Ti[0][0], LDS, &sm.dQ2b[0][0], LDS, 0, lane);
      mask_lower(dbm, true, lane);
      store_acc_bf16(&sm.dBmb[0][0], LDS, 0, 0, dbm[0], lane);
      store_acc_bf16(&sm.dBmb[0][0], LDS, 0, 8, dbm[1], lane);
    }
    __syncthreads();

    // ---------------- B4: column-indexed key-side gradients (own columns) ----------------
    mm16<false, true, 1>(dAt, &sm.dAb[0][0], LDS, &ks.Bb[0][0], LD, j0, lane);
    mm16<false, true, 1>(dAt, &sm.dBmb[0][0], LDS, &ks.Kb[0][0], LD, j0, lane);
    float dBb[2][4] = {}, dKb[2][4] = {};
    mm16<true, true, 1>(dBb, &sm.dAb[0][0], LDS, &ks.At[0][0], LD, j0, lane);
    mm16<true, true, 1>(dBb, &sm.dCmb[0][0], LDS, &ks.Rt[0][0], LD, j0, lane);
    mm16<true, true, 1>(dKb, &sm.dBmb[0][0], LDS, &ks.At[0][0], LD, j0, lane);
    mm16<true, true, 1>(dKb, &sm.dPb[0][0], LDS, &ks.Rt[0][0], LD, j0, lane);
    float* dRt = &dQy[0][0];  // dRt = dQy + dCm Bb + dP Kb
    mm16<false, true, 1>(dQy, &sm.dCmb[0][0], LDS, &ks.Bb[0][0], LD, j0, lane);
    mm16<false, true, 1>(dQy, &sm.dPb[0][0], LDS, &ks.Kb[0][0], LD, j0, lane);
    (void)dRt;

#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float xl[2] = {0.f, 0.f};  // dlam contributions of this thread's two columns
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = g + (e >= 2 ? 8 : 0), j = j0 + 8 * nt + 2 * q + (e & 1);
        const float cm = ks.cum[t][j], sg = ks.sig[t][j], lamj = ks.lam[j];
        const float Lam = __expf(cm), Lamx = __expf(cm - kWScale * sg), iLam = __expf(-cm);
        const float rr = __bfloat162float(raw[IN_R][t][j]), kk = __bfloat162float(raw[IN_K][t][j]);
        const float aa = __bfloat162float(raw[IN_A][t][j]), bb = __bfloat162float(raw[IN_B][t][j]);
        const float Bbf = bb * iLam, Kbf = kk * iLam;
        xl[e & 1] += dBh[nt][e] * Bbf + dKh[nt][e] * Kbf;
        const float dbb = dBb[nt][e] + dBh[nt][e] * lamj;
        const float dkb = dKb[nt][e] + dKh[nt][e] * lamj;
        const float drt = dQy[nt][e], dat = dAt[nt][e];
        sm.out[OUT_DA][t][j] = __float2bfloat16_rn(dat * Lamx);
        sm.out[OUT_DR][t][j] = __float2bfloat16_rn(drt * Lam);
        sm.out[OUT_DK][t][j] = __float2bfloat16_rn(dkb * iLam);
        sm.out[OUT_DB][t][j] = __float2bfloat16_rn(dbb * iLam);
        sm.dcum[t][j] = drt * rr * Lam - dkb * Kbf - dbb * Bbf;
        sm.dcumx[t][j] = dat * aa * Lamx;
      }
#pragma unroll
      for (int m = 4; m < 32; m <<= 1) {
        xl[0] += __shfl_xor_sync(0xffffffffu, xl[0], m);
        xl[1] += __shfl_xor_sync(0xffffffffu, xl[1], m);
      }
      if (g == 0) {
        sm.dlamx[j0 + 8 * nt + 2 * q] = xl[0];
        sm.dlamx[j0 + 8 * nt + 2 * q + 1] = xl[1];
      }
    }
    __syncwarp();
    if (lane < 16) {  // reverse scans along t of column j
      const int j = j0 + lane;
      const float dl = sm.dlam[j] + sm.dlamx[j];
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int t = L - 1; t >= 0; --t) {
        float dc = sm.dcum[t][j];
        if (t == L - 1) dc += dl * ks.lam[j];
        s1 += dc;
        const float dlw = s1 + s2;
        s2 += sm.dcumx[t][j];
        const float sg = ks.sig[t][j];
        sm.out[OUT_DW][t][j] = __float2bfloat16_rn(dlw * kWScale * sg * (1.0f - sg));
      }
    }
    __syncthreads();

    // ---------------- write the chunk's six gradients ----------------
    for (int idx = tid; idx < 6 * L * 8; idx += kThreads) {
      const int tens = idx / (L * 8), rem = idx % (L * 8);
      const int u = rem >> 3, part = rem & 7;
      const int64_t t = c * L + u;
      if (t >= T) continue;
      void* dst = tens == OUT_DR ? p.dr : tens == OUT_DW ? p.dw : tens == OUT_DK ? p.dk
                : tens == OUT_DA ? p.da : tens == OUT_DB ? p.db : p.dv;
      *reinterpret_cast<uint4*>(static_cast<bf16*>(dst) + cbase + t * ts + part * 8) =
          *reinterpret_cast<const uint4*>(&sm.out[tens][u][part * 8]);
    }
  }
}

cudaError_t launch_bwd(const BwdArgs& p, cudaStream_t stream) {
  const size_t smem = sizeof(BwdSmem);
  cudaError_t e = cudaFuncSetAttribute(chunked_bwd_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  chunked_bwd_kernel<<<(unsigned)p.g.chains(), kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

// one bf16 64 x 64 state per chunk and chain
size_t ckpt_bytes(int64_t chains, int64_t T) {
  return static_cast<size_t>(chains * ((T + kChunk - 1) / kChunk)) * kN * kN * 2;
}

}  // namespace chunked
}  // namespace camoe
