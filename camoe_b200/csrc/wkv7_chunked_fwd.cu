// Chunked WKV-7 ClampW forward on the tensor cores (bf16 operands, fp32
// accumulation and fp32 state), the bf16 path of the operator.
//
// Per chain (b, h), chunks of L = 16 steps are processed in order.  With the
// log-decay lw = -e^{-1/2} sigmoid(w_in) (camoe/cuda/rwkv7_clampw.cu:42),
// cum_t = sum_{s<=t} lw_s inside the chunk, Lam = exp(cum) and lam = Lam_{L-1},
// the 16 steps of
//     S_t = S_{t-1} (diag w_t + a_t b_t^T) + v_t k_t^T,  y_t = S_t r_t,  sa_t = S_{t-1} a_t
// starting from the state S (rows = value index i, columns = key index j) are
//     SA = W S^T + Q V          (L x N, row t = sa_t)
//     Y  = Qy S^T + P V
//     S' = (S + SA^T Bb + V^T Kb) diag(lam)
// with the key-side matrices (functions of r, w, k, a, b only)
//     At = a exp(cum - lw), Rt = r Lam, Kb = k / Lam, Bb = b / Lam,
//     A  = strict_lower(At Bb^T), Bm = strict_lower(At Kb^T),
//     Cm = lower(Rt Bb^T),        Dm = lower(Rt Kb^T),     Ti = (I - A)^{-1},
//     W = Ti At, Q = Ti Bm, Qy = Rt + Cm W, P = Cm Q + Dm
// (the WY / UT-transform form of chunked delta-rule recurrences, e.g. Yang et
// al. 2024, "Parallelizing Linear Transformers with the Delta Rule over
// Sequence Length").  ClampW bounds every decay below by exp(-e^{-1/2}) =
// 0.545, so 1/Lam <= 0.545^-16 ~ 1.6e4: nothing over- or underflows.
//
// One CTA per chain, 12 warps in three roles:
//   value warps 0-3   own state rows 16w..16w+15 as mma accumulators for the
//                     whole sequence; per chunk they wait for its key-side
//                     slot, chain SA, Y and the state update in registers
//                     (accumulators reused as A fragments), write y, sa and
//                     the checkpoint, and release the slot;
//   key groups 4-7 and 8-11 compute the key-side matrices of alternate
//                     chunks into a ring of NS slots, two chunks in flight,
//                     their inputs arriving by TMA tile loads
//                     (cp.async.bulk.tensor, mbarrier complete_tx, 128-byte
//                     swizzle) NRAW chunks ahead.
// All hand-offs are mbarriers with bounded waits (wkv7_sync.cuh).
//
// Checkpoint: at the start of every chunk c > 0 the state is stored in bf16,
// in mma A-fragment order (8 KiB per chunk and chain): the backward loads it
// straight into A fragments.
#include "wkv7_common.cuh"
#include "wkv7_keyside.cuh"
#include "wkv7_mma.cuh"
#include "wkv7_sync.cuh"
#include "wkv7_tma.cuh"

namespace camoe {
namespace chunked {

using namespace camoe::mma;
using ks::L;
using ks::LD;
using ks::LDS;
using ks::Tile;
using ks::Tile16;

namespace fwd {

constexpr int NS = 4;         // key-side slots
constexpr int NRAW = 3;       // input buffers per key group
constexpr int kGroups = 2;
constexpr int kThreads = (4 + 4 * kGroups) * 32;  // 384
constexpr int kNumRaw = 6;    // r, w, k, a, b, v
enum { R_R = 0, R_W, R_K, R_A, R_B, R_V };

struct Slot {
  Tile W, Qy, Bb, Kb, v;
  Tile16 Q, P;
  float lam[kN];
};

struct Scratch {  // one per key group
  Tile At, Rt;
  Tile16 Bm, Cm, Dm, Ti;
  float Ga[L][L + 1], Tf[L][L + 1], Mf[8][9];
};

using RawTile = bf16[L * kN];  // 16 x 64, TMA 128-byte swizzled (2 KiB, 1 KiB aligned)

struct Smem {
  RawTile raw[kGroups][NRAW][kNumRaw];  // first: 1 KiB aligned for the swizzle
  Slot slot[NS];
  Scratch scr[kGroups];
  uint64_t full[NS], empty[NS], rawbar[kGroups][NRAW];
};

struct Params {
  CUtensorMap maps[kNumRaw];  // r, w, k, a, b, v as (N, H, T, B)
  FwdArgs a;
};

// Issued by one thread: TMA-load the 6 input tiles of chunk c into buf
// (rows past T arrive zero-filled); completion is tracked by `bar`.
__device__ __forceinline__ void issue_raw(RawTile* buf, uint64_t* bar, const Params& P, int h,
                                          int b, int64_t c) {
  mbar_arrive_expect_tx(bar, kNumRaw * tma::kTileBytes);
#pragma unroll
  for (int t = 0; t < kNumRaw; ++t) tma::load_tile(buf[t], &P.maps[t], h, static_cast<int>(c * L), b, bar);
}

__global__ void __launch_bounds__(kThreads, 1) chunked_fwd_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // round up to 1 KiB with pointer arithmetic (keeps the shared address space visible)
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024u - (sm_addr(smem_raw) & 1023u)) & 1023u));
  const FwdArgs& p = P.a;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ch = blockIdx.x;
  const int64_t nchunk = p.g.nchunk, T = p.g.T, ts = p.g.tstride();
  const int64_t cbase = p.g.base(ch);
  const int hh = static_cast<int>(p.g.h0 + ch % p.g.hc), bb = static_cast<int>(ch / p.g.hc);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 4);
    }
    for (int g = 0; g < kGroups; ++g)
      for (int b = 0; b < NRAW; ++b) mbar_init(&sm.rawbar[g][b], 1);
    mbar_fence_init();
  }
  __syncthreads();

  if (warp < 4) {
    // ------------------------------ value warps ------------------------------
    const int wq = warp, g = lane >> 2, q = lane & 3, i0 = 16 * wq;
    float S[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) S[nt][e] = 0.f;
    bf16* yp = static_cast<bf16*>(p.y);
    for (int64_t c = 0; c < nchunk; ++c) {
      const int s = static_cast<int>(c % NS);
      if (!mbar_wait(&sm.full[s], static_cast<uint32_t>((c / NS) & 1))) break;
      const Slot& sl = sm.slot[s];

      uint32_t sA[4][4], vA[4], b[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) acc_to_a(sA[kk], S[2 * kk], S[2 * kk + 1]);
      if (p.ckpt != nullptr && c > 0) {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.ckpt) +
                                              (ch * nchunk + c) * (kN * kN * 2));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          dst[(wq * 4 + kk) * 32 + lane] = make_uint4(sA[kk][0], sA[kk][1], sA[kk][2], sA[kk][3]);
      }
      lda_colmajor(vA, &sl.v[0][0], LD, i0, 0, lane);
      float sa[2][4] = {}, yv[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ldb_nk(b, &sl.W[0][0], LD, 0, 16 * kk, lane);
        mma16816(sa[0], sA[kk], b[0], b[1]);
        mma16816(sa[1], sA[kk], b[2], b[3]);
        ldb_nk(b, &sl.Qy[0][0], LD, 0, 16 * kk, lane);
        mma16816(yv[0], sA[kk], b[0], b[1]);
        mma16816(yv[1], sA[kk], b[2], b[3]);
      }
      ldb_nk(b, &sl.Q[0][0], LDS, 0, 0, lane);
      mma16816(sa[0], vA, b[0], b[1]);
      mma16816(sa[1], vA, b[2], b[3]);
      ldb_nk(b, &sl.P[0][0], LDS, 0, 0, lane);
      mma16816(yv[0], vA, b[0], b[1]);
      mma16816(yv[1], vA, b[2], b[3]);

      // S' = (S + SA^T Bb + V^T Kb) diag(lam)
      uint32_t saA[4];
      acc_to_a(saA, sa[0], sa[1]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        ldb_kn(b, &sl.Bb[0][0], LD, 16 * m, 0, lane);
        mma16816(S[2 * m], saA, b[0], b[1]);
        mma16816(S[2 * m + 1], saA, b[2], b[3]);
        ldb_kn(b, &sl.Kb[0][0], LD, 16 * m, 0, lane);
        mma16816(S[2 * m], vA, b[0], b[1]);
        mma16816(S[2 * m + 1], vA, b[2], b[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float2 l = *reinterpret_cast<const float2*>(&sl.lam[8 * nt + 2 * q]);
        S[nt][0] *= l.x; S[nt][1] *= l.y; S[nt][2] *= l.x; S[nt][3] *= l.y;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);

      // outputs: element (i = i0 + g (+8), t = 8 nt + 2q (+1))
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = i0 + g + (e >= 2 ? 8 : 0);
          const int64_t t = c * L + 8 * nt + 2 * q + (e & 1);
          if (t < T) {
            const int64_t o = cbase + t * ts + i;
            p.sa[o] = sa[nt][e];
            yp[o] = __float2bfloat16_rn(yv[nt][e]);
          }
        }
    }
  } else {
    // ------------------------------ key groups ------------------------------
    const int grp = (warp - 4) >> 2, gw = (warp - 4) & 3, gtid = tid - 128 - 128 * grp;
    const int bar_id = 1 + grp;
    Scratch& sc = sm.scr[grp];
    const int64_t nk = nchunk > grp ? (nchunk - grp + 1) / 2 : 0;  // chunks grp, grp+2, ...
    if (gtid == 0)
      for (int64_t kb = 0; kb < nk && kb < NRAW; ++kb)
        issue_raw(sm.raw[grp][kb], &sm.rawbar[grp][kb], P, hh, bb, grp + 2 * kb);
    bool ok = true;
    int64_t k = 0;
    for (; k < nk; ++k) {
      const int64_t c = grp + 2 * k;
      const int rb = static_cast<int>(k % NRAW), s = static_cast<int>(c % NS);
      RawTile* raw = sm.raw[grp][rb];
      Slot& sl = sm.slot[s];
      ok = mbar_wait(&sm.rawbar[grp][rb], static_cast<uint32_t>((k / NRAW) & 1));
      if (ok && c >= NS) ok = mbar_wait(&sm.empty[s], static_cast<uint32_t>((c / NS - 1) & 1));
      ok = named_sync_and(bar_id, 128, ok);  // the group leaves together on a timeout
      if (!ok) break;
      ks::decays<true>(raw[R_R], raw[R_W], raw[R_K], raw[R_A], raw[R_B], sc.At, sc.Rt, sl.Kb,
                       sl.Bb, sl.lam, nullptr, nullptr, gtid);
      {  // v tile -> slot, un-swizzled (one 16-byte piece per thread)
        const int u = gtid >> 3, part = gtid & 7;
        *reinterpret_cast<uint4*>(&sl.v[u][part * 8]) =
            *reinterpret_cast<const uint4*>(&raw[R_V][tma::swz(u, part * 8)]);
      }
      named_sync(bar_id, 128);
      ks::grams(sc.At, sc.Rt, sl.Bb, sl.Kb, sc.Ga, sc.Bm, sc.Cm, sc.Dm, gw, lane);
      named_sync(bar_id, 128);
      if (gw == 0) ks::inverse(sc.Ga, sc.Tf, sc.Mf, sc.Ti, lane);
      named_sync(bar_id, 128);
      ks::w_and_q(sc.Ti, sc.At, sc.Bm, sl.W, sl.Q, gw, lane);
      named_sync(bar_id, 128);
      ks::qy_and_p(sc.Cm, sl.W, sc.Rt, sl.Q, sc.Dm, sl.Qy, sl.P, gw, lane);
      named_sync(bar_id, 128);
      if (gtid == 0) mbar_arrive(&sm.full[s]);
      if (gtid == 0 && k + NRAW < nk)
        issue_raw(raw, &sm.rawbar[grp][rb], P, hh, bb, grp + 2 * (k + NRAW));
    }
    if (!ok && gtid == 0) {
      // a wait timed out: let this group's copies in flight land before exiting
      for (int64_t kk = k; kk < nk && kk < k + NRAW; ++kk)
        mbar_wait(&sm.rawbar[grp][kk % NRAW], static_cast<uint32_t>((kk / NRAW) & 1));
    }
  }
}

}  // namespace fwd

// wait timeouts recorded by this file's kernels on the current device
unsigned int fwd_timeouts() {
  unsigned int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_wkv7_timeouts, sizeof(n)) != cudaSuccess) return ~0u;
  return n;
}

cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream) {
  fwd::Params P;
  P.a = p;
  const void* src[fwd::kNumRaw] = {p.r, p.w, p.k, p.a, p.b, p.v};
  for (int t = 0; t < fwd::kNumRaw; ++t)
    if (!tma::encode_bhtn(&P.maps[t], src[t], p.g.B, p.g.T, p.g.H)) return cudaErrorInvalidValue;
  const size_t smem = sizeof(fwd::Smem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(fwd::chunked_fwd_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  fwd::chunked_fwd_kernel<<<(unsigned)p.g.chains(), fwd::kThreads, smem, stream>>>(P);
  return cudaGetLastError();
}

}  // namespace chunked
}  // namespace camoe
