// Chunked WKV-7 ClampW backward on the tensor cores: two kernels.
//
// With the forward of one chunk written (wkv7_chunked_fwd.cu) as
//     SA = W S^T + Q V,   Y = Qy S^T + P V,   S' = (S + SA^T Bb + V^T Kb) diag(lam),
// and G = dL/dS' the gradient carried in from the following chunk, G'' = G diag(lam):
//     dSA  = dSA_ext + Bb G''^T
//     dS   = G'' + dY^T Qy + dSA^T W                (carried to the previous chunk)
//     dV   = Kb G''^T + P^T dY + Q^T dSA
// and the key-side gradients need, summed over the 64 state rows i,
//     dW = dSA S,  dQy = dY S,  dBb = SA G'',  dKb = V G'',
//     dQ = strict(dSA V^T),  dP = lower(dY V^T),  dll = colsum(G o S')
// (dll is d(lam) * lam: lam scales the chunk's end state S').
//
// value_bwd_kernel (chunks in reverse, one to four CTAs per chain): carries G
// through the recurrence, writing dv and, per chunk, a rec::XRec (bf16 G'',
// SA^T, dSA^T, and the start state S where the forward checkpoint lacks it)
// to the workspace; the state at the start of every chunk comes from the
// checkpoint (even chunks) or is recomputed from the preceding even chunk
// (odd chunks).
//
// keyside_bwd_kernel (chunk-parallel, every SM): forms the row sums above from
// the chunk's XRec and its v, dy tiles, recomputes the decays and W, Q from
// r, w, k, a, b and the forward's triangular record (Ti, Bm, Cm), and turns
// both into dr, dw, dk, da, db:
//     dW += Cm^T dQy,  dQ += Cm^T dP,  dCm = lower(dQy W^T + dP Q^T)
//     dTi = dW At^T + dQ Bm^T,  dA = strict(Ti^T dTi Ti^T),  dBm = strict(Ti^T dQ)
//     dAt = Ti^T dW + dA Bb + dBm Kb,   dRt = dQy + dCm Bb + dP Kb
//     dBb += dA^T At + dCm^T Rt,        dKb += dBm^T At + dP^T Rt
//     da = dAt Lamx, dr = dRt Lam, dk = dKb / Lam, db = dBb / Lam
//     dcum = dRt o Rt - dKb o Kb - dBb o Bb (+ dll at the last step), dcumx = dAt o At
//     dlw_s = sum_{t>=s} dcum_t + sum_{t>s} dcumx_t,  dw_in = dlw (-e^{-1/2}) sig (1 - sig)
// (the chain rule of the forward algebra; per-element it is the gradient of
// camoe/cuda/rwkv7_clampw.cu:83-170 summed over a chunk).
#include "wkv7_common.cuh"
#include "wkv7_keyside.cuh"
#include "wkv7_mma.cuh"
#include "wkv7_record.cuh"
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

namespace vb {

// The state rows are independent in the recurrence (the transition acts on the
// key dimension), so a chain's 64 rows are split over 4 / RB CTAs of RB row
// blocks (16 rows) each.  Per row block:
//   G warp      the gradient recurrence G -> G'' -> dSA -> dS (the critical
//               path).  It loads all of a chunk's operand fragments before
//               its mma chains and publishes G'' and dSA in a small ring only
//               after them, so no shared-memory store sits in front of its
//               loads; no fences, no output stores;
//   dV warp     reads them, forms dV and stages dv and the G'', dSA^T rows of
//               the chunk's XRec;
//   state warp  start states (checkpointed or recomputed), SA; stages the
//               SA^T rows of the XRec and, for chunks 0, 1 and the odd ones,
//               its S rows (the key-side backward reads the other chunks'
//               start states from the forward checkpoint).
// A producer warp streams the inputs and a store warp writes the staged rows
// and the dv tile with bulk copies, KEEP groups in flight.
constexpr int NX = 4;    // output stages (power of two)
constexpr int KEEP = 2;  // store groups still reading shared memory, < NX

template <int RB>
struct alignas(1024) Slot {
  bf16 v[L * kN];   // TMA 128-byte swizzled, all 64 columns
  bf16 dy[L * kN];  // TMA 128-byte swizzled
  float dsa[L][16 * RB];  // this CTA's columns of the external dSA (no swizzle)
  rec::KeyRec k;
  bf16 S[16 * RB * kN];  // Swz64: this CTA's rows of the state at the chunk start (even chunks >= 2)
};

template <int RB>
struct alignas(128) GPub {  // G warp -> dV warp, one chunk
  bf16 G[16 * RB * kN];     // Swz64
  bf16 dSAT[16 * RB * L];   // Swz16
};

template <int RB>
struct alignas(1024) Stage {
  bf16 dv[L][16 * RB];     // dV tile [t][i] of this CTA's rows (TMA store)
  bf16 S[16 * RB * kN];    // Swz64, this CTA's rows of the XRec tiles
  bf16 G[16 * RB * kN];    // Swz64
  bf16 SAT[16 * RB * L];   // Swz16
  bf16 dSAT[16 * RB * L];  // Swz16
};

template <int RB>
struct Smem {
  // input slots and G'' / dSA ring entries (powers of two): eight slots keep the
  // producer far enough ahead of the state warp, which holds two at a time
  static constexpr int NS = RB == 4 ? 4 : 8;
  static constexpr int NG = RB == 1 ? 4 : 2;
  Slot<RB> slot[NS];
  Stage<RB> st[NX];
  GPub<RB> gp[NG];
  uint64_t full[NS], empty[NS], gfull[NG], gfree[NG], sfull[NX], sempty[NX];
};

struct Params {
  CUtensorMap map_v, map_dy, map_dsa, map_dv;
  BwdArgs a;
  void* work;
};

// Chunks are taken from the end in groups: one lone even chunk first when
// nchunk is odd, then (even, odd) pairs; lo is loaded before hi, hi is
// processed before lo.  Returns lo, hi (hi == lo for a lone chunk) and the
// load index of lo.
__device__ __forceinline__ void group_of(int nchunk, int gi, int& lo, int& hi, int& idx_lo) {
  if (nchunk & 1) {
    if (gi == 0) { lo = hi = nchunk - 1; idx_lo = 0; return; }
    lo = nchunk - 1 - 2 * gi;
    idx_lo = 1 + 2 * (gi - 1);
  } else {
    lo = nchunk - 2 - 2 * gi;
    idx_lo = 2 * gi;
  }
  hi = lo + 1;
}

// Load index (slot order) of chunk c; its processing index is nchunk - 1 - c.
__device__ __forceinline__ int load_idx(int nchunk, int c) {
  if ((nchunk & 1) && c == nchunk - 1) return 0;
  return (c & 1) ? nchunk - c : nchunk - 2 - c;
}

__device__ __forceinline__ uint32_t par(int idx, int n) { return static_cast<uint32_t>((idx / n) & 1); }

// SA^T fragments (rows = one row block, cols = t) of a chunk: S W^T + V Q^T.
__device__ __forceinline__ void sa_of(float (&sat)[2][4], const rec::KeyRec& kr,
                                      const uint32_t (&sA)[4][4], const uint32_t (&vA)[4], int lane) {
  uint32_t bW[4][4], bQ[4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) ldb_nk(bW[kk], kr.W, Swz64{}, 0, 16 * kk, lane);
  ldb_nk(bQ, kr.Q, Swz16{}, 0, 0, lane);
  mma_k64_k16(sat, sA, vA, bW, bQ);
}

// Whether chunk c's start state goes into its hand-off record: the key-side
// backward takes the states of even chunks >= 2 from the checkpoint instead,
// where the forward stored the same bf16 values in the same layout.
__device__ __forceinline__ bool record_state(int64_t c) { return c < 2 || (c & 1) != 0; }

// State warp, one chunk c (processing index pi): stage its SA^T rows, and its
// S rows when they go into the record.
template <int RB>
__device__ __forceinline__ bool s_chunk(Smem<RB>& sm, int pi, int c, int s, const uint32_t (&sA)[4][4],
                                        const float (&sat)[2][4], int il, int lane) {
  const int x = pi & (NX - 1);
  if (pi >= NX && !mbar_wait(&sm.sempty[x], par(pi - NX, NX))) return false;
  Stage<RB>& st = sm.st[x];
  if (record_state(c))
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) sta_rm(st.S, Swz64{}, il, 16 * kk, sA[kk], lane);
  uint32_t saA[4];
  acc_to_a(saA, sat[0], sat[1]);
  sta_rm(st.SAT, Swz16{}, il, 0, saA, lane);
  fence_proxy_async();
  __syncwarp();
  if (lane == 0) {
    mbar_arrive(&sm.sfull[x]);
    mbar_arrive(&sm.empty[s]);
  }
  return true;
}

template <int RB>
__global__ void __launch_bounds__(32 * (3 * RB + 2), 1) value_bwd_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem<RB>& sm = *reinterpret_cast<Smem<RB>*>(smem_raw + ((1024u - (sm_addr(smem_raw) & 1023u)) & 1023u));
  constexpr int NRG = 4 / RB;  // CTAs per chain
  constexpr int NG = Smem<RB>::NG;
  constexpr int NS = Smem<RB>::NS;
  const BwdArgs& p = P.a;
  const int tid = threadIdx.x, lane = tid & 31, warp = role_warp<RB>(tid >> 5);
  const int64_t ch = blockIdx.x / NRG;
  const int row0 = 16 * RB * static_cast<int>(blockIdx.x % NRG);  // first state row of this CTA
  const int nchunk = static_cast<int>(p.g.nchunk);
  const int ngroups = (nchunk + 1) / 2;
  const bool has_dsa = p.dsa != nullptr;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 2 * RB);  // state and dV warps (see the G warp)
    }
    for (int x = 0; x < NG; ++x) {
      mbar_init(&sm.gfull[x], RB);
      mbar_init(&sm.gfree[x], RB);
    }
    for (int x = 0; x < NX; ++x) {
      mbar_init(&sm.sfull[x], 2 * RB);
      mbar_init(&sm.sempty[x], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  const int hh = static_cast<int>(p.g.h0 + ch % p.g.hc), bb = static_cast<int>(ch / p.g.hc);
  if (warp == 3 * RB) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    const int64_t chains = p.g.chains();
    int issued = 0;
    bool ok = true;
    for (int gi = 0; gi < ngroups && ok; ++gi) {
      int lo, hi, idx;
      group_of(nchunk, gi, lo, hi, idx);
      for (int c = lo; c <= hi && ok; ++c, ++idx) {
        const int s = idx & (NS - 1);
        if (idx >= NS) ok = mbar_wait(&sm.empty[s], par(idx - NS, NS));
        if (!ok) break;
        const bool with_state = c == lo && lo >= 2;
        const uint32_t bytes = sizeof(rec::KeyRec) + 2 * tma::kTileBytes +
                               (has_dsa ? L * 64 * RB : 0) + (with_state ? 2048 * RB : 0);
        Slot<RB>& sl = sm.slot[s];
        mbar_arrive_expect_tx(&sm.full[s], bytes);
        bulk_g2s(&sl.k, rec::keyrec(const_cast<float*>(p.ckpt), ch, nchunk, c), sizeof(rec::KeyRec), &sm.full[s]);
        tma::load_tile(sl.v, &P.map_v, hh, c * L, bb, &sm.full[s]);
        tma::load_tile(sl.dy, &P.map_dy, hh, c * L, bb, &sm.full[s]);
        if (has_dsa) tma::load_tile_at(&sl.dsa[0][0], &P.map_dsa, row0, hh, c * L, bb, &sm.full[s]);
        if (with_state)
          bulk_g2s(sl.S, rec::state_ptr(const_cast<float*>(p.ckpt), chains, ch, nchunk, lo) + row0 * 128,
                   2048 * RB, &sm.full[s]);
        ++issued;
      }
    }
    if (!ok)  // stopped on a timeout: let the copies in flight land
      for (int i = issued > NS ? issued - NS : 0; i < issued; ++i)
        mbar_wait(&sm.full[i & (NS - 1)], par(i, NS));
    return;
  }

  if (warp == 3 * RB + 1) {
    // ------------------------------ store warp ------------------------------
    if (lane != 0) return;
    for (int pi = 0; pi < nchunk; ++pi) {
      const int c = nchunk - 1 - pi, x = pi & (NX - 1);
      if (!mbar_wait(&sm.sfull[x], par(pi, NX))) break;
      const Stage<RB>& st = sm.st[x];
      rec::XRec* xr = rec::xrec(P.work, ch, nchunk, c);
      if (record_state(c)) bulk_s2g(xr->S + row0 * kN, st.S, 2048 * RB);
      bulk_s2g(xr->G + row0 * kN, st.G, 2048 * RB);
      bulk_s2g(xr->SAT + row0 * L, st.SAT, 512 * RB);
      bulk_s2g(xr->dSAT + row0 * L, st.dSAT, 512 * RB);
      tma::store_tile(&P.map_dv, &st.dv[0][0], row0, hh, c * L, bb);
      bulk_commit();
      bulk_wait_read_n<KEEP>();
      if (pi >= KEEP) mbar_arrive(&sm.sempty[(pi - KEEP) & (NX - 1)]);
    }
    bulk_wait_all();
    return;
  }

  const int role = warp / RB, r = warp % RB;
  const int il = 16 * r, i0 = row0 + il;  // local and global first row of this warp's block
  const int q = lane & 3, g = lane >> 2;
  if (role == 0) {
    // ------------------------------ G warp: the gradient recurrence ------------------------------
    float G[8][4];  // dL/dS' of the chunk being processed: element (i0 + g (+8), 8 nt + 2q (+1))
    if (p.dsT != nullptr) {  // the gradient of the final state enters at the last chunk
      const float* src = p.dsT + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float2 lo = *reinterpret_cast<const float2*>(src + 8 * nt);
        const float2 hi = *reinterpret_cast<const float2*>(src + 8 * kN + 8 * nt);
        G[nt][0] = lo.x; G[nt][1] = lo.y; G[nt][2] = hi.x; G[nt][3] = hi.y;
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) G[nt][e] = 0.f;
    }
    if (nchunk > 0) {
      const int li0 = load_idx(nchunk, nchunk - 1);
      if (!mbar_wait(&sm.full[li0 & (NS - 1)], par(li0, NS))) return;
    }
    for (int pi = 0; pi < nchunk; ++pi) {
      const int c = nchunk - 1 - pi, li = load_idx(nchunk, c);
      const int s = li & (NS - 1), xg = pi & (NG - 1);
      const int lin = c >= 1 ? load_idx(nchunk, c - 1) : 0, sn = lin & (NS - 1);
      // barrier tests for the end of this chunk and the next one, answered while the chunk computes
      const bool next_ready = c == 0 || mbar_test(&sm.full[sn], par(lin, NS));
      const bool pub_ready = pi < NG || mbar_test(&sm.gfree[xg], par(pi - NG, NG));
      const Slot<RB>& sl = sm.slot[s];
      const rec::KeyRec& kr = sl.k;
      // all operand fragments of the chunk first
      uint32_t bB[4][4], bQy[4][4], bW[4][4], dyA[4];
      float2 lam[8];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ldb_nk(bB[kk], kr.Bb, Swz64{}, 0, 16 * kk, lane);
        ldb_kn(bQy[kk], kr.Qy, Swz64{}, 16 * kk, 0, lane);
        ldb_kn(bW[kk], kr.W, Swz64{}, 16 * kk, 0, lane);
      }
      lda_cm(dyA, sl.dy, Swz64{}, i0, 0, lane);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) lam[nt] = *reinterpret_cast<const float2*>(&kr.lam[8 * nt + 2 * q]);
      float dsat[2][4], dso[2][4];  // dSA = dSA_ext + Bb G''^T (rows i, cols t), odd k-steps apart
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dsat[nt][e] = has_dsa ? sl.dsa[8 * nt + 2 * q + (e & 1)][il + g + (e >= 2 ? 8 : 0)] : 0.f;
          dso[nt][e] = 0.f;
        }
      // G'' = G diag(lam)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        G[nt][0] *= lam[nt].x; G[nt][1] *= lam[nt].y; G[nt][2] *= lam[nt].x; G[nt][3] *= lam[nt].y;
      }
      uint32_t gA[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) acc_to_a(gA[kk], G[2 * kk], G[2 * kk + 1]);
#pragma unroll
      for (int kk = 0; kk < 4; kk += 2) {
        mma16816(dsat[0], gA[kk], bB[kk][0], bB[kk][1]);
        mma16816(dsat[1], gA[kk], bB[kk][2], bB[kk][3]);
        mma16816(dso[0], gA[kk + 1], bB[kk + 1][0], bB[kk + 1][1]);
        mma16816(dso[1], gA[kk + 1], bB[kk + 1][2], bB[kk + 1][3]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) dsat[nt][e] += dso[nt][e];
      // dS = G'' + dY^T Qy + dSA^T W  -> G of the previous chunk
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        mma16816(G[2 * m], dyA, bQy[m][0], bQy[m][1]);
        mma16816(G[2 * m + 1], dyA, bQy[m][2], bQy[m][3]);
      }
      uint32_t dsaA[4];
      acc_to_a(dsaA, dsat[0], dsat[1]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        mma16816(G[2 * m], dsaA, bW[m][0], bW[m][1]);
        mma16816(G[2 * m + 1], dsaA, bW[m][2], bW[m][3]);
      }
      // publish G'' and dSA
      if (!pub_ready && !mbar_wait(&sm.gfree[xg], par(pi - NG, NG))) return;
      GPub<RB>& gp = sm.gp[xg];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) sta_rm(gp.G, Swz64{}, il, 16 * kk, gA[kk], lane);
      sta_rm(gp.dSAT, Swz16{}, il, 0, dsaA, lane);
      __syncwarp();
      if (lane == 0) {
        // no release of slot s here: the dV warp releases it after waiting for
        // this publication, which follows every read of the slot above
        mbar_arrive(&sm.gfull[xg]);
      }
      if (!next_ready && !mbar_wait(&sm.full[sn], par(lin, NS))) return;
    }
    if (p.ds0 != nullptr) {  // after chunk 0, G is the gradient of the start state
      float* dst = p.ds0 + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        *reinterpret_cast<float2*>(dst + 8 * nt) = make_float2(G[nt][0], G[nt][1]);
        *reinterpret_cast<float2*>(dst + 8 * kN + 8 * nt) = make_float2(G[nt][2], G[nt][3]);
      }
    }
    return;
  }

  if (role == 2) {
    // ------------------------------ dV warp ------------------------------
    if (nchunk > 0) {
      const int li0 = load_idx(nchunk, nchunk - 1);
      if (!mbar_wait(&sm.full[li0 & (NS - 1)], par(li0, NS))) return;
    }
    for (int pi = 0; pi < nchunk; ++pi) {
      const int c = nchunk - 1 - pi, li = load_idx(nchunk, c);
      const int s = li & (NS - 1), xg = pi & (NG - 1), x = pi & (NX - 1);
      const int lin = c >= 1 ? load_idx(nchunk, c - 1) : 0, sn = lin & (NS - 1);
      const bool next_ready = c == 0 || mbar_test(&sm.full[sn], par(lin, NS));
      const bool st_ready = pi < NX || mbar_test(&sm.sempty[x], par(pi - NX, NX));
      const Slot<RB>& sl = sm.slot[s];
      const rec::KeyRec& kr = sl.k;
      uint32_t bK[4][4], bP[4], bQ[4], dyA[4], dsaA[4], gA[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) ldb_nk(bK[kk], kr.Kb, Swz64{}, 0, 16 * kk, lane);
      ldb_kn(bP, kr.P, Swz16{}, 0, 0, lane);
      ldb_kn(bQ, kr.Q, Swz16{}, 0, 0, lane);
      lda_cm(dyA, sl.dy, Swz64{}, i0, 0, lane);
      if (!mbar_wait(&sm.gfull[xg], par(pi, NG))) return;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) lda_rm(gA[kk], sm.gp[xg].G, Swz64{}, il, 16 * kk, lane);
      lda_rm(dsaA, sm.gp[xg].dSAT, Swz16{}, il, 0, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.gfree[xg]);
      // dV^T = G'' Kb^T + dY^T P + dSA^T Q (two accumulator chains, summed)
      float dvt[2][4] = {}, dvo[2][4] = {};
      mma16816(dvt[0], dyA, bP[0], bP[1]);
      mma16816(dvt[1], dyA, bP[2], bP[3]);
      mma16816(dvo[0], dsaA, bQ[0], bQ[1]);
      mma16816(dvo[1], dsaA, bQ[2], bQ[3]);
#pragma unroll
      for (int kk = 0; kk < 4; kk += 2) {
        mma16816(dvt[0], gA[kk], bK[kk][0], bK[kk][1]);
        mma16816(dvt[1], gA[kk], bK[kk][2], bK[kk][3]);
        mma16816(dvo[0], gA[kk + 1], bK[kk + 1][0], bK[kk + 1][1]);
        mma16816(dvo[1], gA[kk + 1], bK[kk + 1][2], bK[kk + 1][3]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) dvt[nt][e] += dvo[nt][e];
      uint32_t dvA[4];
      acc_to_a(dvA, dvt[0], dvt[1]);
      if (!st_ready && !mbar_wait(&sm.sempty[x], par(pi - NX, NX))) return;
      Stage<RB>& st = sm.st[x];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) sta_rm(st.G, Swz64{}, il, 16 * kk, gA[kk], lane);
      sta_rm(st.dSAT, Swz16{}, il, 0, dsaA, lane);
      sta_cm(&st.dv[0][0], Padded{16 * RB}, il, 0, dvA, lane);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.sfull[x]);
        mbar_arrive(&sm.empty[s]);
      }
      if (!next_ready && !mbar_wait(&sm.full[sn], par(lin, NS))) return;
    }
    return;
  }

  // ------------------------------ state warp ------------------------------
  for (int gi = 0; gi < ngroups; ++gi) {
    int lo, hi, idx_lo;
    group_of(nchunk, gi, lo, hi, idx_lo);
    const int s_lo = idx_lo & (NS - 1), s_hi = (idx_lo + 1) & (NS - 1);
    if (!mbar_wait(&sm.full[s_lo], par(idx_lo, NS))) return;
    if (hi != lo && !mbar_wait(&sm.full[s_hi], par(idx_lo + 1, NS))) return;
    const Slot<RB>& slo = sm.slot[s_lo];
    const rec::KeyRec& kr = slo.k;

    uint32_t sLo[4][4], vA[4];
    if (lo >= 2) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) lda_rm(sLo[kk], slo.S, Swz64{}, il, 16 * kk, lane);
    } else if (p.s0 != nullptr) {  // chunk 0 starts from the state carried in (bf16, as stored)
      const float* src = p.s0 + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
      float Sf[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float2 a = *reinterpret_cast<const float2*>(src + 8 * nt);
        const float2 c2 = *reinterpret_cast<const float2*>(src + 8 * kN + 8 * nt);
        Sf[nt][0] = a.x; Sf[nt][1] = a.y; Sf[nt][2] = c2.x; Sf[nt][3] = c2.y;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) acc_to_a(sLo[kk], Sf[2 * kk], Sf[2 * kk + 1]);
    } else {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) sLo[kk][0] = sLo[kk][1] = sLo[kk][2] = sLo[kk][3] = 0u;
    }
    lda_cm(vA, slo.v, Swz64{}, i0, 0, lane);
    float satLo[2][4];
    sa_of(satLo, kr, sLo, vA, lane);
    if (hi != lo) {
      // S(hi) = (S(lo) + SA^T Bb + V^T Kb) diag(lam), from chunk lo
      uint32_t sHi[4][4], b[4];
      {
        float Sf[8][4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // sLo[kk] is the A fragment of n8 tiles (2kk, 2kk+1): regs 0,1 -> 2kk, 2,3 -> 2kk+1
            const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sLo[kk][h]));
            const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sLo[kk][2 + h]));
            Sf[2 * kk][2 * h] = a0.x;
            Sf[2 * kk][2 * h + 1] = a0.y;
            Sf[2 * kk + 1][2 * h] = a1.x;
            Sf[2 * kk + 1][2 * h + 1] = a1.y;
          }
        uint32_t saA[4];
        acc_to_a(saA, satLo[0], satLo[1]);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          ldb_kn(b, kr.Bb, Swz64{}, 16 * m, 0, lane);
          mma16816(Sf[2 * m], saA, b[0], b[1]);
          mma16816(Sf[2 * m + 1], saA, b[2], b[3]);
          ldb_kn(b, kr.Kb, Swz64{}, 16 * m, 0, lane);
          mma16816(Sf[2 * m], vA, b[0], b[1]);
          mma16816(Sf[2 * m + 1], vA, b[2], b[3]);
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const float2 l = *reinterpret_cast<const float2*>(&kr.lam[8 * nt + 2 * q]);
          Sf[nt][0] *= l.x; Sf[nt][1] *= l.y; Sf[nt][2] *= l.x; Sf[nt][3] *= l.y;
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) acc_to_a(sHi[kk], Sf[2 * kk], Sf[2 * kk + 1]);
      }
      const Slot<RB>& shi = sm.slot[s_hi];
      uint32_t vHi[4];
      lda_cm(vHi, shi.v, Swz64{}, i0, 0, lane);
      float satHi[2][4];
      sa_of(satHi, shi.k, sHi, vHi, lane);
      if (!s_chunk(sm, nchunk - 1 - hi, hi, s_hi, sHi, satHi, il, lane)) return;
    }
    if (!s_chunk(sm, nchunk - 1 - lo, lo, s_lo, sLo, satLo, il, lane)) return;
  }
}

template <int RB>
cudaError_t launch(const Params& V, int64_t chains, cudaStream_t stream) {
  const size_t smem = sizeof(Smem<RB>) + 1024;
  cudaError_t e = cudaFuncSetAttribute(value_bwd_kernel<RB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  value_bwd_kernel<RB><<<static_cast<unsigned>(chains * (4 / RB)), 32 * (3 * RB + 2), smem, stream>>>(V);
  return cudaGetLastError();
}

}  // namespace vb

namespace kb {

constexpr int kThreads = 128;  // one group of 4 warps per CTA, 4 CTAs per SM

// Inputs are single-buffered: v, dy and the XRec (part A), and r, w, k, a, b
// (part B) of the next item are loaded once this item's outputs, staged in
// place in the r, w, k, a, b tiles, have been copied out; the record's space
// serves as scratch in between.  Four CTAs per SM cover each other's loads.
struct alignas(1024) KGroup {
  bf16 raw[7][L * kN];  // r, w, k, a, b, v, dy as landed by TMA (1 KiB aligned);
                        // r, w, k, a, b then hold dr, dw, dk, da, db until copied out
  // The hand-off record is read only by the row sums; the tiles of the later
  // phases reuse its space (54 KB per CTA: four CTAs per SM)
  union Shared {
    rec::XRec x;
    struct Scratch {
      Tile dQyb, dW2b;
      Tile At, Rt, Bb, Kb;
      Tile W;
      bf16 dCmb[L][LDS], dAb[L][LDS], dBmb[L][LDS];
    } s;
  } u;
  float lam[kN], cum[L][ks::LDF], lw[L][ks::LDF];
  float dllp[1][kN], dll[kN];  // colsum(G'' o S) (own columns per warp), then dll
  bf16 dPb[L][LDS];
  Tile16 Ti, Q;
  alignas(16) rec::TriRec tri;  // Tf = Ti in fp32, Bm, Cm: from the forward, with part B
  float Ga[L][L + 1];           // scratch of the dA product
  bf16 dQ2b[L][LDS];
  float dTf[L][L + 1];
  uint64_t barA, barB;
};

// four CTAs per SM: each takes its dynamic shared memory (the struct plus 1 KiB
// of alignment slack) and 1 KiB the runtime reserves, out of 228 KiB
static_assert(4 * (sizeof(KGroup) + 2048) <= 228 * 1024, "keyside_bwd: four CTAs per SM");

struct Params {
  CUtensorMap in[7];  // r, w, k, a, b, v, dy
  BwdArgs a;
  void* work;
};

// loads of the item at walk position w
__device__ __forceinline__ void issue_a(KGroup& G, const Params& P, const ItemWalk& w) {
  const int64_t ch = w.ch, c = w.c;
  const int h = w.head(P.a.g), b = static_cast<int>(w.b);
  mbar_arrive_expect_tx(&G.barA, 2 * tma::kTileBytes + sizeof(rec::XRec));
  tma::load_tile(G.raw[5], &P.in[5], h, static_cast<int>(c * L), b, &G.barA);
  tma::load_tile(G.raw[6], &P.in[6], h, static_cast<int>(c * L), b, &G.barA);
  const rec::XRec* xr = rec::xrec(P.work, ch, P.a.g.nchunk, c);
  if (vb::record_state(c)) {
    bulk_g2s(&G.u.x, xr, sizeof(rec::XRec), &G.barA);
  } else {  // the start state from the checkpoint, the rest of the record from the workspace
    constexpr uint32_t kS = sizeof(rec::XRec::S);
    bulk_g2s(G.u.x.S, rec::state_ptr(const_cast<float*>(P.a.ckpt), P.a.g.chains(), ch,
                                     P.a.g.nchunk, c), kS, &G.barA);
    bulk_g2s(G.u.x.G, xr->G, sizeof(rec::XRec) - kS, &G.barA);
  }
}

__device__ __forceinline__ void issue_b(KGroup& G, const Params& P, const ItemWalk& w) {
  const int64_t ch = w.ch, c = w.c;
  const int h = w.head(P.a.g), b = static_cast<int>(w.b);
  mbar_arrive_expect_tx(&G.barB, 5 * tma::kTileBytes + sizeof(rec::TriRec));
#pragma unroll
  for (int t = 0; t < 5; ++t) tma::load_tile(G.raw[t], &P.in[t], h, static_cast<int>(c * L), b, &G.barB);
  bulk_g2s(&G.tri, rec::trirec(const_cast<float*>(P.a.ckpt), P.a.g.chains(), ch, P.a.g.nchunk, c),
           sizeof(rec::TriRec), &G.barB);
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc (16 x 8 at columns n0) = A (16 x 16) B (16 x 16) with tf32 operands, one warp;
// A(m, k) and B(k, n) are element accessors.
template <typename FA, typename FB>
__device__ __forceinline__ void mm8_tf32(float (&acc)[4], FA A, FB B, int n0, int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < 16; k0 += 8) {
    const uint32_t a[4] = {to_tf32(A(g, k0 + q)), to_tf32(A(g + 8, k0 + q)),
                           to_tf32(A(g, k0 + q + 4)), to_tf32(A(g + 8, k0 + q + 4))};
    mma_tf32(acc, a, to_tf32(B(k0 + q, n0 + g)), to_tf32(B(k0 + q + 4, n0 + g)));
  }
}

__global__ void __launch_bounds__(kThreads, 4) keyside_bwd_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  KGroup& G = *reinterpret_cast<KGroup*>(smem_raw + ((1024u - (sm_addr(smem_raw) & 1023u)) & 1023u));
  const BwdArgs& p = P.a;
  const int tid = threadIdx.x, lane = tid & 31, gw = tid >> 5, gq = lane >> 2, q = lane & 3;
  const int j0 = 16 * gw;
  if (tid == 0) {
    mbar_init(&G.barA, 1);
    mbar_init(&G.barB, 1);
    mbar_fence_init();
  }
  __syncthreads();
  const int64_t nchunk = p.g.nchunk;
  const int64_t total = p.g.chains() * nchunk;
  // thread 0's count of part A / part B loads issued and of their completions seen
  int64_t issued_a = 0, issued_b = 0, seen_a = 0, seen_b = 0;
  ItemWalk walk;  // this CTA's current item
  walk.init(p.g, blockIdx.x, gridDim.x);
  if (tid == 0 && blockIdx.x < total) {
    issue_a(G, P, walk);
    issue_b(G, P, walk);
    issued_a = issued_b = 1;
  }
  const bf16* raw_r = G.raw[0];
  const bf16* raw_k = G.raw[2];
  const bf16* raw_a = G.raw[3];
  const bf16* raw_b = G.raw[4];
  const bf16* raw_v = G.raw[5];
  const bf16* raw_dy = G.raw[6];
  rec::XRec& xr = G.u.x;
  int64_t j = 0;
  for (;; ++j) {
    const int64_t item = blockIdx.x + j * gridDim.x;
    if (item >= total) break;
    const int64_t next = item + gridDim.x;
    const uint32_t ph = static_cast<uint32_t>(j & 1);
    bool ok = mbar_wait(&G.barA, ph);  // v, dy, XRec
    seen_a += ok;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const int64_t c = walk.c;

    // ---- row sums over the 64 state rows (own columns j0 .. j0 + 15), and the key side ----
    //   dW = dSA S, dQy = dY S, dBb = SA G'', dKb = V G'', and colsum(G'' o S) as the
    //   diagonal of G''^T S; dQ = strict(dSA V^T) (warp 1, kept in registers),
    //   dP = lower(dY V^T) (warp 2).  One pass over the 64 rows in k-steps of 16:
    //   the S and G'' fragments of a k-step serve every product that needs them.
    float dW[2][4] = {}, dQy[2][4] = {}, dBp[2][4] = {}, dKp[2][4] = {}, dq[2][4] = {};
    {
      float dd[2][4] = {}, dp[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t bS[4], bG[4], aD[4], aY[4], aA[4], aV[4], aT[4];
        ldb_kn(bS, xr.S, Swz64{}, j0, 16 * kk, lane);
        ldb_kn(bG, xr.G, Swz64{}, j0, 16 * kk, lane);
        lda_cm(aD, xr.dSAT, Swz16{}, 0, 16 * kk, lane);   // dSA (t x i)
        lda_rm(aY, raw_dy, Swz64{}, 0, 16 * kk, lane);    // dY
        lda_cm(aA, xr.SAT, Swz16{}, 0, 16 * kk, lane);    // SA
        lda_rm(aV, raw_v, Swz64{}, 0, 16 * kk, lane);     // V
        lda_cm(aT, xr.G, Swz64{}, j0, 16 * kk, lane);     // G''^T (own columns as rows)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          mma16816(dW[nt], aD, bS[2 * nt], bS[2 * nt + 1]);
          mma16816(dQy[nt], aY, bS[2 * nt], bS[2 * nt + 1]);
          mma16816(dBp[nt], aA, bG[2 * nt], bG[2 * nt + 1]);
          mma16816(dKp[nt], aV, bG[2 * nt], bG[2 * nt + 1]);
          mma16816(dd[nt], aT, bS[2 * nt], bS[2 * nt + 1]);
        }
        if (gw == 1 || gw == 2) {  // V^T as the B operand (k = i, n = s)
          uint32_t bV[4];
          ldb_nk(bV, raw_v, Swz64{}, 0, 16 * kk, lane);
          if (gw == 1) {
            mma16816(dq[0], aD, bV[0], bV[1]);
            mma16816(dq[1], aD, bV[2], bV[3]);
          } else {
            mma16816(dp[0], aY, bV[0], bV[1]);
            mma16816(dp[1], aY, bV[2], bV[3]);
          }
        }
      }
      if (gw == 1) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = gq + (e >= 2 ? 8 : 0), u = 8 * nt + 2 * q + (e & 1);
            if (u >= t) dq[nt][e] = 0.f;
          }
      } else if (gw == 2) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = gq + (e >= 2 ? 8 : 0), u = 8 * nt + 2 * q + (e & 1);
            if (u > t) dp[nt][e] = 0.f;
          }
        store_acc_bf16(&G.dPb[0][0], LDS, 0, 0, dp[0], lane);
        store_acc_bf16(&G.dPb[0][0], LDS, 0, 8, dp[1], lane);
      }
      // diagonal of the 16 x 16 block G''^T S: lanes with gq / 2 == q hold columns
      // j0 + gq (tile 0) and j0 + 8 + gq (tile 1)
      if ((gq >> 1) == q) {
        const bool x = gq & 1;  // selects, not an index: keeps dd in registers
        G.dllp[0][j0 + gq] = x ? dd[0][1] : dd[0][0];
        G.dllp[0][j0 + 8 + gq] = x ? dd[1][3] : dd[1][2];
      }
    }
    ok = mbar_wait(&G.barB, ph);  // r, w, k, a, b
    seen_b += ok;
    // every warp's row sums are done: v, dy and the hand-off record are dead,
    // and the scratch tiles may overwrite the record
    ok = __syncthreads_and(ok);
    if (!ok) break;
    ks::decays<true>(raw_r, G.raw[1], raw_k, raw_a, raw_b, &G.u.s.At[0][0], &G.u.s.Rt[0][0],
                     Padded{LD}, &G.u.s.Kb[0][0], &G.u.s.Bb[0][0], Padded{LD}, G.lam, G.cum, G.lw,
                     tid, p.g.decay);
    __syncthreads();
    for (int e = tid; e < L * L; e += kThreads)  // Ti = bf16(Tf) for the bf16 products
      G.Ti[e >> 4][e & 15] = __float2bfloat16_rn(G.tri.Tf[e >> 4][e & 15]);
    {  // dll = colsum(G'' o S') / lam = colsum(G'' o S) + colsum(Bb o SA G'') + colsum(Kb o V G'')
      float v[4];  // columns j0 + 8 nt + 2q + x, as v[2 nt + x]; rows gq, gq + 8 of this lane
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int jj = j0 + 8 * nt + 2 * q + x;
          v[2 * nt + x] = __bfloat162float(G.u.s.Bb[gq][jj]) * dBp[nt][x] + __bfloat162float(G.u.s.Kb[gq][jj]) * dKp[nt][x] +
                          __bfloat162float(G.u.s.Bb[gq + 8][jj]) * dBp[nt][2 + x] +
                          __bfloat162float(G.u.s.Kb[gq + 8][jj]) * dKp[nt][2 + x];
        }
#pragma unroll
      for (int m = 4; m < 32; m <<= 1)
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], m);
      if (gq == 0)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int jj = j0 + 8 * (i >> 1) + 2 * q + (i & 1);
          G.dll[jj] = G.dllp[0][jj] + v[i];
        }
    }
    store_acc_bf16(&G.u.s.dQyb[0][0], LD, 0, j0, dQy[0], lane);
    store_acc_bf16(&G.u.s.dQyb[0][0], LD, 0, j0 + 8, dQy[1], lane);
    __syncwarp();
    // dW += Cm^T dQy (own columns of dQy, written by this warp)
    mm16<true, true, 1>(dW, &G.tri.Cm[0][0], Padded{LDS}, &G.u.s.dQyb[0][0], Padded{LD}, j0, lane);
    store_acc_bf16(&G.u.s.dW2b[0][0], LD, 0, j0, dW[0], lane);
    store_acc_bf16(&G.u.s.dW2b[0][0], LD, 0, j0 + 8, dW[1], lane);
    __syncthreads();
    ks::w_and_q(G.Ti, &G.u.s.At[0][0], Padded{LD}, G.tri.Bm, &G.u.s.W[0][0], Padded{LD}, &G.Q[0][0],
                Padded{LDS}, gw, lane);
    __syncthreads();  // W, Q and dW ready

    // ---- 16x16 pieces ----
    if (gw == 0) {  // dCm = lower(dQy W^T + dP Q^T)
      float dcm[2][4] = {};
      mm16<false, false, 4>(dcm, &G.u.s.dQyb[0][0], Padded{LD}, &G.u.s.W[0][0], Padded{LD}, 0, lane);
      mm16<false, false, 1>(dcm, &G.dPb[0][0], Padded{LDS}, &G.Q[0][0], Padded{LDS}, 0, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = gq + (e >= 2 ? 8 : 0), u = 8 * nt + 2 * q + (e & 1);
          if (u > t) dcm[nt][e] = 0.f;
        }
      store_acc_bf16(&G.u.s.dCmb[0][0], LDS, 0, 0, dcm[0], lane);
      store_acc_bf16(&G.u.s.dCmb[0][0], LDS, 0, 8, dcm[1], lane);
    } else if (gw == 1) {  // dQ += Cm^T dP;  dTi = dW At^T + dQ Bm^T
      mm16<true, true, 1>(dq, &G.tri.Cm[0][0], Padded{LDS}, &G.dPb[0][0], Padded{LDS}, 0, lane);
      store_acc_bf16(&G.dQ2b[0][0], LDS, 0, 0, dq[0], lane);
      store_acc_bf16(&G.dQ2b[0][0], LDS, 0, 8, dq[1], lane);
      __syncwarp();
      float dti[2][4] = {};
      mm16<false, false, 4>(dti, &G.u.s.dW2b[0][0], Padded{LD}, &G.u.s.At[0][0], Padded{LD}, 0, lane);
      mm16<false, false, 1>(dti, &G.dQ2b[0][0], Padded{LDS}, &G.tri.Bm[0][0], Padded{LDS}, 0, lane);
      store_acc_f32(&G.dTf[0][0], L + 1, 0, 0, dti[0], lane);
      store_acc_f32(&G.dTf[0][0], L + 1, 0, 8, dti[1], lane);
    }
    float dAt[2][4] = {};  // Ti^T dW (own columns)
    mm16<true, true, 1>(dAt, &G.Ti[0][0], Padded{LDS}, &G.u.s.dW2b[0][0], Padded{LD}, j0, lane);
    __syncthreads();
    // dA = strict(Ti^T dTi Ti^T) with tf32 operands, columns 0-7 on warp 0 and 8-15 on
    // warp 2 (a column block of dA needs only that block of M1 = dTi Ti^T);
    // dBm = strict(Ti^T dQ) on warp 1; every warp also forms the column products
    // that need neither.
    if (gw == 0 || gw == 2) {
      const int n0 = gw == 0 ? 0 : 8;
      float m1[4] = {};
      mm8_tf32(m1, [&](int m, int k) { return G.dTf[m][k]; },
               [&](int k, int n) { return G.tri.Tf[n][k]; }, n0, lane);
      store_acc_f32(&G.Ga[0][0], L + 1, 0, n0, m1, lane);
      __syncwarp();
      float da[4] = {};
      mm8_tf32(da, [&](int m, int k) { return G.tri.Tf[k][m]; },
               [&](int k, int n) { return G.Ga[k][n]; }, n0, lane);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = gq + (e >= 2 ? 8 : 0), u = n0 + 2 * q + (e & 1);
        if (u >= t) da[e] = 0.f;
      }
      store_acc_bf16(&G.u.s.dAb[0][0], LDS, 0, n0, da, lane);
    } else if (gw == 1) {
      float dbm[2][4] = {};
      mm16<true, true, 1>(dbm, &G.Ti[0][0], Padded{LDS}, &G.dQ2b[0][0], Padded{LDS}, 0, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = gq + (e >= 2 ? 8 : 0), u = 8 * nt + 2 * q + (e & 1);
          if (u >= t) dbm[nt][e] = 0.f;
        }
      store_acc_bf16(&G.u.s.dBmb[0][0], LDS, 0, 0, dbm[0], lane);
      store_acc_bf16(&G.u.s.dBmb[0][0], LDS, 0, 8, dbm[1], lane);
    }
    float dBb[2][4] = {}, dKb[2][4] = {}, dRt[2][4] = {};
    mm16<true, true, 1>(dBb, &G.u.s.dCmb[0][0], Padded{LDS}, &G.u.s.Rt[0][0], Padded{LD}, j0, lane);
    mm16<true, true, 1>(dKb, &G.dPb[0][0], Padded{LDS}, &G.u.s.Rt[0][0], Padded{LD}, j0, lane);
    mm16<false, true, 1>(dRt, &G.u.s.dCmb[0][0], Padded{LDS}, &G.u.s.Bb[0][0], Padded{LD}, j0, lane);
    mm16<false, true, 1>(dRt, &G.dPb[0][0], Padded{LDS}, &G.u.s.Kb[0][0], Padded{LD}, j0, lane);
    __syncthreads();

    // ---- column-indexed gradients that need dA, dBm (own columns) ----
    mm16<false, true, 1>(dAt, &G.u.s.dAb[0][0], Padded{LDS}, &G.u.s.Bb[0][0], Padded{LD}, j0, lane);
    mm16<false, true, 1>(dAt, &G.u.s.dBmb[0][0], Padded{LDS}, &G.u.s.Kb[0][0], Padded{LD}, j0, lane);
    mm16<true, true, 1>(dBb, &G.u.s.dAb[0][0], Padded{LDS}, &G.u.s.At[0][0], Padded{LD}, j0, lane);
    mm16<true, true, 1>(dKb, &G.u.s.dBmb[0][0], Padded{LDS}, &G.u.s.At[0][0], Padded{LD}, j0, lane);
    // outputs in place of the inputs they replace (same thread, same element):
    // dr -> r, dk -> k, da -> a, db -> b tiles; dw -> the w tile.  This lane
    // holds rows gq (hf 0) and gq + 8 (hf 1) of columns j0 + 8 nt + 2q + x.
    // the column pair x = 0, 1 of each (nt, hf) runs as packed two-lane fp32
    float u[2][2][2], cx[2][2][2], lws[2][2][2];  // [nt][x][hf]: dcum + dcumx, dcumx, lw
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int t = gq + 8 * hf, jj = j0 + 8 * nt + 2 * q, o = tma::swz(t, jj);
        const float2 cm = *reinterpret_cast<const float2*>(&G.cum[t][jj]);
        const float2 lg = *reinterpret_cast<const float2*>(&G.lw[t][jj]);
        const float2 rr = ks::ld_bf2(raw_r + o), kk = ks::ld_bf2(raw_k + o);
        const float2 aa = ks::ld_bf2(raw_a + o), bb = ks::ld_bf2(raw_b + o);
        const float2 Lam = ks::exp_pair(cm), iLam = ks::exp_pair(make_float2(-cm.x, -cm.y));
        const float2 Lamx = ks::exp_pair(make_float2(cm.x - lg.x, cm.y - lg.y));
        const int e = 2 * hf;
        const float2 dat = make_float2(dAt[nt][e], dAt[nt][e + 1]);
        const float2 drt = __fadd2_rn(make_float2(dRt[nt][e], dRt[nt][e + 1]), make_float2(dQy[nt][e], dQy[nt][e + 1]));
        const float2 dbb = __fadd2_rn(make_float2(dBb[nt][e], dBb[nt][e + 1]), make_float2(dBp[nt][e], dBp[nt][e + 1]));
        const float2 dkb = __fadd2_rn(make_float2(dKb[nt][e], dKb[nt][e + 1]), make_float2(dKp[nt][e], dKp[nt][e + 1]));
        const float2 oda = __fmul2_rn(dat, Lamx), odr = __fmul2_rn(drt, Lam);
        const float2 odk = __fmul2_rn(dkb, iLam), odb = __fmul2_rn(dbb, iLam);
        const float2 dcx = __fmul2_rn(__fmul2_rn(dat, aa), Lamx);
        // drt r Lam - dkb k iLam - dbb b iLam + dcx
        const float2 t1 = __fmul2_rn(__fmul2_rn(drt, rr), Lam);
        const float2 t2 = __fmul2_rn(__fmul2_rn(dkb, kk), iLam);
        const float2 t3 = __fmul2_rn(__fmul2_rn(dbb, bb), iLam);
        const float2 uu = __fadd2_rn(__fadd2_rn(__fadd2_rn(t1, make_float2(-t2.x, -t2.y)),
                                                make_float2(-t3.x, -t3.y)), dcx);
        cx[nt][0][hf] = dcx.x;
        cx[nt][1][hf] = dcx.y;
        u[nt][0][hf] = uu.x;
        u[nt][1][hf] = uu.y;
        lws[nt][0][hf] = lg.x;
        lws[nt][1][hf] = lg.y;
        *reinterpret_cast<__nv_bfloat162*>(G.raw[3] + o) = __floats2bfloat162_rn(oda.x, oda.y);
        *reinterpret_cast<__nv_bfloat162*>(G.raw[0] + o) = __floats2bfloat162_rn(odr.x, odr.y);
        *reinterpret_cast<__nv_bfloat162*>(G.raw[2] + o) = __floats2bfloat162_rn(odk.x, odk.y);
        *reinterpret_cast<__nv_bfloat162*>(G.raw[4] + o) = __floats2bfloat162_rn(odb.x, odb.y);
      }
    // reverse scans along t: dlw_s = sum_{t>=s} (dcum_t + dcumx_t) - dcumx_s, with dll
    // added at the last step; rows gq + 8 hf sit in the 8 lanes of equal q (lane stride 4)
    if (gq == 7)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int x = 0; x < 2; ++x) u[nt][x][1] += G.dll[j0 + 8 * nt + 2 * q + x];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float s1 = u[nt][x][1];  // suffix over rows 8..15
#pragma unroll
        for (int d = 1; d < 8; d <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, s1, 4 * d);
          if (gq + d < 8) s1 += y;
        }
        const float tot1 = __shfl_sync(0xffffffffu, s1, q);
        float s0 = u[nt][x][0];  // suffix over rows 0..7
#pragma unroll
        for (int d = 1; d < 8; d <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, s0, 4 * d);
          if (gq + d < 8) s0 += y;
        }
        s0 += tot1;
        u[nt][x][0] = s0 - cx[nt][x][0];
        u[nt][x][1] = s1 - cx[nt][x][1];
      }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int t = gq + 8 * hf, jj = j0 + 8 * nt + 2 * q;
        float dwv[2];
#pragma unroll
        for (int x = 0; x < 2; ++x) dwv[x] = u[nt][x][hf] * dlog_decay(lws[nt][x][hf], p.g.decay);
        *reinterpret_cast<__nv_bfloat162*>(G.raw[1] + tma::swz(t, jj)) = __floats2bfloat162_rn(dwv[0], dwv[1]);
      }
    __syncthreads();
    {  // output tiles -> global, one 16-byte piece of each tile per thread (rows past T skipped)
      const int t = tid >> 3, k = tid & 7;
      const int64_t tg = c * L + t;
      if (tg < p.g.T) {
        const int64_t off = walk.base(p.g) + tg * p.g.tstride() + 8 * k;
        const int o = tma::swz(t, 8 * k);
        bf16* const dst[5] = {static_cast<bf16*>(p.dr), static_cast<bf16*>(p.dw),
                              static_cast<bf16*>(p.dk), static_cast<bf16*>(p.da),
                              static_cast<bf16*>(p.db)};
#pragma unroll
        for (int i = 0; i < 5; ++i)
          *reinterpret_cast<uint4*>(dst[i] + off) = *reinterpret_cast<const uint4*>(G.raw[i] + o);
      }
    }
    __syncthreads();  // every tile and the scratch free: load the next item
    walk.next(p.g);
    if (tid == 0 && next < total) {
      issue_a(G, P, walk);
      ++issued_a;
      issue_b(G, P, walk);
      ++issued_b;
    }
  }
  if (tid == 0) {
    // after a timeout, let loads still in flight land before the CTA exits
    if (issued_a > seen_a) mbar_wait(&G.barA, static_cast<uint32_t>((issued_a - 1) & 1));
    if (issued_b > seen_b) mbar_wait(&G.barB, static_cast<uint32_t>((issued_b - 1) & 1));
  }
}

}  // namespace kb

unsigned int bwd_timeouts() {
  unsigned int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_wkv7_timeouts, sizeof(n)) != cudaSuccess) return ~0u;
  return n;
}

// test hook: the wait limit of this file's kernels
cudaError_t bwd_test_hooks(long long wait_limit_cycles) {
  return cudaMemcpyToSymbol(g_wkv7_wait_limit, &wait_limit_cycles, sizeof(long long));
}

size_t ckpt_bytes(int64_t chains, int64_t T) {
  return rec::ckpt_bytes(chains, (T + kChunk - 1) / kChunk);
}

size_t infer_bytes(int64_t chains, int64_t T) {
  return rec::infer_bytes(chains, (T + kChunk - 1) / kChunk);
}

size_t work_bytes(int64_t chains, int64_t T) {
  return rec::work_bytes(chains, (T + kChunk - 1) / kChunk);
}

cudaError_t launch_bwd(const BwdArgs& p, void* work, cudaStream_t stream) {
  if (!tma::bind_context()) return cudaErrorNoDevice;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int rb = rows_per_cta(p.g.chains(), sms);
  vb::Params V;
  V.a = p;
  V.work = work;
  if (!tma::encode_bhtn(&V.map_v, p.v, p.g.B, p.g.T, p.g.H) ||
      !tma::encode_bhtn(&V.map_dy, p.dy, p.g.B, p.g.T, p.g.H) ||
      !tma::encode_bhtn_cols(&V.map_dv, p.dv, p.g.B, p.g.T, p.g.H, 16 * rb, false))
    return cudaErrorInvalidValue;
  if (p.dsa != nullptr && !tma::encode_bhtn_cols(&V.map_dsa, p.dsa, p.g.B, p.g.T, p.g.H, 16 * rb, true))
    return cudaErrorInvalidValue;
  cudaError_t e = rb == 1 ? vb::launch<1>(V, p.g.chains(), stream)
                : rb == 2 ? vb::launch<2>(V, p.g.chains(), stream)
                          : vb::launch<4>(V, p.g.chains(), stream);
  if (e != cudaSuccess) return e;

  // a carried backward that wants only dv and the start-state gradient
  // (dr, dw, dk, da, db all null) needs no key-side pass
  if (p.dr == nullptr && p.dw == nullptr && p.dk == nullptr && p.da == nullptr && p.db == nullptr)
    return cudaGetLastError();
  kb::Params K;
  K.a = p;
  K.work = work;
  const void* src[7] = {p.r, p.w, p.k, p.a, p.b, p.v, p.dy};
  for (int t = 0; t < 7; ++t)
    if (!tma::encode_bhtn(&K.in[t], src[t], p.g.B, p.g.T, p.g.H)) return cudaErrorInvalidValue;
  const size_t ksmem = sizeof(kb::KGroup) + 1024;
  e = cudaFuncSetAttribute(kb::keyside_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)ksmem);
  if (e != cudaSuccess) return e;
  const int64_t items = p.g.chains() * p.g.nchunk;
  const int64_t kgrid = items < 4LL * sms ? items : 4LL * sms;  // 4 CTAs per SM
  kb::keyside_bwd_kernel<<<(unsigned)kgrid, kb::kThreads, ksmem, stream>>>(K);
  return cudaGetLastError();
}

}  // namespace chunked
}  // namespace camoe
