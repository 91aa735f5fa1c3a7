// Chunked WKV-7 ClampW forward on the tensor cores (bf16 operands, fp32
// accumulation and fp32 state), the bf16 path of the operator.
//
// Per chain (b, h), chunks of L = 16 steps are processed in order.  With the
// log-decay lw = -e^{-1/2} sigmoid(w_in) (camoe/cuda/rwkv7_clampw.cu:42; or
// -exp(w_in) for the wind_backstepping decay, camoe/cuda/wkv7_cuda.cu:21),
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
// 0.545, so 1/Lam <= 0.545^-16 ~ 1.6e4: nothing over- or underflows.  The
// wind decay has no such bound; RWKV-7's time mix feeds it w_in <= -1/2
// (the same 0.545 bound), and fp32 1/Lam stays finite while the chunk's
// summed -lw stays below 88 (w_in up to about 1.7 in every step).
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
    float S[8][4];  // element (i0 + g (+8 for e >= 2), 8 nt + 2q + (e & 1))
    if (p.s0 != nullptr) {
      const float* s0 = p.s0 + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float2 lo = *reinterpret_cast<const float2*>(s0 + 8 * nt);
        const float2 hi = *reinterpret_cast<const float2*>(s0 + 8 * kN + 8 * nt);
        S[nt][0] = lo.x; S[nt][1] = lo.y; S[nt][2] = hi.x; S[nt][3] = hi.y;
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] = 0.f;
    }
    bf16* yp = static_cast<bf16*>(p.y);
    for (int64_t c = 0; c < nchunk; ++c) {
      const int s = static_cast<int>(c % NS);
      if (!mbar_wait(&sm.full[s], static_cast<uint32_t>((c / NS) & 1))) break;
      const Slot& sl = sm.slot[s];

      uint32_t sA[4][4], vA[4], b[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) acc_to_a(sA[kk], S[2 * kk], S[2 * kk + 1]);
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
    if (p.sT != nullptr) {  // after a timed-out wait this is the state reached so far
      float* sT = p.sT + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        *reinterpret_cast<float2*>(sT + 8 * nt) = make_float2(S[nt][0], S[nt][1]);
        *reinterpret_cast<float2*>(sT + 8 * kN + 8 * nt) = make_float2(S[nt][2], S[nt][3]);
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
      const int nvalid = T - c * L < L ? static_cast<int>(T - c * L) : L;
      ks::decays<true>(raw[R_R], raw[R_W], raw[R_K], raw[R_A], raw[R_B], &sc.At[0][0], &sc.Rt[0][0],
                       Padded{LD}, &sl.Kb[0][0], &sl.Bb[0][0], Padded{LD}, sl.lam, nullptr, nullptr, gtid,
                       p.g.decay, nvalid);
      {  // v tile -> slot, un-swizzled (one 16-byte piece per thread)
        const int u = gtid >> 3, part = gtid & 7;
        *reinterpret_cast<uint4*>(&sl.v[u][part * 8]) =
            *reinterpret_cast<const uint4*>(&raw[R_V][tma::swz(u, part * 8)]);
      }
      named_sync(bar_id, 128);
      ks::grams(&sc.At[0][0], &sc.Rt[0][0], Padded{LD}, &sl.Bb[0][0], &sl.Kb[0][0], Padded{LD}, sc.Ga,
                sc.Bm, sc.Cm, sc.Dm, gw, lane);
      named_sync(bar_id, 128);
      if (gw == 0) ks::inverse(sc.Ga, sc.Tf, sc.Mf, sc.Ti, lane);
      named_sync(bar_id, 128);
      ks::w_and_q(sc.Ti, &sc.At[0][0], Padded{LD}, sc.Bm, &sl.W[0][0], Padded{LD}, &sl.Q[0][0],
                  Padded{LDS}, gw, lane);
      named_sync(bar_id, 128);
      ks::qy_and_p(sc.Cm, &sl.W[0][0], Padded{LD}, &sc.Rt[0][0], Padded{LD}, &sl.Q[0][0], Padded{LDS},
                   sc.Dm, &sl.Qy[0][0], Padded{LD}, &sl.P[0][0], Padded{LDS}, gw, lane);
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

// ===========================================================================
// Forward with a checkpoint: two kernels.
//
// keyside_kernel (chunk-parallel, every SM): for every (chain, chunk) the key
// side matrices W, Qy, Bb, Kb, Q, P and lam, written as one rec::KeyRec into
// the checkpoint buffer.  Groups of 4 warps work on independent chunks; two
// groups per CTA, grid-stride over all chunks, TMA loads one chunk ahead.
//
// value_fwd_kernel (one CTA per chain): 4 value warps hold the state rows as
// mma accumulators and walk the chunks in order; a producer warp streams each
// chunk's KeyRec (one bulk copy) and v tile (TMA) into a ring of NS slots.
// The value warps write y, sa and, at the start of every even chunk >= 2, the
// bf16 state (rec::state_ptr) for the backward.
// ===========================================================================

namespace ka {

constexpr int kGroups = 2;
constexpr int kThreads = 128 * kGroups;
constexpr int NR = 2;  // input buffers per group

struct alignas(1024) Group {
  bf16 raw[NR][5][L * kN];  // r, w, k, a, b tiles as landed by TMA (1 KiB aligned)
  struct Out {
    rec::KeyRec k;
    rec::TriRec t;
  } out[2];                 // the records, written in place, then bulk-stored; two, so
                            // the stores of one item overlap the next
  Tile At, Rt;
  Tile16 Dm, Ti;
  float Ga[L][L + 1], Mf[8][9];
  float lam[kN];
  uint64_t rawbar[NR];
};

struct Params {
  CUtensorMap maps[5];  // r, w, k, a, b
  Geom g;
  void* ckpt;        // record base: KeyRec array, then TriRec array
  bool tri = true;   // store the TriRecs (only the backward reads them)
};

// loads of the item at walk position w into raw buffer rb
__device__ __forceinline__ void issue(Group& G, int rb, const Params& P, const ItemWalk& w) {
  const int h = w.head(P.g), b = static_cast<int>(w.b), t0 = static_cast<int>(w.c * L);
  mbar_arrive_expect_tx(&G.rawbar[rb], 5 * tma::kTileBytes);
#pragma unroll
  for (int t = 0; t < 5; ++t) tma::load_tile(G.raw[rb][t], &P.maps[t], h, t0, b, &G.rawbar[rb]);
}

__global__ void __launch_bounds__(kThreads) keyside_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Group* groups = reinterpret_cast<Group*>(smem_raw + ((1024u - (sm_addr(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = warp >> 2, gw = warp & 3, gtid = tid & 127, bar_id = 1 + grp;
  Group& G = groups[grp];
  if (gtid == 0) {
    for (int i = 0; i < NR; ++i) mbar_init(&G.rawbar[i], 1);
    mbar_fence_init();
  }
  named_sync(bar_id, 128);
  const int64_t total = P.g.chains() * P.g.nchunk;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * kGroups + grp;
  const int64_t ngroups = static_cast<int64_t>(gridDim.x) * kGroups;
  // cur: this group's current item; ahead: the item NR steps further, whose
  // loads go out once the current item has released its raw buffer
  ItemWalk cur, ahead;
  cur.init(P.g, gid, ngroups);
  ahead = cur;
  for (int i = 0; i < NR; ++i) {
    if (gtid == 0 && gid + i * ngroups < total) issue(G, i, P, ahead);
    ahead.next(P.g);
  }
  int64_t j = 0;
  for (;; ++j) {
    const int64_t item = gid + j * ngroups;
    if (item >= total) break;
    const int rb = static_cast<int>(j % NR);
    bool ok = mbar_wait(&G.rawbar[rb], static_cast<uint32_t>((j / NR) & 1));
    if (gtid == 0) bulk_wait_read_n<1>();  // the record of item j - 2 has left out[j & 1]
    ok = named_sync_and(bar_id, 128, ok);
    if (!ok) break;
    rec::KeyRec& o = G.out[j & 1].k;
    rec::TriRec& tr = G.out[j & 1].t;
    // steps past T (a ragged last chunk) do not decay the state
    int nvalid = L;
    if ((P.g.T & (L - 1)) != 0 && cur.c == P.g.nchunk - 1) nvalid = static_cast<int>(P.g.T - cur.c * L);
    ks::decays<true>(G.raw[rb][0], G.raw[rb][1], G.raw[rb][2], G.raw[rb][3], G.raw[rb][4],
                     &G.At[0][0], &G.Rt[0][0], Padded{LD}, o.Kb, o.Bb, Swz64{}, o.lam, nullptr,
                     nullptr, gtid, P.g.decay, nvalid);
    named_sync(bar_id, 128);
    if (gtid == 0 && item + NR * ngroups < total) issue(G, rb, P, ahead);
    ahead.next(P.g);
    ks::grams(&G.At[0][0], &G.Rt[0][0], Padded{LD}, o.Bb, o.Kb, Swz64{}, G.Ga, tr.Bm, tr.Cm, G.Dm,
              gw, lane);
    named_sync(bar_id, 128);
    if (gw == 0) ks::inverse(G.Ga, tr.Tf, G.Mf, G.Ti, lane);
    named_sync(bar_id, 128);
    ks::w_and_q(G.Ti, &G.At[0][0], Padded{LD}, tr.Bm, o.W, Swz64{}, o.Q, Swz16{}, gw, lane);
    named_sync(bar_id, 128);
    ks::qy_and_p(tr.Cm, o.W, Swz64{}, &G.Rt[0][0], Padded{LD}, o.Q, Swz16{}, G.Dm, o.Qy, Swz64{},
                 o.P, Swz16{}, gw, lane);
    fence_proxy_async();
    named_sync(bar_id, 128);
    if (gtid == 0) {
      bulk_s2g(rec::keyrec(P.ckpt, cur.ch, P.g.nchunk, cur.c), &o, sizeof(rec::KeyRec));
      if (P.tri) bulk_s2g(rec::trirec(P.ckpt, P.g.chains(), cur.ch, P.g.nchunk, cur.c), &tr, sizeof(rec::TriRec));
      bulk_commit();
    }
    cur.next(P.g);
  }
  if (gtid == 0) {
    bulk_wait_all();
    // after a timeout, let loads in flight land before the CTA exits
    for (int64_t jj = j; jj < j + NR; ++jj)
      if (gid + jj * ngroups < total) mbar_wait(&G.rawbar[jj % NR], static_cast<uint32_t>((jj / NR) & 1));
  }
}

}  // namespace ka

namespace vf {

// As in the backward (wkv7_chunked_bwd.cu), a chain's 64 state rows are split
// over 4 / RB CTAs of RB row blocks.  Per row block:
//   S warp   carries the fp32 state through the sequence (SA and the update:
//            the critical path).  It loads all of a chunk's operand fragments
//            before its mma chains and publishes the chunk's start state next
//            to the chunk's inputs only after them, so no shared-memory store
//            sits in front of its loads; it issues no fence, no output store
//            and one mbarrier wait per chunk (each costs a round trip of
//            about 50-120 cycles): the published state lives in the chunk's
//            input slot, which is refilled only after the Y warp has
//            released it, so no "buffer free" check is needed.  It writes sa
//            straight from its accumulators to global memory (store
//            instructions, off its dependency chain): staging sa through a
//            second consumer warp cost that warp a recomputation of SA on the
//            SMSPs the Y warps use, which then set the pace;
//   Y warp   reads the published start state, forms Y and stages y and (even
//            chunks) the checkpoint copy of the start state.
// A producer warp streams each chunk's KeyRec and v tile; a store warp writes
// the staged tiles (TMA tile stores, bulk copies) with KEEP groups in flight.

struct alignas(1024) Slot {
  bf16 v[L * kN];  // v tile as landed by TMA (1 KiB aligned)
  rec::KeyRec k;
};

template <int RB>
struct alignas(128) Pub {
  bf16 S[16 * RB * kN];  // Swz64 rows: a chunk's start state
};

template <int RB>
struct alignas(1024) Stage {
  bf16 y[L][16 * RB];    // [t][i] of this CTA's rows (TMA store)
  bf16 S[16 * RB * kN];  // Swz64 rows: checkpoint copy of the start state
};

template <int RB>
struct Smem {
  // input slots (even), output stages (power of two) and store groups left
  // reading shared memory (< NX)
  static constexpr int NS = RB == 4 ? 8 : 12;
  static constexpr int NX = RB == 1 ? 8 : 4;
  static constexpr int KEEP = NX / 2;
  Slot slot[NS];
  Stage<RB> st[NX];
  Pub<RB> pub[NS];  // start state of the chunk in slot s
  // inputs land two chunks at a time on one barrier (consumers wait once per pair)
  uint64_t fullp[NS / 2], empty[NS], pfull[NS], done[NX], sempty[NX];
};

struct Params {
  CUtensorMap map_v, map_y;
  FwdArgs a;
};

// Test hook (camoe_wkv7_test_hooks): the producer never issues the loads of
// this chunk pair, so every role's next wait runs out and the kernel returns
// with the timeouts counted.  -1 (the default) withholds nothing.
static __device__ int g_test_skip_pair = -1;

__device__ __forceinline__ uint32_t par(int idx, int n) { return static_cast<uint32_t>((idx / n) & 1); }

template <int RB>
__global__ void __launch_bounds__(32 * (2 * RB + 2), 1) value_fwd_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem<RB>& sm = *reinterpret_cast<Smem<RB>*>(smem_raw + ((1024u - (sm_addr(smem_raw) & 1023u)) & 1023u));
  constexpr int NRG = 4 / RB;  // CTAs per chain
  constexpr int NS = Smem<RB>::NS, NX = Smem<RB>::NX, KEEP = Smem<RB>::KEEP;
  const FwdArgs& p = P.a;
  // warps [S x RB][Y x RB][producer][store]: with RB == 2 the two S warps run on
  // SMSPs 0 and 1 beside the light producer and store warps, the Y warps on 2, 3
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ch = blockIdx.x / NRG;
  const int row0 = 16 * RB * static_cast<int>(blockIdx.x % NRG);
  const int nchunk = static_cast<int>(p.g.nchunk);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      if (s < NS / 2) mbar_init(&sm.fullp[s], 1);
      mbar_init(&sm.empty[s], RB);  // the Y warps (see the S warp)
    }
    for (int x = 0; x < NS; ++x) mbar_init(&sm.pfull[x], RB);
    for (int x = 0; x < NX; ++x) {
      mbar_init(&sm.done[x], RB);
      mbar_init(&sm.sempty[x], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  const int hh = static_cast<int>(p.g.h0 + ch % p.g.hc), bb = static_cast<int>(ch / p.g.hc);
  // records come from the checkpoint (training) or the workspace (inference);
  // only a checkpoint receives the bf16 states for the backward
  void* const recs = p.ckpt != nullptr ? static_cast<void*>(p.ckpt) : p.work;
  const bool states = p.ckpt != nullptr;
  if (warp == 2 * RB) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    constexpr int NB = NS / 2;
    const int skip = *static_cast<volatile int*>(&g_test_skip_pair);
    int pc = 0;
    bool ok = true;
    for (; 2 * pc < nchunk && ok; ++pc) {
      const int c0 = 2 * pc, n = nchunk - c0 < 2 ? nchunk - c0 : 2;
      for (int k = 0; k < n && ok; ++k) {
        const int c = c0 + k;
        if (c >= NS) ok = mbar_wait(&sm.empty[c % NS], par(c - NS, NS));
      }
      if (!ok) break;
      if (pc == skip) continue;  // test hook: this pair never arrives
      uint64_t* bar = &sm.fullp[pc % NB];
      mbar_arrive_expect_tx(bar, n * (sizeof(rec::KeyRec) + tma::kTileBytes));
      for (int k = 0; k < n; ++k) {
        const int c = c0 + k, s = c % NS;
        bulk_g2s(&sm.slot[s].k, rec::keyrec(recs, ch, nchunk, c), sizeof(rec::KeyRec), bar);
        tma::load_tile(sm.slot[s].v, &P.map_v, hh, c * L, bb, bar);
      }
    }
    // stopped on a timeout, or a pair withheld (the consumers then stop early):
    // let the copies in flight land.  Pairs older than the last NB were
    // consumed before their slots were refilled; the withheld pair's wait runs
    // out (bounded) since nothing arrives on it.
    if (!ok || skip >= 0)
      for (int pp = pc > NB ? pc - NB : 0; pp < pc; ++pp) mbar_wait(&sm.fullp[pp % NB], par(pp, NB));
    return;
  }

  if (warp == 2 * RB + 1) {
    // ------------------------------ store warp ------------------------------
    if (lane != 0) return;
    const int64_t chains = p.g.chains();
    for (int c = 0; c < nchunk; ++c) {
      const int x = c & (NX - 1);
      if (!mbar_wait(&sm.done[x], par(c, NX))) break;
      const Stage<RB>& st = sm.st[x];
      tma::store_tile(&P.map_y, &st.y[0][0], row0, hh, c * L, bb);
      if (states && c >= 2 && (c & 1) == 0)
        bulk_s2g(rec::state_ptr(p.ckpt, chains, ch, nchunk, c) + row0 * 128, st.S, 2048 * RB);
      bulk_commit();
      bulk_wait_read_n<KEEP>();
      if (c >= KEEP) mbar_arrive(&sm.sempty[(c - KEEP) & (NX - 1)]);
    }
    bulk_wait_all();
    return;
  }

  const int role = warp / RB, r = warp % RB;
  const int il = 16 * r, i0 = row0 + il;
  const int g = lane >> 2, q = lane & 3;
  if (role == 0) {
    // ------------------------------ S warp: the state recurrence ------------------------------
    float S[8][4];  // element (i0 + g (+8 for e >= 2), 8 nt + 2q + (e & 1))
    if (p.s0 != nullptr) {
      const float* s0 = p.s0 + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float2 lo = *reinterpret_cast<const float2*>(s0 + 8 * nt);
        const float2 hi = *reinterpret_cast<const float2*>(s0 + 8 * kN + 8 * nt);
        S[nt][0] = lo.x; S[nt][1] = lo.y; S[nt][2] = hi.x; S[nt][3] = hi.y;
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] = 0.f;
    }
    // sa element (t, i) of this warp's rows goes to sa_row[t * ts + i]
    float* const sa_row = p.sa + p.g.base(ch) + i0 + g;
    const int64_t ts = p.g.tstride(), T = p.g.T;
    if (nchunk > 0 && !mbar_wait(&sm.fullp[0], 0)) return;
    for (int c = 0; c < nchunk; ++c) {
      const int s = c % NS;
      const rec::KeyRec& kr = sm.slot[s].k;
      uint32_t bW[4][4], bQ[4], bB[4][4], bK[4][4], vA[4];
      float2 lam[8];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ldb_nk(bW[kk], kr.W, Swz64{}, 0, 16 * kk, lane);
        ldb_kn(bB[kk], kr.Bb, Swz64{}, 16 * kk, 0, lane);
        ldb_kn(bK[kk], kr.Kb, Swz64{}, 16 * kk, 0, lane);
      }
      ldb_nk(bQ, kr.Q, Swz16{}, 0, 0, lane);
      lda_cm(vA, sm.slot[s].v, Swz64{}, i0, 0, lane);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) lam[nt] = *reinterpret_cast<const float2*>(&kr.lam[8 * nt + 2 * q]);
      uint32_t sA[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) acc_to_a(sA[kk], S[2 * kk], S[2 * kk + 1]);
      float sa[2][4];
      mma_k64_k16(sa, sA, vA, bW, bQ);
      // S' = (S + SA^T Bb + V^T Kb) diag(lam)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        mma16816(S[2 * m], vA, bK[m][0], bK[m][1]);
        mma16816(S[2 * m + 1], vA, bK[m][2], bK[m][3]);
      }
      uint32_t saA[4];
      acc_to_a(saA, sa[0], sa[1]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        mma16816(S[2 * m], saA, bB[m][0], bB[m][1]);
        mma16816(S[2 * m + 1], saA, bB[m][2], bB[m][3]);
      }
      // sa of the chunk: element (t = 16c + 8 nt + 2q + (e & 1), i = i0 + g (+8 for e >= 2))
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t t = static_cast<int64_t>(c) * L + 8 * nt + 2 * q + (e & 1);
          if (t < T) sa_row[t * ts + (e >= 2 ? 8 : 0)] = sa[nt][e];
        }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        S[nt][0] *= lam[nt].x; S[nt][1] *= lam[nt].y; S[nt][2] *= lam[nt].x; S[nt][3] *= lam[nt].y;
      }
      // publish the chunk's start state beside its inputs
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) sta_rm(sm.pub[s].S, Swz64{}, il, 16 * kk, sA[kk], lane);
      __syncwarp();
      if (lane == 0) {
        // no release of slot s here: the Y warps release it after waiting for
        // this publication, which follows every read of the slot above
        mbar_arrive(&sm.pfull[s]);
      }
      if (c + 1 < nchunk && ((c + 1) & 1) == 0 &&
          !mbar_wait(&sm.fullp[((c + 1) >> 1) % (NS / 2)], par((c + 1) >> 1, NS / 2)))
        return;
    }
    if (p.sT != nullptr) {
      float* sT = p.sT + p.g.state_off(ch) + (i0 + g) * kN + 2 * q;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        *reinterpret_cast<float2*>(sT + 8 * nt) = make_float2(S[nt][0], S[nt][1]);
        *reinterpret_cast<float2*>(sT + 8 * kN + 8 * nt) = make_float2(S[nt][2], S[nt][3]);
      }
    }
    return;
  }

  // ------------------------------ Y warp (role 1) ------------------------------
  for (int c = 0; c < nchunk; ++c) {
    const int s = c % NS, x = c & (NX - 1);
    if ((c & 1) == 0 && !mbar_wait(&sm.fullp[(c >> 1) % (NS / 2)], par(c >> 1, NS / 2))) return;
    const rec::KeyRec& kr = sm.slot[s].k;
    uint32_t bM[4][4], bV[4], vA[4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) ldb_nk(bM[kk], kr.Qy, Swz64{}, 0, 16 * kk, lane);
    ldb_nk(bV, kr.P, Swz16{}, 0, 0, lane);
    lda_cm(vA, sm.slot[s].v, Swz64{}, i0, 0, lane);
    if (!mbar_wait(&sm.pfull[s], par(c, NS))) return;
    uint32_t sA[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) lda_rm(sA[kk], sm.pub[s].S, Swz64{}, il, 16 * kk, lane);
    // Y = Qy S^T + P V
    float acc[2][4];
    mma_k64_k16(acc, sA, vA, bM, bV);
    if (c >= NX && !mbar_wait(&sm.sempty[x], par(c - NX, NX))) return;
    Stage<RB>& st = sm.st[x];
    uint32_t yA[4];
    acc_to_a(yA, acc[0], acc[1]);
    sta_cm(&st.y[0][0], Padded{16 * RB}, il, 0, yA, lane);
    if (states && c >= 2 && (c & 1) == 0)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) sta_rm(st.S, Swz64{}, il, 16 * kk, sA[kk], lane);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&sm.done[x]);
      mbar_arrive(&sm.empty[s]);
    }
  }
}

template <int RB>
cudaError_t launch(const Params& V, int64_t chains, cudaStream_t stream) {
  const size_t smem = sizeof(Smem<RB>) + 1024;
  cudaError_t e = cudaFuncSetAttribute(value_fwd_kernel<RB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  value_fwd_kernel<RB><<<static_cast<unsigned>(chains * (4 / RB)), 32 * (2 * RB + 2), smem, stream>>>(V);
  return cudaGetLastError();
}

}  // namespace vf


// wait timeouts recorded by this file's kernels on the current device
unsigned int fwd_timeouts() {
  unsigned int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_wkv7_timeouts, sizeof(n)) != cudaSuccess) return ~0u;
  return n;
}

// test hook: the wait limit of this file's kernels, and the chunk pair whose
// loads value_fwd_kernel's producer withholds (-1: none)
cudaError_t fwd_test_hooks(long long wait_limit_cycles, int skip_pair) {
  cudaError_t e = cudaMemcpyToSymbol(g_wkv7_wait_limit, &wait_limit_cycles, sizeof(long long));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(vf::g_test_skip_pair, &skip_pair, sizeof(int));
  return e;
}

cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream) {
  if (!tma::bind_context()) return cudaErrorNoDevice;
  if (p.ckpt == nullptr && p.work == nullptr) {  // inference: one fused kernel, nothing stored
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
  // key-side records over all SMs, then the sequential value pass (training:
  // into the checkpoint, with TriRecs and states; inference: into the workspace)
  ka::Params K;
  K.g = p.g;
  K.ckpt = p.ckpt != nullptr ? static_cast<void*>(p.ckpt) : p.work;
  K.tri = p.ckpt != nullptr;
  const void* ksrc[5] = {p.r, p.w, p.k, p.a, p.b};
  for (int t = 0; t < 5; ++t)
    if (!tma::encode_bhtn(&K.maps[t], ksrc[t], p.g.B, p.g.T, p.g.H)) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int rb = rows_per_cta(p.g.chains(), sms);
  vf::Params V;
  V.a = p;
  if (!tma::encode_bhtn(&V.map_v, p.v, p.g.B, p.g.T, p.g.H) ||
      !tma::encode_bhtn_cols(&V.map_y, p.y, p.g.B, p.g.T, p.g.H, 16 * rb, false))
    return cudaErrorInvalidValue;
  if (!(p.records_ready && p.ckpt != nullptr)) {
    const size_t ksmem = ka::kGroups * sizeof(ka::Group) + 1024;
    cudaError_t e = cudaFuncSetAttribute(ka::keyside_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ksmem);
    if (e != cudaSuccess) return e;
    const int64_t items = p.g.chains() * p.g.nchunk;
    const int64_t want = (items + ka::kGroups - 1) / ka::kGroups;
    const int64_t kgrid = want < 2LL * sms ? want : 2LL * sms;
    ka::keyside_kernel<<<(unsigned)kgrid, ka::kThreads, ksmem, stream>>>(K);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }

  return rb == 1 ? vf::launch<1>(V, p.g.chains(), stream)
       : rb == 2 ? vf::launch<2>(V, p.g.chains(), stream)
                 : vf::launch<4>(V, p.g.chains(), stream);
}

}  // namespace chunked
}  // namespace camoe
