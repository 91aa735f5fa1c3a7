// Per-step WKV-7 ClampW scan on CUDA cores, fp32 state and arithmetic: the
// fp32-exact path of the operator (any element type in, fp32 math).
//
// Forward (scan_fwd_kernel): the state rows are independent recurrences that
// share the transition, so a chain's 64 rows are split over 4 CTAs of 16
// rows; 16 threads own one row (4 state columns each in registers, 8 warps per
// CTA so each SMSP switches between warps of the latency-bound step loop) and
// combine row sums (sa = S a, y = S r) with four xor-shuffles.  Chunks of 16
// steps of r, w, k, a, b (and the CTA's slice of v) are streamed into shared
// memory with cp.async, double-buffered, and converted once per chunk
// (decay w = exp(log_decay(w_in)) computed there, ClampW or wind).  The state at the
// start of every chunk is the checkpoint, stored row-major in fp32.
//
// Backward (scan_bwd_kernel): one cluster of two 256-thread CTAs per chain,
// each owning 32 rows of dS (row i = 32 rank + tid/8, eight columns 8q..8q+7
// with q = tid%8), walking chunks in reverse.  Each chunk's states are
// recomputed forward from its checkpoint into shared memory (all 16 in one
// pass; with one 64-row CTA per chain, two halves of 8 steps so 9 states fit),
// never reversed through 1/w as camoe/cuda/rwkv7_clampw.cu:133 does.  Per step
// the row sums (dsa = dS b, dv = dS k) use shuffles; the five column sums over
// the rows (dr, dw, dk, db, da) use a shuffle reduce-scatter over the 4 rows of
// a warp and a shared-memory pass over the 8 warps, and the two CTAs' sums are
// added once per chunk through distributed shared memory.  The elementwise
// work of both kernels runs as packed two-lane fp32 (float2) operations.
// The per-element formulas are those of camoe/cuda/rwkv7_clampw.cu:123-168,
// plus the external sa-gradient.
#include <cooperative_groups.h>

#include "wkv7_common.cuh"

namespace cg = cooperative_groups;

namespace camoe {
namespace scan {

constexpr int kRows = 16;                 // forward: state rows per CTA
constexpr int kFwdTpr = 16;               // forward: threads per row
constexpr int kFwdCols = kN / kFwdTpr;    // state columns per thread
constexpr int kFwdThreads = kRows * kFwdTpr;
static_assert(kFwdCols == 4 || kFwdCols == 8, "dot_cols takes one or two 4-column groups");
constexpr int kRowGroups = kN / kRows;    // forward: CTAs per chain
constexpr int kHalf = kChunk / 2;         // backward: states held per half chunk

template <typename Tin>
struct FwdSmem {
  Tin raw[2][5][kChunk][kN];       // r, w, k, a, b of one chunk, double-buffered
  Tin rawv[2][kChunk][kRows];      // this CTA's slice of v
  float r[kChunk][kN], w[kChunk][kN], k[kChunk][kN], a[kChunk][kN], b[kChunk][kN];
  float v[kChunk][kRows];
  float y[kChunk][kRows], sa[kChunk][kRows];
};

// one chunk's copies, element (t, j) of the chain at cb + t * ts + j
template <typename Tin>
__device__ __forceinline__ void fwd_issue(FwdSmem<Tin>& sm, int buf, const FwdArgs& p, int64_t cb,
                                          int64_t ts, int64_t c, int rg) {
  constexpr int V = 16 / sizeof(Tin);  // elements per 16-byte copy
  constexpr int PR = kN / V;           // copies per 64-wide row
  constexpr int VR = kRows / V;        // copies per v slice row
  const int64_t t0 = c * kChunk;
  const Tin* src[5] = {static_cast<const Tin*>(p.r), static_cast<const Tin*>(p.w), static_cast<const Tin*>(p.k),
                       static_cast<const Tin*>(p.a), static_cast<const Tin*>(p.b)};
  for (int idx = threadIdx.x; idx < kChunk * PR; idx += kFwdThreads) {
    const int u = idx / PR, part = idx % PR;
    const bool ok = t0 + u < p.g.T;
    const int64_t o = ok ? cb + (t0 + u) * ts + part * V : 0;
#pragma unroll
    for (int tens = 0; tens < 5; ++tens) cp_async16(&sm.raw[buf][tens][u][part * V], src[tens] + o, ok);
  }
  for (int idx = threadIdx.x; idx < kChunk * VR; idx += kFwdThreads) {
    const int u = idx / VR, part = idx % VR;
    const bool ok = t0 + u < p.g.T;
    const int64_t o = ok ? cb + (t0 + u) * ts + rg * kRows + part * V : 0;
    cp_async16(&sm.rawv[buf][u][part * V], static_cast<const Tin*>(p.v) + o, ok);
  }
}

// sum over the TPR threads of a row (the low lane bits)
template <int TPR>
__device__ __forceinline__ float row_sum(float x) {
#pragma unroll
  for (int d = 1; d < TPR; d <<= 1) x += __shfl_xor_sync(0xffffffffu, x, d);
  return x;
}

// The per-thread column arrays are float2 pairs (pair 2g + h holds elements
// 4g + 2h, 4g + 2h + 1 of register group g), so the elementwise work issues
// as packed two-lane fp32 operations (__ffma2_rn, __fmul2_rn, __fadd2_rn:
// each lane rounded as the scalar operation).
__device__ __forceinline__ float2 bc2(float x) { return make_float2(x, x); }
__device__ __forceinline__ float2 lo2(const float4& v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(const float4& v) { return make_float2(v.z, v.w); }

// this thread's part of a row dot product: its kFwdCols state columns (as
// pairs) times a shared-memory row segment.  Register group m holds column
// group m ^ sw.  With 8 columns per thread, sw = 1 for the upper four threads
// of a row, so that the eight threads of a row (a quarter warp) read eight
// different bank groups; with 4 columns a quarter warp reads 128 contiguous
// bytes and sw = 0.
constexpr int kFwdPairs = kFwdCols / 2;
__device__ __forceinline__ float dot_cols(const float2 (&S)[kFwdPairs], const float* x, int sw) {
  const float4* x4 = reinterpret_cast<const float4*>(x);
  if constexpr (kFwdCols == 4) {
    const float4 e = x4[0];
    const float2 acc = __ffma2_rn(S[1], hi2(e), __fmul2_rn(S[0], lo2(e)));
    return acc.x + acc.y;
  } else {
    const float4 e = x4[sw], f = x4[1 ^ sw];
    const float2 a0 = __ffma2_rn(S[1], hi2(e), __fmul2_rn(S[0], lo2(e)));
    const float2 a1 = __ffma2_rn(S[3], hi2(f), __fmul2_rn(S[2], lo2(f)));
    return (a0.x + a0.y) + (a1.x + a1.y);
  }
}

template <typename Tin>
__global__ void __launch_bounds__(kFwdThreads) scan_fwd_kernel(FwdArgs p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FwdSmem<Tin>& sm = *reinterpret_cast<FwdSmem<Tin>*>(smem_raw);
  const int tid = threadIdx.x, rl = tid / kFwdTpr, q = tid % kFwdTpr;
  const int sw = (kFwdCols == 8 && q >= kFwdTpr / 2) ? 1 : 0;  // register group m = column group m ^ sw
  const int64_t ch = blockIdx.x / kRowGroups;
  const int rg = blockIdx.x % kRowGroups;
  const int i = rg * kRows + rl;
  const int64_t nchunk = p.g.nchunk;
  const int64_t cb = p.g.base(ch), ts = p.g.tstride();

  float2 S[kFwdPairs];
  if (p.s0 != nullptr) {  // start state: row i, columns q kFwdCols .. q kFwdCols + kFwdCols - 1
    const float4* src = reinterpret_cast<const float4*>(p.s0 + p.g.state_off(ch) + i * kN + q * kFwdCols);
#pragma unroll
    for (int m = 0; m < kFwdCols / 4; ++m) {
      const float4 x = src[m ^ sw];
      S[2 * m] = lo2(x);
      S[2 * m + 1] = hi2(x);
    }
  } else {
#pragma unroll
    for (int pp = 0; pp < kFwdPairs; ++pp) S[pp] = make_float2(0.f, 0.f);
  }

  fwd_issue(sm, 0, p, cb, ts, 0, rg);
  cp_async_commit();
  for (int64_t c = 0; c < nchunk; ++c) {
    const int buf = c & 1;
    // steps of this chunk inside the sequence (the rest are never applied,
    // so the final state is the state after step T - 1)
    const int nu = p.g.T - c * kChunk < kChunk ? static_cast<int>(p.g.T - c * kChunk) : kChunk;
    if (c + 1 < nchunk) fwd_issue(sm, buf ^ 1, p, cb, ts, c + 1, rg);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    for (int idx = tid; idx < nu * kN; idx += kFwdThreads) {
      const int u = idx / kN, j = idx % kN;
      sm.r[u][j] = to_f32(sm.raw[buf][0][u][j]);
      sm.w[u][j] = expf(log_decay(to_f32(sm.raw[buf][1][u][j]), p.g.decay));
      sm.k[u][j] = to_f32(sm.raw[buf][2][u][j]);
      sm.a[u][j] = to_f32(sm.raw[buf][3][u][j]);
      sm.b[u][j] = to_f32(sm.raw[buf][4][u][j]);
    }
    for (int idx = tid; idx < nu * kRows; idx += kFwdThreads)
      sm.v[idx / kRows][idx % kRows] = to_f32(sm.rawv[buf][idx / kRows][idx % kRows]);
    __syncthreads();

    if (p.ckpt != nullptr && c > 0) {
      float4* dst = reinterpret_cast<float4*>(p.ckpt + ((ch * nchunk + c) * kN + i) * kN + q * kFwdCols);
#pragma unroll
      for (int m = 0; m < kFwdCols / 4; ++m)
        dst[m ^ sw] = make_float4(S[2 * m].x, S[2 * m].y, S[2 * m + 1].x, S[2 * m + 1].y);
    }

    // y_u = S_u r_u and sa_{u+1} = S_u a_{u+1} both read only S_u, so their
    // row sums run interleaved: one shuffle chain per step instead of two
    // (sa holds the whole row's sum at the top of every step)
    float sa = row_sum<kFwdTpr>(dot_cols(S, &sm.a[0][q * kFwdCols], sw));
#pragma unroll 1
    for (int u = 0; u < nu; ++u) {
      const float2 vi2 = bc2(sm.v[u][rl]), sa2 = bc2(sa);
      const float4* w4 = reinterpret_cast<const float4*>(&sm.w[u][q * kFwdCols]);
      const float4* b4 = reinterpret_cast<const float4*>(&sm.b[u][q * kFwdCols]);
      const float4* k4 = reinterpret_cast<const float4*>(&sm.k[u][q * kFwdCols]);
#pragma unroll
      for (int m = 0; m < kFwdCols / 4; ++m) {
        const float4 wv = w4[m ^ sw], bv = b4[m ^ sw], kv = k4[m ^ sw];
        S[2 * m] = __ffma2_rn(S[2 * m], lo2(wv), __ffma2_rn(sa2, lo2(bv), __fmul2_rn(lo2(kv), vi2)));
        S[2 * m + 1] = __ffma2_rn(S[2 * m + 1], hi2(wv), __ffma2_rn(sa2, hi2(bv), __fmul2_rn(hi2(kv), vi2)));
      }
      // the last step of the chunk reads a row of a again (its sum is unused)
      const int un = u + 1 < nu ? u + 1 : u;
      float y = dot_cols(S, &sm.r[u][q * kFwdCols], sw);
      float sn = dot_cols(S, &sm.a[un][q * kFwdCols], sw);
#pragma unroll
      for (int d = 1; d < kFwdTpr; d <<= 1) {
        const float yo = __shfl_xor_sync(0xffffffffu, y, d);
        const float so = __shfl_xor_sync(0xffffffffu, sn, d);
        y += yo;
        sn += so;
      }
      if (q == 0) {
        sm.y[u][rl] = y;
        sm.sa[u][rl] = sa;
      }
      sa = sn;
    }
    __syncthreads();
    // write y, sa of this chunk: thread -> (step u, 4 consecutive rows), 16 x 4 of them
    if (tid < kChunk * (kRows / 4)) {
      const int u = tid >> 2, part = tid & 3;
      const int64_t t = c * kChunk + u;
      if (t < p.g.T) {
        const int64_t o = cb + t * ts + rg * kRows + part * 4;
        const float* ys = &sm.y[u][part * 4];
        Tin* yo = static_cast<Tin*>(p.y) + o;
#pragma unroll
        for (int e = 0; e < 4; ++e) yo[e] = from_f32<Tin>(ys[e]);
        *reinterpret_cast<float4*>(p.sa + o) = *reinterpret_cast<const float4*>(&sm.sa[u][part * 4]);
      }
    }
  }
  if (p.sT != nullptr) {
    float4* dst = reinterpret_cast<float4*>(p.sT + p.g.state_off(ch) + i * kN + q * kFwdCols);
#pragma unroll
    for (int m = 0; m < kFwdCols / 4; ++m)
      dst[m ^ sw] = make_float4(S[2 * m].x, S[2 * m].y, S[2 * m + 1].x, S[2 * m + 1].y);
  }
}

// ---------------------------------------------------------------------------
// decode step (step_fwd_kernel): a few steps from a stored state, no
// checkpoint.  The cost is the state itself (16 KiB read and 16 KiB written
// per chain), so the kernel is laid out for HBM: 2 CTAs of 128 threads per
// chain (32 rows each), 8 threads per row, thread o of row pair (i, i + 16)
// holding S[i (+16)][4o + 32m .. 4o + 32m + 3] for m = 0, 1.  Each warp load
// or store instruction then moves 4 whole 128-byte lines (4 rows x 8 threads
// x 16 B), the row sums (sa = S a, y = S r) take three xor-shuffles, and each
// staged input value serves two rows.  Per step the CTA stages r, decay(w),
// k, a, b and its 32 values of v in shared memory (double-buffered, one
// barrier per step), the next step's inputs already loaded into registers;
// the arithmetic is the scan's (camoe/cuda/rwkv7_clampw.cu:48-63).  On B200
// one token for 16384 chains (256 MiB of state) takes 84.5 us, the measured
// copy bandwidth.

constexpr int kStepRows = 32;                        // rows per CTA (2 per thread)
constexpr int kStepTpr = 8;                          // threads per row
constexpr int kStepThreads = kStepRows / 2 * kStepTpr;   // 128
constexpr int kStepCtas = kN / kStepRows;            // CTAs per chain
constexpr int kStepLoaders = 5 * kN / 4 + kStepRows / 4;  // 88

// thread tid < 80 loads 4 consecutive columns of r, w, k, a, b (tensor tid / 16);
// threads 80..87 load 4 consecutive rows of this CTA's slice of v.  `src` is
// the thread's element at step 0; step t is t * tstride further.
template <typename Tin>
__device__ __forceinline__ void step_load(float (&x)[4], const Tin* src) {
  if constexpr (sizeof(Tin) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(src);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    x[0] = lo.x; x[1] = lo.y; x[2] = hi.x; x[3] = hi.y;
  }
}

template <typename Tin>
__global__ void __launch_bounds__(kStepThreads, 8) step_fwd_kernel(FwdArgs p) {
  __shared__ __align__(16) float xin[2][5][kN];
  __shared__ __align__(16) float vin[2][kStepRows];
  const int tid = threadIdx.x, rl = tid >> 3, o = tid & 7;
  const unsigned ch = blockIdx.x / kStepCtas, hc = static_cast<unsigned>(p.g.hc);
  const int rg = static_cast<int>(blockIdx.x % kStepCtas);
  const int i = rg * kStepRows + rl;  // rows i and i + 16
  const int64_t T = p.g.T, ts = p.g.tstride();
  // chain (b, h): one 32-bit division (the grid is below 2^31 chains)
  const unsigned bb = ch / hc;
  const int64_t hh = p.g.h0 + (ch - bb * hc);
  const int64_t cbase = (static_cast<int64_t>(bb) * T * p.g.H + hh) * kN;  // element (t=0, i=0)
  const int64_t srow = ((static_cast<int64_t>(bb) * p.g.H + hh) * kN + i) * kN + 4 * o;

  const Tin* src = nullptr;
  if (tid < kStepLoaders) {
    const int tens = tid < 80 ? tid >> 4 : 5;
    const int col = tid < 80 ? 4 * (tid & 15) : rg * kStepRows + 4 * (tid - 80);
    const void* base = tens == 0 ? p.r : tens == 1 ? p.w : tens == 2 ? p.k : tens == 3 ? p.a
                     : tens == 4 ? p.b : p.v;
    src = static_cast<const Tin*>(base) + cbase + col;
  }
  float x[4] = {0.f, 0.f, 0.f, 0.f};
  if (src != nullptr) step_load<Tin>(x, src);
  float S[2][8];  // S[h][4m + e] = S[i + 16h][4o + 32m + e]
  if (p.s0 != nullptr) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const float4 v = *reinterpret_cast<const float4*>(p.s0 + srow + h * 16 * kN + 32 * m);
        S[h][4 * m] = v.x; S[h][4 * m + 1] = v.y; S[h][4 * m + 2] = v.z; S[h][4 * m + 3] = v.w;
      }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) S[h][e] = 0.f;
  }
  Tin* yo = static_cast<Tin*>(p.y) + cbase + i;
  float* sao = p.sa + cbase + i;

  for (int64_t t = 0; t < T; ++t) {
    const int buf = static_cast<int>(t & 1);
    if (tid < 80) {
      const int tens = tid >> 4, col = 4 * (tid & 15);
      if (tens == 1) {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = expf(log_decay(x[e], p.g.decay));
      }
      *reinterpret_cast<float4*>(&xin[buf][tens][col]) = make_float4(x[0], x[1], x[2], x[3]);
    } else if (tid < kStepLoaders) {
      *reinterpret_cast<float4*>(&vin[buf][4 * (tid - 80)]) = make_float4(x[0], x[1], x[2], x[3]);
    }
    __syncthreads();
    if (src != nullptr && t + 1 < T) step_load<Tin>(x, src + (t + 1) * ts);

    float sa[2] = {0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const float4 av = *reinterpret_cast<const float4*>(&xin[buf][3][4 * o + 32 * m]);
#pragma unroll
      for (int h = 0; h < 2; ++h)
        sa[h] += S[h][4 * m] * av.x + S[h][4 * m + 1] * av.y + S[h][4 * m + 2] * av.z + S[h][4 * m + 3] * av.w;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      sa[h] += __shfl_xor_sync(0xffffffffu, sa[h], 1);
      sa[h] += __shfl_xor_sync(0xffffffffu, sa[h], 2);
      sa[h] += __shfl_xor_sync(0xffffffffu, sa[h], 4);
    }
    const float vi[2] = {vin[buf][rl], vin[buf][rl + 16]};
    float yv[2] = {0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int c = 4 * o + 32 * m;
      const float4 wv = *reinterpret_cast<const float4*>(&xin[buf][1][c]);
      const float4 bv = *reinterpret_cast<const float4*>(&xin[buf][4][c]);
      const float4 kv = *reinterpret_cast<const float4*>(&xin[buf][2][c]);
      const float4 rv = *reinterpret_cast<const float4*>(&xin[buf][0][c]);
      const float wa[4] = {wv.x, wv.y, wv.z, wv.w}, ba[4] = {bv.x, bv.y, bv.z, bv.w};
      const float ka[4] = {kv.x, kv.y, kv.z, kv.w}, ra[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float sv = S[h][4 * m + e] * wa[e] + (sa[h] * ba[e] + ka[e] * vi[h]);
          S[h][4 * m + e] = sv;
          yv[h] += sv * ra[e];
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      yv[h] += __shfl_xor_sync(0xffffffffu, yv[h], 1);
      yv[h] += __shfl_xor_sync(0xffffffffu, yv[h], 2);
      yv[h] += __shfl_xor_sync(0xffffffffu, yv[h], 4);
    }
    if (o == 0) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        yo[t * ts + 16 * h] = from_f32<Tin>(yv[h]);
        sao[t * ts + 16 * h] = sa[h];
      }
    }
  }
  if (p.sT != nullptr) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int m = 0; m < 2; ++m)
        *reinterpret_cast<float4*>(p.sT + srow + h * 16 * kN + 32 * m) =
            make_float4(S[h][4 * m], S[h][4 * m + 1], S[h][4 * m + 2], S[h][4 * m + 3]);
  }
}

// ---------------------------------------------------------------------------
// backward
//
// A chain's 64 rows of dS are independent recurrences (row i of the update
// dS <- dS (diag w + a b^T)^T + dy r^T only reads row i), so each chain is a
// cluster of two CTAs of 32 rows: 128 CTAs for the 64 chains of a 4-sequence
// shard instead of 64.  Every per-step output indexed by the key column j (dr,
// dw, dk, db, da) is a sum over all 64 rows: each CTA forms the sum over its
// own 32 rows per step (warp shuffles, then shared memory over its 8 warps)
// into a partial-sum buffer, and once per chunk, after a cluster barrier, each
// CTA adds its peer's partials for its half of the columns (read through
// distributed shared memory) and writes the outputs.  The partial buffers are
// double-buffered by chunk parity, so one cluster barrier per chunk keeps a
// buffer from being refilled while the peer still reads it.  dv (a sum over
// j, within a row) needs no exchange.

// ROWS = 32: a cluster of two CTAs per chain, eight threads per row (8
// columns each): 16 warps per chain, so that every SMSP has two warps of the
// latency-bound step loop to switch between, and the per-step partial sums
// double-buffered (one block barrier per step).  ROWS = 64: one CTA per chain
// (taken when two CTAs per chain would not fit the SMs in one wave), four
// threads per row and one partial-sum buffer, to fit its shared memory.
template <int ROWS>
struct BwdCfg {
  static constexpr int kCtas = kN / ROWS;        // CTAs per chain (one cluster)
  static constexpr int kTpr = ROWS == 32 ? 8 : 4;   // threads per state row
  static constexpr int kCols = kN / kTpr;           // columns per thread
  static constexpr int kThreads = ROWS * kTpr;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kRed = ROWS == 32 ? 2 : 1;   // per-step partial-sum buffers
  static constexpr int kParts = kCtas > 1 ? 2 : 1;  // per-chunk partial-sum buffers (by parity)
  // 32 rows: all 16 states of a chunk fit in shared memory (the 17th, the end
  // state, stays in registers), one forward pass per chunk; 64 rows: two
  // halves of 8 steps, 9 states each (24 forward steps per chunk)
  static constexpr bool kWhole = ROWS == 32;
  static constexpr int kSlots = kWhole ? kChunk : kHalf + 1;
};

template <int ROWS>
struct BwdSmem {
  float S[BwdCfg<ROWS>::kSlots][ROWS][kN];  // own rows' states, in the threads' order (slot4)
  float r[kChunk][kN], w[kChunk][kN], dlw[kChunk][kN], k[kChunk][kN], a[kChunk][kN], b[kChunk][kN];
  float v[kChunk][ROWS], dy[kChunk][ROWS], dsa[kChunk][ROWS], sa[kChunk][ROWS];
  // per-warp partial column sums of one step (with two buffers, by step parity)
  float red[BwdCfg<ROWS>::kRed][BwdCfg<ROWS>::kWarps][320];
  float part[BwdCfg<ROWS>::kParts][5][kChunk][kN];  // own rows' column sums (dr, dw, dk, db, da)
  float dv[kChunk][ROWS];                          // dv of the own rows
};

// both fit the 227 KB of dynamic shared memory a CTA may have
static_assert(sizeof(BwdSmem<32>) <= 227 * 1024 && sizeof(BwdSmem<64>) <= 227 * 1024,
              "scan backward shared memory");

// Column order of a thread's registers, and where its reduced column sums go.
// The five column sums of a step are reduce-scattered over the rows of a warp
// (the lane bits above a row's threads; 2 levels for 8 threads per row, 3 for
// 4).  For the top log2(kCols / 4) levels a thread holds its 4-column groups in
// an order permuted by its row bits (register group g holds column group
// g ^ perm), so at those levels every lane keeps its first half of groups and
// adds its partner's second half, which holds the same columns: no selects.
// The last level splits the remaining 5 x 4 values by a select on the lane bit.
// The upper half of a row's threads also flip the lowest group bit: the eight
// lanes of a quarter warp then read a shared row's 16-byte pieces from eight
// different bank groups (with the natural order, threads q and q + kTpr / 2 of
// a row hit the same banks).  Partners share q, so the pairing is unchanged.
template <int ROWS>
struct Lanes {
  using Cfg = BwdCfg<ROWS>;
  static constexpr int kG = Cfg::kCols / 4;                 // 4-column groups per thread
  static constexpr int kP = kG == 2 ? 1 : 2;                // select-free levels
  static constexpr int kLevels = Cfg::kTpr == 8 ? 2 : 3;    // row bits within a warp
  static constexpr int kSelBit = 16 >> kP;                  // lane bit of the select level
  static_assert((kG == 2 || kG == 4) && kLevels == kP + 1, "one select level after the permuted ones");
  static_assert(Cfg::kThreads >= 160, "160 threads add the per-warp partial sums");
  __device__ __forceinline__ static int perm(int lane) {
    int pm = 0;
#pragma unroll
    for (int lv = 0; lv < kP; ++lv) pm += ((lane >> (4 - lv)) & 1) * (kG >> (lv + 1));
    return pm ^ ((lane % Cfg::kTpr) >= Cfg::kTpr / 2 ? 1 : 0);
  }
  // offset in part[pb] (quantity, step 0, column) of reduced value pidx, which
  // lane pidx % 32 of every warp holds in its slot pidx / 32
  __device__ __forceinline__ static int part_off(int pidx) {
    const int ln = pidx & 31, k = pidx >> 5;
    const int f = k + ((ln & kSelBit) ? 10 : 0), quant = f >> 2, e = f & 3;
    const int col = (ln % Cfg::kTpr) * Cfg::kCols + 4 * perm(ln) + e;
    return quant * kChunk * kN + col;
  }
};

// A chunk's inputs in 16-byte pieces: r, w, k, a, b as 16 steps x 16 groups of
// 4 columns (threads tid < 256 take one group), v, dy, dsa as 16 steps x
// ROWS / 4 groups of 4 own rows (threads tid < 4 ROWS take one).
template <typename Tin, int ROWS>
struct Prefetch {
  float4 c[5];  // r, w, k, a, b of the thread's column group
  float4 o[3];  // v, dy, dsa of the thread's row group
};

template <typename Tin>
__device__ __forceinline__ float4 load4(const void* base, int64_t off, bool ok) {
  if (!ok) return make_float4(0.f, 0.f, 0.f, 0.f);
  if constexpr (sizeof(Tin) == 4) {
    return *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
  } else {
    const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const bf16*>(base) + off);
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    const float2 l = __bfloat1622float2(lo), h = __bfloat1622float2(hi);
    return make_float4(l.x, l.y, h.x, h.y);
  }
}

template <typename Tin, int ROWS>
__device__ __forceinline__ void bwd_prefetch(Prefetch<Tin, ROWS>& pf, const BwdArgs& p, int64_t cb,
                                             int64_t ts, int64_t c, int row0) {
  const int tid = threadIdx.x;
  if (tid < 256) {
    const int u = tid >> 4, j = (tid & 15) * 4;
    const int64_t t = c * kChunk + u;
    const bool ok = t < p.g.T;
    const int64_t o = ok ? cb + t * ts + j : 0;
    const void* src[5] = {p.r, p.w, p.k, p.a, p.b};
#pragma unroll
    for (int n = 0; n < 5; ++n) pf.c[n] = load4<Tin>(src[n], o, ok);
  }
  if (tid < 4 * ROWS) {
    const int u2 = tid / (ROWS / 4), i4 = row0 + (tid % (ROWS / 4)) * 4;
    const int64_t t2 = c * kChunk + u2;
    const bool ok2 = t2 < p.g.T;
    const int64_t o2 = ok2 ? cb + t2 * ts + i4 : 0;
    pf.o[0] = load4<Tin>(p.v, o2, ok2);
    pf.o[1] = load4<Tin>(p.dy, o2, ok2);
    pf.o[2] = (p.dsa != nullptr) ? load4<float>(p.dsa, o2, ok2) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <typename Tin, int ROWS>
__device__ __forceinline__ void bwd_stage(BwdSmem<ROWS>& sm, const Prefetch<Tin, ROWS>& pf, int kind) {
  const int tid = threadIdx.x;
  if (tid < 256) {
    const int u = tid >> 4, j = (tid & 15) * 4;
    *reinterpret_cast<float4*>(&sm.r[u][j]) = pf.c[0];
    const float wi[4] = {pf.c[1].x, pf.c[1].y, pf.c[1].z, pf.c[1].w};
    float dl[4], wd[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lw = log_decay(wi[e], kind);
      dl[e] = dlog_decay(lw, kind);
      wd[e] = expf(lw);
    }
    *reinterpret_cast<float4*>(&sm.dlw[u][j]) = make_float4(dl[0], dl[1], dl[2], dl[3]);
    *reinterpret_cast<float4*>(&sm.w[u][j]) = make_float4(wd[0], wd[1], wd[2], wd[3]);
    *reinterpret_cast<float4*>(&sm.k[u][j]) = pf.c[2];
    *reinterpret_cast<float4*>(&sm.a[u][j]) = pf.c[3];
    *reinterpret_cast<float4*>(&sm.b[u][j]) = pf.c[4];
  }
  if (tid < 4 * ROWS) {
    const int u2 = tid / (ROWS / 4), il4 = (tid % (ROWS / 4)) * 4;
    *reinterpret_cast<float4*>(&sm.v[u2][il4]) = pf.o[0];
    *reinterpret_cast<float4*>(&sm.dy[u2][il4]) = pf.o[1];
    *reinterpret_cast<float4*>(&sm.dsa[u2][il4]) = pf.o[2];
  }
}

// one forward step of own row il (its kCols columns from q*kCols, register
// group g holding column group g ^ pm); returns sa of the row
template <int ROWS>
__device__ __forceinline__ float fwd_step(const BwdSmem<ROWS>& sm, int u, int il, int q, int pm, float2* S) {
  constexpr int kCols = BwdCfg<ROWS>::kCols, kG = Lanes<ROWS>::kG;
  const float4* a4 = reinterpret_cast<const float4*>(&sm.a[u][q * kCols]);
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    const float4 x = a4[g ^ pm];
    acc0 = __ffma2_rn(S[2 * g], lo2(x), acc0);
    acc1 = __ffma2_rn(S[2 * g + 1], hi2(x), acc1);
  }
  const float sa = row_sum<BwdCfg<ROWS>::kTpr>((acc0.x + acc0.y) + (acc1.x + acc1.y));
  const float2 sa2 = bc2(sa), vi2 = bc2(sm.v[u][il]);
  const float4* w4 = reinterpret_cast<const float4*>(&sm.w[u][q * kCols]);
  const float4* b4 = reinterpret_cast<const float4*>(&sm.b[u][q * kCols]);
  const float4* k4 = reinterpret_cast<const float4*>(&sm.k[u][q * kCols]);
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    const float4 wv = w4[g ^ pm], bv = b4[g ^ pm], kv = k4[g ^ pm];
    S[2 * g] = __ffma2_rn(S[2 * g], lo2(wv), __ffma2_rn(sa2, lo2(bv), __fmul2_rn(lo2(kv), vi2)));
    S[2 * g + 1] = __ffma2_rn(S[2 * g + 1], hi2(wv), __ffma2_rn(sa2, hi2(bv), __fmul2_rn(hi2(kv), vi2)));
  }
  return sa;
}

// A thread's state slot holds only its own registers, so its layout is free:
// float4 (row il, group g, thread q) at ((il kG + g) kTpr + q) ^ 4 (il & 1), which
// gives the eight lanes of a quarter warp (one row of 8 threads, or two rows of
// 4) eight different bank groups.
template <int ROWS>
__device__ __forceinline__ int slot4(int il, int g, int q) {
  return ((il * Lanes<ROWS>::kG + g) * BwdCfg<ROWS>::kTpr + q) ^ (4 * (il & 1));
}

template <int ROWS>
__device__ __forceinline__ void store_state(BwdSmem<ROWS>& sm, int slot, int il, int q, const float2* S) {
  float4* dst = reinterpret_cast<float4*>(&sm.S[slot][0][0]);
#pragma unroll
  for (int g = 0; g < Lanes<ROWS>::kG; ++g)
    dst[slot4<ROWS>(il, g, q)] = make_float4(S[2 * g].x, S[2 * g].y, S[2 * g + 1].x, S[2 * g + 1].y);
}

template <int ROWS>
__device__ __forceinline__ void load_state(const BwdSmem<ROWS>& sm, int slot, int il, int q, float2* S) {
  const float4* src = reinterpret_cast<const float4*>(&sm.S[slot][0][0]);
#pragma unroll
  for (int g = 0; g < Lanes<ROWS>::kG; ++g) {
    const float4 x = src[slot4<ROWS>(il, g, q)];
    S[2 * g] = lo2(x);
    S[2 * g + 1] = hi2(x);
  }
}

// one reverse step u of own row il, with the thread's columns of S_t in Sc and
// of S_{t-1} in Sp (register group g = column group g ^ pm); the own rows'
// column sums go to part[pb], threads below 160 writing two of them at d0, d1
template <int ROWS>
__device__ __forceinline__ void bwd_step(BwdSmem<ROWS>& sm, int u, const float2* Sc, const float2* Sp, int il,
                                         int q, int pm, int lane, int warp, int pb, int d0, int d1,
                                         float2* dS) {
  using Cfg = BwdCfg<ROWS>;
  using Ln = Lanes<ROWS>;
  constexpr int kCols = Cfg::kCols, kG = Ln::kG, kPairs = kCols / 2;
  const float2 dy2 = bc2(sm.dy[u][il]), vi2 = bc2(sm.v[u][il]), sa2 = bc2(sm.sa[u][il]);
  const float4* r4 = reinterpret_cast<const float4*>(&sm.r[u][q * kCols]);
  const float4* b4 = reinterpret_cast<const float4*>(&sm.b[u][q * kCols]);
  const float4* k4 = reinterpret_cast<const float4*>(&sm.k[u][q * kCols]);
  float2 dsa2 = make_float2(0.f, 0.f), dv2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    const float4 rv = r4[g ^ pm], bv = b4[g ^ pm], kv = k4[g ^ pm];
    dS[2 * g] = __ffma2_rn(dy2, lo2(rv), dS[2 * g]);
    dS[2 * g + 1] = __ffma2_rn(dy2, hi2(rv), dS[2 * g + 1]);
    dsa2 = __ffma2_rn(dS[2 * g], lo2(bv), dsa2);
    dv2 = __ffma2_rn(dS[2 * g], lo2(kv), dv2);
    dsa2 = __ffma2_rn(dS[2 * g + 1], hi2(bv), dsa2);
    dv2 = __ffma2_rn(dS[2 * g + 1], hi2(kv), dv2);
  }
  const float dsa = row_sum<Cfg::kTpr>(dsa2.x + dsa2.y) + sm.dsa[u][il];
  const float dv = row_sum<Cfg::kTpr>(dv2.x + dv2.y);
  const float2 dsab = bc2(dsa);

  // per column pair: dr, dw (before the decay's chain factor), dk, db, da
  float2 x[5][kPairs];
#pragma unroll
  for (int pp = 0; pp < kPairs; ++pp) {
    x[0][pp] = __fmul2_rn(Sc[pp], dy2);
    x[1][pp] = __fmul2_rn(dS[pp], Sp[pp]);
    x[2][pp] = __fmul2_rn(dS[pp], vi2);
    x[3][pp] = __fmul2_rn(dS[pp], sa2);
    x[4][pp] = __fmul2_rn(dsab, Sp[pp]);
  }
  const float4* w4 = reinterpret_cast<const float4*>(&sm.w[u][q * kCols]);
  const float4* a4 = reinterpret_cast<const float4*>(&sm.a[u][q * kCols]);
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    const float4 wv = w4[g ^ pm], av = a4[g ^ pm];
    dS[2 * g] = __ffma2_rn(dS[2 * g], lo2(wv), __fmul2_rn(dsab, lo2(av)));
    dS[2 * g + 1] = __ffma2_rn(dS[2 * g + 1], hi2(wv), __fmul2_rn(dsab, hi2(av)));
  }
  if (q == 0) sm.dv[u][il] = dv;

  // reduce-scatter over the rows of this warp: permuted levels, then one select level
#pragma unroll
  for (int lv = 0; lv < Ln::kP; ++lv) {
    const int bit = 16 >> lv, hp = 2 * (kG >> (lv + 1));  // pairs kept
#pragma unroll
    for (int n = 0; n < 5; ++n)
#pragma unroll
      for (int m = 0; m < hp; ++m) {
        const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, x[n][m + hp].x, bit),
                                     __shfl_xor_sync(0xffffffffu, x[n][m + hp].y, bit));
        x[n][m] = __fadd2_rn(x[n][m], o);
      }
  }
  // pairs 0..4 (values 0..9 of the lane's 5 x 4) stay on lanes without the
  // select bit, pairs 5..9 on lanes with it; pair m of a lane (its values 2m,
  // 2m + 1) lands at float2 m * 32 + lane of the warp's 160
  const bool hi = lane & Ln::kSelBit;
  float2* red = reinterpret_cast<float2*>(sm.red[Cfg::kRed == 2 ? (u & 1) : 0][warp]);
#pragma unroll
  for (int m = 0; m < 5; ++m) {
    const float2 lo_v = x[m >> 1][m & 1], hi_v = x[(m + 5) >> 1][(m + 5) & 1];
    const float2 send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
    const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, send.x, Ln::kSelBit),
                                 __shfl_xor_sync(0xffffffffu, send.y, Ln::kSelBit));
    red[m * 32 + lane] = __fadd2_rn(keep, o);
  }
  __syncthreads();
  // sums over the warps: threads 0..159 each add one float2 of every warp's 160
  if (threadIdx.x < 160) {
    const float2* rd = reinterpret_cast<const float2*>(sm.red[Cfg::kRed == 2 ? (u & 1) : 0][0]);
    float2 acc = rd[threadIdx.x];
#pragma unroll
    for (int wv = 1; wv < Cfg::kWarps; ++wv) acc = __fadd2_rn(acc, rd[wv * 160 + threadIdx.x]);
    float* part = &sm.part[pb][0][0][0] + u * kN;
    part[d0] = acc.x;
    part[d1] = acc.y;
  }
  if (Cfg::kRed == 1) __syncthreads();  // red is refilled by the next step
}

template <typename Tin, int ROWS>
__global__ void __cluster_dims__(BwdCfg<ROWS>::kCtas, 1, 1)
    __launch_bounds__(BwdCfg<ROWS>::kThreads, 1) scan_bwd_kernel(BwdArgs p) {
  using Cfg = BwdCfg<ROWS>;
  constexpr int kCols = Cfg::kCols;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem<ROWS>& sm = *reinterpret_cast<BwdSmem<ROWS>*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, il = tid / Cfg::kTpr, q = tid % Cfg::kTpr, lane = tid & 31, warp = tid >> 5;
  // this CTA's rows, and the columns whose outputs it writes
  const int rank = Cfg::kCtas > 1 ? static_cast<int>(cluster.block_rank()) : 0;
  const int64_t ch = blockIdx.x / Cfg::kCtas;
  const int row0 = rank * ROWS, i = row0 + il;
  const int64_t nchunk = p.g.nchunk;
  // the peer's partial sums, in its shared memory (a cluster of two)
  const BwdSmem<ROWS>* peer = Cfg::kCtas > 1 ? cluster.map_shared_rank(&sm, rank ^ 1) : nullptr;
  // register group g holds column group g ^ pm; threads below 160 add the
  // per-warp sums of pair tid / 32 of lane tid % 32 (values 2 (tid / 32) and
  // 2 (tid / 32) + 1 of that lane) and write them to d0, d1
  const int pm = Lanes<ROWS>::perm(lane);
  const int d0 = tid < 160 ? Lanes<ROWS>::part_off(64 * (tid >> 5) + (tid & 31)) : 0;
  const int d1 = tid < 160 ? Lanes<ROWS>::part_off(64 * (tid >> 5) + 32 + (tid & 31)) : 0;
  const int64_t cb = p.g.base(ch), ts = p.g.tstride();

  constexpr int kPairs = kCols / 2;
  float2 dS[kPairs], S0[kPairs], S[kPairs];
  if (p.dsT != nullptr) {  // the gradient of the final state enters at the last step
    const float4* src = reinterpret_cast<const float4*>(p.dsT + p.g.state_off(ch) + i * kN + q * kCols);
#pragma unroll
    for (int g = 0; g < kCols / 4; ++g) {
      const float4 x = src[g ^ pm];
      dS[2 * g] = lo2(x);
      dS[2 * g + 1] = hi2(x);
    }
  } else {
#pragma unroll
    for (int pp = 0; pp < kPairs; ++pp) dS[pp] = make_float2(0.f, 0.f);
  }

  Prefetch<Tin, ROWS> pf;
  if (nchunk > 0) bwd_prefetch<Tin, ROWS>(pf, p, cb, ts, nchunk - 1, row0);
  for (int64_t c = nchunk - 1; c >= 0; --c) {
    const int pb = Cfg::kParts > 1 ? static_cast<int>(c & 1) : 0;
    __syncthreads();
    bwd_stage<Tin, ROWS>(sm, pf, p.g.decay);
    if (c > 0) bwd_prefetch<Tin, ROWS>(pf, p, cb, ts, c - 1, row0);
    if (c > 0) {
      const float4* src = reinterpret_cast<const float4*>(p.ckpt + ((ch * nchunk + c) * kN + i) * kN + q * kCols);
#pragma unroll
      for (int g = 0; g < kCols / 4; ++g) {
        const float4 x = src[g ^ pm];
        S0[2 * g] = lo2(x);
        S0[2 * g + 1] = hi2(x);
      }
    } else if (p.s0 != nullptr) {  // chunk 0 starts from the state carried in
      const float4* src = reinterpret_cast<const float4*>(p.s0 + p.g.state_off(ch) + i * kN + q * kCols);
#pragma unroll
      for (int g = 0; g < kCols / 4; ++g) {
        const float4 x = src[g ^ pm];
        S0[2 * g] = lo2(x);
        S0[2 * g + 1] = hi2(x);
      }
    } else {
#pragma unroll
      for (int pp = 0; pp < kPairs; ++pp) S0[pp] = make_float2(0.f, 0.f);
    }
    __syncthreads();

    if constexpr (Cfg::kWhole) {
      // one forward pass keeps S_0..S_15 in shared memory and S_16 in registers;
      // the reverse walk hands each step's S_{t-1} on as the next step's S_t
#pragma unroll
      for (int pp = 0; pp < kPairs; ++pp) S[pp] = S0[pp];
      store_state(sm, 0, il, q, S);
#pragma unroll 1
      for (int u = 0; u < kChunk; ++u) {
        const float sa = fwd_step(sm, u, il, q, pm, S);
        if (q == 0) sm.sa[u][il] = sa;
        if (u + 1 < kChunk) store_state(sm, u + 1, il, q, S);
      }
      __syncthreads();
#pragma unroll 1
      for (int u = kChunk - 1; u >= 0; --u) {
        float2 Sp[kPairs];
        load_state(sm, u, il, q, Sp);
        bwd_step(sm, u, S, Sp, il, q, pm, lane, warp, pb, d0, d1, dS);
#pragma unroll
        for (int pp = 0; pp < kPairs; ++pp) S[pp] = Sp[pp];
      }
    } else {
      // second half: advance to the middle, keep states of steps kHalf..kChunk-1
      float2 Sc[kPairs], Sp[kPairs];
#pragma unroll
      for (int pp = 0; pp < kPairs; ++pp) S[pp] = S0[pp];
#pragma unroll 1
      for (int u = 0; u < kHalf; ++u) {
        const float sa = fwd_step(sm, u, il, q, pm, S);
        if (q == 0) sm.sa[u][il] = sa;
      }
      store_state(sm, 0, il, q, S);
#pragma unroll 1
      for (int u = kHalf; u < kChunk; ++u) {
        const float sa = fwd_step(sm, u, il, q, pm, S);
        if (q == 0) sm.sa[u][il] = sa;
        store_state(sm, u - kHalf + 1, il, q, S);
      }
      __syncthreads();
#pragma unroll 1
      for (int u = kChunk - 1; u >= kHalf; --u) {
        load_state(sm, u - kHalf + 1, il, q, Sc);
        load_state(sm, u - kHalf, il, q, Sp);
        bwd_step(sm, u, Sc, Sp, il, q, pm, lane, warp, pb, d0, d1, dS);
      }

      // first half
#pragma unroll
      for (int pp = 0; pp < kPairs; ++pp) S[pp] = S0[pp];
      store_state(sm, 0, il, q, S);
#pragma unroll 1
      for (int u = 0; u < kHalf; ++u) {
        fwd_step(sm, u, il, q, pm, S);
        store_state(sm, u + 1, il, q, S);
      }
      __syncthreads();
#pragma unroll 1
      for (int u = kHalf - 1; u >= 0; --u) {
        load_state(sm, u + 1, il, q, Sc);
        load_state(sm, u, il, q, Sp);
        bwd_step(sm, u, Sc, Sp, il, q, pm, lane, warp, pb, d0, d1, dS);
      }
    }

    // both CTAs' column sums of this chunk are complete (and visible across the
    // cluster; with one CTA per chain, across the CTA)
    if (Cfg::kCtas > 1) cluster.sync(); else __syncthreads();
    // this CTA writes the columns [ROWS rank, ROWS rank + ROWS): thread -> (tensor, step, 4 columns)
    for (int idx = tid; idx < 5 * kChunk * (ROWS / 4); idx += Cfg::kThreads) {
      const int tens = idx / (kChunk * (ROWS / 4)), rem = idx % (kChunk * (ROWS / 4));
      const int u = rem / (ROWS / 4), j = row0 + (rem % (ROWS / 4)) * 4;
      const int64_t t = c * kChunk + u;
      if (t >= p.g.T) continue;
      const float4 own = *reinterpret_cast<const float4*>(&sm.part[pb][tens][u][j]);
      float s[4] = {own.x, own.y, own.z, own.w};
      if (Cfg::kCtas > 1) {
        const float4 oth = *reinterpret_cast<const float4*>(&peer->part[pb][tens][u][j]);
        s[0] += oth.x; s[1] += oth.y; s[2] += oth.z; s[3] += oth.w;
      }
      if (tens == 1)  // dw_in = dL/dw * w * dlw/dw_in
#pragma unroll
        for (int e = 0; e < 4; ++e) s[e] *= sm.w[u][j + e] * sm.dlw[u][j + e];
      // part[] order: dr, dw, dk, db, da
      void* dst = tens == 0 ? p.dr : tens == 1 ? p.dw : tens == 2 ? p.dk : tens == 3 ? p.db : p.da;
      Tin* o = static_cast<Tin*>(dst) + cb + t * ts + j;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = from_f32<Tin>(s[e]);
    }
    if (tid < 4 * ROWS) {  // dv of the own rows: thread -> (step, 4 rows), 16 x ROWS / 4 of them
      const int u = tid / (ROWS / 4), j = (tid % (ROWS / 4)) * 4;
      const int64_t t = c * kChunk + u;
      if (t < p.g.T) {
        Tin* o = static_cast<Tin*>(p.dv) + cb + t * ts + row0 + j;
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = from_f32<Tin>(sm.dv[u][j + e]);
      }
    }
  }
  if (p.ds0 != nullptr) {  // after chunk 0, dS is the gradient of the start state
    float4* dst = reinterpret_cast<float4*>(p.ds0 + p.g.state_off(ch) + i * kN + q * kCols);
#pragma unroll
    for (int g = 0; g < kCols / 4; ++g)
      dst[g ^ pm] = make_float4(dS[2 * g].x, dS[2 * g].y, dS[2 * g + 1].x, dS[2 * g + 1].y);
  }
  // the peer may still be reading this CTA's partial sums of the last chunk
  if (Cfg::kCtas > 1) cluster.sync();
}

template <typename Tin>
cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream) {
  if (p.ckpt == nullptr && p.g.T <= kChunk) {  // a few steps without checkpoint: decode
    step_fwd_kernel<Tin><<<(unsigned)(p.g.chains() * kStepCtas), kStepThreads, 0, stream>>>(p);
    return cudaGetLastError();
  }
  const size_t smem = sizeof(FwdSmem<Tin>);
  cudaError_t e = cudaFuncSetAttribute(scan_fwd_kernel<Tin>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t blocks = p.g.chains() * kRowGroups;
  scan_fwd_kernel<Tin><<<(unsigned)blocks, kFwdThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename Tin, int ROWS>
cudaError_t launch_bwd_rows(const BwdArgs& p, cudaStream_t stream) {
  using Cfg = BwdCfg<ROWS>;
  const size_t smem = sizeof(BwdSmem<ROWS>);
  cudaError_t e = cudaFuncSetAttribute(scan_bwd_kernel<Tin, ROWS>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // Cfg::kCtas CTAs per chain, one cluster (the cluster shape is compiled in)
  scan_bwd_kernel<Tin, ROWS><<<(unsigned)(p.g.chains() * Cfg::kCtas), Cfg::kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

// Two 32-row CTAs per chain while they fit the SMs in one wave (a CTA holds
// an SM: 222 KB of shared memory), else one 64-row CTA per chain.
template <typename Tin>
cudaError_t launch_bwd(const BwdArgs& p, cudaStream_t stream) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return p.g.chains() * 2 <= sms ? launch_bwd_rows<Tin, 32>(p, stream)
                                 : launch_bwd_rows<Tin, 64>(p, stream);
}

template cudaError_t launch_fwd<float>(const FwdArgs&, cudaStream_t);
template cudaError_t launch_fwd<bf16>(const FwdArgs&, cudaStream_t);
template cudaError_t launch_bwd<float>(const BwdArgs&, cudaStream_t);
template cudaError_t launch_bwd<bf16>(const BwdArgs&, cudaStream_t);

}  // namespace scan
}  // namespace camoe
