// Per-step WKV-7 ClampW scan on CUDA cores, fp32 state and arithmetic: the
// fp32-exact path of the operator (any element type in, fp32 math).
//
// Forward (scan_fwd_kernel): the state rows are independent recurrences that
// share the transition, so a chain's 64 rows are split over 4 CTAs of 16
// rows; 4 threads own one row (16 state columns each in registers) and
// combine row sums (sa = S a, y = S r) with two xor-shuffles.  Chunks of 16
// steps of r, w, k, a, b (and the CTA's slice of v) are streamed into shared
// memory with cp.async, double-buffered, and converted once per chunk
// (decay w = exp(log_decay(w_in)) computed there, ClampW or wind).  The state at the
// start of every chunk is the checkpoint, stored row-major in fp32.
//
// Backward (scan_bwd_kernel): one CTA of 256 threads per chain (row i =
// tid/4, column quarter q = tid%4), walking chunks in reverse.  Each chunk's
// states are recomputed forward from its checkpoint into shared memory (two
// halves of 8 steps so 9 states fit), never reversed through 1/w as
// camoe/cuda/rwkv7_clampw.cu:133 does.  Per step the row sums (dsa = dS b,
// dv = dS k) use shuffles; the five column sums over the 64 rows (dr, dw, dk,
// db, da) use a shuffle reduce-scatter over the 8 rows of a warp and a
// shared-memory pass over the 8 warps.  The per-element formulas are those
// of camoe/cuda/rwkv7_clampw.cu:123-168, plus the external sa-gradient.
#include "wkv7_common.cuh"

namespace camoe {
namespace scan {

constexpr int kRows = 16;                 // forward: state rows per CTA
constexpr int kFwdThreads = kRows * 4;    // forward: 4 threads per row
constexpr int kRowGroups = kN / kRows;    // forward: CTAs per chain
constexpr int kBwdThreads = kN * 4;       // backward: whole chain per CTA
constexpr int kHalf = kChunk / 2;         // backward: states held per half chunk

template <typename Tin>
struct FwdSmem {
  Tin raw[2][5][kChunk][kN];       // r, w, k, a, b of one chunk, double-buffered
  Tin rawv[2][kChunk][kRows];      // this CTA's slice of v
  float r[kChunk][kN], w[kChunk][kN], k[kChunk][kN], a[kChunk][kN], b[kChunk][kN];
  float v[kChunk][kRows];
  float y[kChunk][kRows], sa[kChunk][kRows];
};

template <typename Tin>
__device__ __forceinline__ void fwd_issue(FwdSmem<Tin>& sm, int buf, const FwdArgs& p,
                                          int64_t ch, int64_t c, int rg) {
  constexpr int V = 16 / sizeof(Tin);  // elements per 16-byte copy
  constexpr int PR = kN / V;           // copies per 64-wide row
  constexpr int VR = kRows / V;        // copies per v slice row
  const int64_t t0 = c * kChunk;
  for (int idx = threadIdx.x; idx < 5 * kChunk * PR; idx += kFwdThreads) {
    const int tens = idx / (kChunk * PR), rem = idx % (kChunk * PR);
    const int u = rem / PR, part = rem % PR;
    const Tin* src = static_cast<const Tin*>(tens == 0 ? p.r : tens == 1 ? p.w : tens == 2 ? p.k
                                             : tens == 3 ? p.a : p.b);
    const bool ok = t0 + u < p.g.T;
    cp_async16(&sm.raw[buf][tens][u][part * V], src + (ok ? p.g.off(ch, t0 + u, part * V) : 0), ok);
  }
  for (int idx = threadIdx.x; idx < kChunk * VR; idx += kFwdThreads) {
    const int u = idx / VR, part = idx % VR;
    const bool ok = t0 + u < p.g.T;
    const Tin* src = static_cast<const Tin*>(p.v);
    cp_async16(&sm.rawv[buf][u][part * V],
               src + (ok ? p.g.off(ch, t0 + u, rg * kRows + part * V) : 0), ok);
  }
}

template <typename Tin>
__global__ void __launch_bounds__(kFwdThreads) scan_fwd_kernel(FwdArgs p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FwdSmem<Tin>& sm = *reinterpret_cast<FwdSmem<Tin>*>(smem_raw);
  const int tid = threadIdx.x, rl = tid >> 2, q = tid & 3;
  const int64_t ch = blockIdx.x / kRowGroups;
  const int rg = blockIdx.x % kRowGroups;
  const int i = rg * kRows + rl;
  const int64_t nchunk = p.g.nchunk;

  float S[16];
  if (p.s0 != nullptr) {  // start state: row i, columns 16q..16q+15
    const float4* src = reinterpret_cast<const float4*>(p.s0 + p.g.state_off(ch) + i * kN + q * 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float4 x = src[m];
      S[4 * m] = x.x; S[4 * m + 1] = x.y; S[4 * m + 2] = x.z; S[4 * m + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) S[jj] = 0.f;
  }

  fwd_issue(sm, 0, p, ch, 0, rg);
  cp_async_commit();
  for (int64_t c = 0; c < nchunk; ++c) {
    const int buf = c & 1;
    // steps of this chunk inside the sequence (the rest are never applied,
    // so the final state is the state after step T - 1)
    const int nu = p.g.T - c * kChunk < kChunk ? static_cast<int>(p.g.T - c * kChunk) : kChunk;
    if (c + 1 < nchunk) fwd_issue(sm, buf ^ 1, p, ch, c + 1, rg);
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
      float4* dst = reinterpret_cast<float4*>(p.ckpt + ((ch * nchunk + c) * kN + i) * kN + q * 16);
#pragma unroll
      for (int m = 0; m < 4; ++m) dst[m] = make_float4(S[4 * m], S[4 * m + 1], S[4 * m + 2], S[4 * m + 3]);
    }

#pragma unroll 1
    for (int u = 0; u < nu; ++u) {
      const float4* a4 = reinterpret_cast<const float4*>(&sm.a[u][q * 16]);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int m = 0; m < 4; m += 2) {
        const float4 x = a4[m], z = a4[m + 1];
        s0 += S[4 * m] * x.x + S[4 * m + 1] * x.y + S[4 * m + 2] * x.z + S[4 * m + 3] * x.w;
        s1 += S[4 * m + 4] * z.x + S[4 * m + 5] * z.y + S[4 * m + 6] * z.z + S[4 * m + 7] * z.w;
      }
      float sa = s0 + s1;
      sa += __shfl_xor_sync(0xffffffffu, sa, 1);
      sa += __shfl_xor_sync(0xffffffffu, sa, 2);
      const float vi = sm.v[u][rl];
      const float4* w4 = reinterpret_cast<const float4*>(&sm.w[u][q * 16]);
      const float4* b4 = reinterpret_cast<const float4*>(&sm.b[u][q * 16]);
      const float4* k4 = reinterpret_cast<const float4*>(&sm.k[u][q * 16]);
      const float4* r4 = reinterpret_cast<const float4*>(&sm.r[u][q * 16]);
      float y0 = 0.f, y1 = 0.f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float4 wv = w4[m], bv = b4[m], kv = k4[m], rv = r4[m];
        const float wa[4] = {wv.x, wv.y, wv.z, wv.w}, ba[4] = {bv.x, bv.y, bv.z, bv.w};
        const float ka[4] = {kv.x, kv.y, kv.z, kv.w}, ra[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float s = S[4 * m + e] * wa[e] + (sa * ba[e] + ka[e] * vi);
          S[4 * m + e] = s;
          if (e & 1) y1 += s * ra[e]; else y0 += s * ra[e];
        }
      }
      float y = y0 + y1;
      y += __shfl_xor_sync(0xffffffffu, y, 1);
      y += __shfl_xor_sync(0xffffffffu, y, 2);
      if (q == 0) {
        sm.y[u][rl] = y;
        sm.sa[u][rl] = sa;
      }
    }
    __syncthreads();
    // write y, sa of this chunk: thread -> (step u, 4 consecutive rows)
    {
      const int u = tid >> 2, part = tid & 3;
      const int64_t t = c * kChunk + u;
      if (t < p.g.T) {
        const int64_t o = p.g.off(ch, t, rg * kRows + part * 4);
        const float* ys = &sm.y[u][part * 4];
        Tin* yo = static_cast<Tin*>(p.y) + o;
#pragma unroll
        for (int e = 0; e < 4; ++e) yo[e] = from_f32<Tin>(ys[e]);
        *reinterpret_cast<float4*>(p.sa + o) = *reinterpret_cast<const float4*>(&sm.sa[u][part * 4]);
      }
    }
  }
  if (p.sT != nullptr) {
    float4* dst = reinterpret_cast<float4*>(p.sT + p.g.state_off(ch) + i * kN + q * 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) dst[m] = make_float4(S[4 * m], S[4 * m + 1], S[4 * m + 2], S[4 * m + 3]);
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

struct BwdSmem {
  float S[kHalf + 1][kN][kN];  // states of one half chunk, columns xor-swizzled by row
  float r[kChunk][kN], w[kChunk][kN], dlw[kChunk][kN], k[kChunk][kN], a[kChunk][kN],
      b[kChunk][kN], v[kChunk][kN], dy[kChunk][kN], dsa[kChunk][kN];
  float sa[kChunk][kN];
  float red[kBwdThreads / 32][320];  // per-warp partial column sums
  float out[6][kChunk][kN];          // dr, dw, dk, db, da, dv of the chunk
};

// physical column of element (i, j) in BwdSmem::S (keeps 4-column groups contiguous)
__device__ __forceinline__ int swz(int i, int j) { return j ^ ((i & 7) << 2); }

template <typename Tin>
struct Prefetch {  // one thread's share (4 consecutive columns of one step) of a chunk
  float4 x[8];     // r, w, k, v, a, b, dy, dsa
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

template <typename Tin>
__device__ __forceinline__ void bwd_prefetch(Prefetch<Tin>& pf, const BwdArgs& p, int64_t ch,
                                             int64_t c) {
  const int u = threadIdx.x >> 4, j = (threadIdx.x & 15) * 4;
  const int64_t t = c * kChunk + u;
  const bool ok = t < p.g.T;
  const int64_t o = ok ? p.g.off(ch, t, j) : 0;
  pf.x[0] = load4<Tin>(p.r, o, ok);
  pf.x[1] = load4<Tin>(p.w, o, ok);
  pf.x[2] = load4<Tin>(p.k, o, ok);
  pf.x[3] = load4<Tin>(p.v, o, ok);
  pf.x[4] = load4<Tin>(p.a, o, ok);
  pf.x[5] = load4<Tin>(p.b, o, ok);
  pf.x[6] = load4<Tin>(p.dy, o, ok);
  pf.x[7] = (p.dsa != nullptr) ? load4<float>(p.dsa, o, ok) : make_float4(0.f, 0.f, 0.f, 0.f);
}

template <typename Tin>
__device__ __forceinline__ void bwd_stage(BwdSmem& sm, const Prefetch<Tin>& pf, int kind) {
  const int u = threadIdx.x >> 4, j = (threadIdx.x & 15) * 4;
  *reinterpret_cast<float4*>(&sm.r[u][j]) = pf.x[0];
  const float wi[4] = {pf.x[1].x, pf.x[1].y, pf.x[1].z, pf.x[1].w};
  float dl[4], wd[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float lw = log_decay(wi[e], kind);
    dl[e] = dlog_decay(lw, kind);
    wd[e] = expf(lw);
  }
  *reinterpret_cast<float4*>(&sm.dlw[u][j]) = make_float4(dl[0], dl[1], dl[2], dl[3]);
  *reinterpret_cast<float4*>(&sm.w[u][j]) = make_float4(wd[0], wd[1], wd[2], wd[3]);
  *reinterpret_cast<float4*>(&sm.k[u][j]) = pf.x[2];
  *reinterpret_cast<float4*>(&sm.v[u][j]) = pf.x[3];
  *reinterpret_cast<float4*>(&sm.a[u][j]) = pf.x[4];
  *reinterpret_cast<float4*>(&sm.b[u][j]) = pf.x[5];
  *reinterpret_cast<float4*>(&sm.dy[u][j]) = pf.x[6];
  *reinterpret_cast<float4*>(&sm.dsa[u][j]) = pf.x[7];
}

// one forward step of row i (columns q*16..q*16+15); returns sa_i
__device__ __forceinline__ float fwd_step(const BwdSmem& sm, int u, int i, int q, float* S) {
  const float4* a4 = reinterpret_cast<const float4*>(&sm.a[u][q * 16]);
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int m = 0; m < 4; m += 2) {
    const float4 x = a4[m], z = a4[m + 1];
    s0 += S[4 * m] * x.x + S[4 * m + 1] * x.y + S[4 * m + 2] * x.z + S[4 * m + 3] * x.w;
    s1 += S[4 * m + 4] * z.x + S[4 * m + 5] * z.y + S[4 * m + 6] * z.z + S[4 * m + 7] * z.w;
  }
  float sa = s0 + s1;
  sa += __shfl_xor_sync(0xffffffffu, sa, 1);
  sa += __shfl_xor_sync(0xffffffffu, sa, 2);
  const float vi = sm.v[u][i];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float4 wv = reinterpret_cast<const float4*>(&sm.w[u][q * 16])[m];
    const float4 bv = reinterpret_cast<const float4*>(&sm.b[u][q * 16])[m];
    const float4 kv = reinterpret_cast<const float4*>(&sm.k[u][q * 16])[m];
    const float wa[4] = {wv.x, wv.y, wv.z, wv.w}, ba[4] = {bv.x, bv.y, bv.z, bv.w};
    const float ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) S[4 * m + e] = S[4 * m + e] * wa[e] + (sa * ba[e] + ka[e] * vi);
  }
  return sa;
}

__device__ __forceinline__ void store_state(BwdSmem& sm, int slot, int i, int q, const float* S) {
#pragma unroll
  for (int m = 0; m < 4; ++m)
    *reinterpret_cast<float4*>(&sm.S[slot][i][swz(i, q * 16 + 4 * m)]) =
        make_float4(S[4 * m], S[4 * m + 1], S[4 * m + 2], S[4 * m + 3]);
}

__device__ __forceinline__ void load_state(const BwdSmem& sm, int slot, int i, int q, float* S) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float4 x = *reinterpret_cast<const float4*>(&sm.S[slot][i][swz(i, q * 16 + 4 * m)]);
    S[4 * m] = x.x; S[4 * m + 1] = x.y; S[4 * m + 2] = x.z; S[4 * m + 3] = x.w;
  }
}

// one reverse step u with S_t in slot st and S_{t-1} in slot sp
__device__ __forceinline__ void bwd_step(BwdSmem& sm, int u, int st, int sp, int i, int q,
                                         int lane, int warp, float* dS) {
  float Sc[16], Sp[16];
  load_state(sm, st, i, q, Sc);
  load_state(sm, sp, i, q, Sp);
  const float dyi = sm.dy[u][i], vi = sm.v[u][i], sai = sm.sa[u][i];
  float dsa0 = 0.f, dsa1 = 0.f, dv0 = 0.f, dv1 = 0.f;
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const int j = q * 16 + jj;
    dS[jj] += dyi * sm.r[u][j];
    if (jj & 1) { dsa1 += dS[jj] * sm.b[u][j]; dv1 += dS[jj] * sm.k[u][j]; }
    else { dsa0 += dS[jj] * sm.b[u][j]; dv0 += dS[jj] * sm.k[u][j]; }
  }
  float dsa = dsa0 + dsa1, dv = dv0 + dv1;
  dsa += __shfl_xor_sync(0xffffffffu, dsa, 1);
  dv += __shfl_xor_sync(0xffffffffu, dv, 1);
  dsa += __shfl_xor_sync(0xffffffffu, dsa, 2);
  dv += __shfl_xor_sync(0xffffffffu, dv, 2);
  dsa += sm.dsa[u][i];

  float x[80];
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    x[jj] = Sc[jj] * dyi;       // dr
    x[16 + jj] = dS[jj] * Sp[jj];  // dw (before the sigmoid chain factor)
    x[32 + jj] = dS[jj] * vi;   // dk
    x[48 + jj] = dS[jj] * sai;  // db
    x[64 + jj] = dsa * Sp[jj];  // da
  }
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const int j = q * 16 + jj;
    dS[jj] = dS[jj] * sm.w[u][j] + dsa * sm.a[u][j];
  }
  if (q == 0) sm.out[5][u][i] = dv;

  // reduce-scatter the 80 partials over the 8 rows of this warp (lane bits 4,3,2)
  const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4;
#pragma unroll
  for (int m = 0; m < 40; ++m) {
    const float send = h4 ? x[m] : x[m + 40];
    const float keep = h4 ? x[m + 40] : x[m];
    x[m] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int m = 0; m < 20; ++m) {
    const float send = h3 ? x[m] : x[m + 20];
    const float keep = h3 ? x[m + 20] : x[m];
    x[m] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int m = 0; m < 10; ++m) {
    const float send = h2 ? x[m] : x[m + 10];
    const float keep = h2 ? x[m + 10] : x[m];
    x[m] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
#pragma unroll
  for (int s = 0; s < 10; ++s) sm.red[warp][lane * 10 + s] = x[s];
  __syncthreads();
  for (int pidx = threadIdx.x; pidx < 320; pidx += kBwdThreads) {
    float acc = 0.f;
#pragma unroll
    for (int wv = 0; wv < kBwdThreads / 32; ++wv) acc += sm.red[wv][pidx];
    const int ln = pidx / 10, s = pidx % 10, qq = ln & 3, rb = ln >> 2;
    const int m = 40 * ((rb >> 2) & 1) + 20 * ((rb >> 1) & 1) + 10 * (rb & 1) + s;
    const int quant = m >> 4, j = qq * 16 + (m & 15);
    if (quant == 1) acc = acc * sm.w[u][j] * sm.dlw[u][j];  // dw_in = dL/dw * w * dlw/dw_in
    sm.out[quant][u][j] = acc;
  }
  __syncthreads();
}

template <typename Tin>
__global__ void __launch_bounds__(kBwdThreads, 1) scan_bwd_kernel(BwdArgs p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>(smem_raw);
  const int tid = threadIdx.x, i = tid >> 2, q = tid & 3, lane = tid & 31, warp = tid >> 5;
  const int64_t ch = blockIdx.x;
  const int64_t nchunk = p.g.nchunk;

  float dS[16], S0[16], S[16];
  if (p.dsT != nullptr) {  // the gradient of the final state enters at the last step
    const float4* src = reinterpret_cast<const float4*>(p.dsT + p.g.state_off(ch) + i * kN + q * 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float4 x = src[m];
      dS[4 * m] = x.x; dS[4 * m + 1] = x.y; dS[4 * m + 2] = x.z; dS[4 * m + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) dS[jj] = 0.f;
  }

  Prefetch<Tin> pf;
  if (nchunk > 0) bwd_prefetch<Tin>(pf, p, ch, nchunk - 1);
  for (int64_t c = nchunk - 1; c >= 0; --c) {
    __syncthreads();
    bwd_stage<Tin>(sm, pf, p.g.decay);
    if (c > 0) bwd_prefetch<Tin>(pf, p, ch, c - 1);
    if (c > 0) {
      const float4* src = reinterpret_cast<const float4*>(p.ckpt + ((ch * nchunk + c) * kN + i) * kN + q * 16);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float4 x = src[m];
        S0[4 * m] = x.x; S0[4 * m + 1] = x.y; S0[4 * m + 2] = x.z; S0[4 * m + 3] = x.w;
      }
    } else if (p.s0 != nullptr) {  // chunk 0 starts from the state carried in
      const float4* src = reinterpret_cast<const float4*>(p.s0 + p.g.state_off(ch) + i * kN + q * 16);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float4 x = src[m];
        S0[4 * m] = x.x; S0[4 * m + 1] = x.y; S0[4 * m + 2] = x.z; S0[4 * m + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) S0[jj] = 0.f;
    }
    __syncthreads();

    // second half: advance to the middle, keep states of steps kHalf..kChunk-1
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) S[jj] = S0[jj];
#pragma unroll 1
    for (int u = 0; u < kHalf; ++u) {
      const float sa = fwd_step(sm, u, i, q, S);
      if (q == 0) sm.sa[u][i] = sa;
    }
    store_state(sm, 0, i, q, S);
#pragma unroll 1
    for (int u = kHalf; u < kChunk; ++u) {
      const float sa = fwd_step(sm, u, i, q, S);
      if (q == 0) sm.sa[u][i] = sa;
      store_state(sm, u - kHalf + 1, i, q, S);
    }
    __syncthreads();
#pragma unroll 1
    for (int u = kChunk - 1; u >= kHalf; --u) bwd_step(sm, u, u - kHalf + 1, u - kHalf, i, q, lane, warp, dS);

    // first half
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) S[jj] = S0[jj];
    store_state(sm, 0, i, q, S);
#pragma unroll 1
    for (int u = 0; u < kHalf; ++u) {
      fwd_step(sm, u, i, q, S);
      store_state(sm, u + 1, i, q, S);
    }
    __syncthreads();
#pragma unroll 1
    for (int u = kHalf - 1; u >= 0; --u) bwd_step(sm, u, u + 1, u, i, q, lane, warp, dS);

    // write the chunk's gradients: thread -> (tensor, step, 4 columns)
    for (int idx = tid; idx < 6 * kChunk * (kN / 4); idx += kBwdThreads) {
      const int tens = idx / (kChunk * (kN / 4)), rem = idx % (kChunk * (kN / 4));
      const int u = rem / (kN / 4), j = (rem % (kN / 4)) * 4;
      const int64_t t = c * kChunk + u;
      if (t >= p.g.T) continue;
      // out[] order: dr, dw, dk, db, da, dv
      void* dst = tens == 0 ? p.dr : tens == 1 ? p.dw : tens == 2 ? p.dk : tens == 3 ? p.db
                : tens == 4 ? p.da : p.dv;
      Tin* o = static_cast<Tin*>(dst) + p.g.off(ch, t, j);
      const float* s = &sm.out[tens][u][j];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = from_f32<Tin>(s[e]);
    }
  }
  if (p.ds0 != nullptr) {  // after chunk 0, dS is the gradient of the start state
    float4* dst = reinterpret_cast<float4*>(p.ds0 + p.g.state_off(ch) + i * kN + q * 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) dst[m] = make_float4(dS[4 * m], dS[4 * m + 1], dS[4 * m + 2], dS[4 * m + 3]);
  }
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

template <typename Tin>
cudaError_t launch_bwd(const BwdArgs& p, cudaStream_t stream) {
  const size_t smem = sizeof(BwdSmem);
  cudaError_t e = cudaFuncSetAttribute(scan_bwd_kernel<Tin>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  scan_bwd_kernel<Tin><<<(unsigned)p.g.chains(), kBwdThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

template cudaError_t launch_fwd<float>(const FwdArgs&, cudaStream_t);
template cudaError_t launch_fwd<bf16>(const FwdArgs&, cudaStream_t);
template cudaError_t launch_bwd<float>(const BwdArgs&, cudaStream_t);
template cudaError_t launch_bwd<bf16>(const BwdArgs&, cudaStream_t);

}  // namespace scan
}  // namespace camoe
