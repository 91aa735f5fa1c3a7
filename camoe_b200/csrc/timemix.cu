// Fused elementwise kernels of RWKV-7's time mix around the WKV-7 op
// (camoe/backbone.py:296-373), declared in include/camoe_timemix.h.
//
// Each kernel is one pass over HBM for what the reference runs as chains of
// eager PyTorch ops (each a separate read and write of [B, T, C] tensors).
// Layout: one CTA of C/2 threads owns whole rows (one time step of one
// sequence); thread i holds columns 2i and 2i+1 (bf16x2 / float2 accesses,
// each warp one coalesced 128-byte line per bf16 tensor), so warp w is head w
// and the per-head sums (key normalisation, GroupNorm, the bonus term) are
// warp shuffles; the LayerNorm over C adds one shared-memory step.  CTAs walk
// work items of kRows consecutive steps of one sequence (the token shift
// reads the previous step from registers).  Parameter gradients are summed
// over a CTA's rows in registers, written as one partial row per CTA and
// added by partial_reduce_kernel in a fixed order (deterministic).
// All arithmetic is fp32; activations are stored in bf16.
#include <initializer_list>

#include "camoe_timemix.h"
#include "wkv7_common.cuh"

namespace camoe {
void set_last_cuda_error(int e);  // wkv7_capi.cu: reported by camoe_wkv7_last_cuda_error()

namespace tm {

constexpr int kRows = 4;      // time steps per work item (small items balance the one wave)
constexpr int kMaxGrid = 1024;
constexpr int kMaxParams = 6;  // parameter vectors of the backward with the most (mix)

struct Shape {
  int64_t B, T, C;
  int64_t nblk;  // ceil(T / kRows)
  __host__ __device__ int64_t items() const { return B * nblk; }
};

__device__ __forceinline__ float2 ld2(const bf16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ void st2(bf16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
__device__ __forceinline__ void st2(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }
// torch.nn.functional.softplus with its default threshold 20
__device__ __forceinline__ float softplus(float z) { return z > 20.0f ? z : log1pf(expf(z)); }

// rows [t0, t1) of sequence b for work item `item`
__device__ __forceinline__ void item_rows(const Shape& S, int64_t item, int64_t& b, int64_t& t0,
                                          int64_t& t1) {
  b = item / S.nblk;
  t0 = (item - b * S.nblk) * kRows;
  t1 = t0 + kRows < S.T ? t0 + kRows : S.T;
}

// -------------------------------------------------------------------------
// Every kernel walks its item's rows U at a time: the loads of U rows are
// issued before any of them is used (U independent rows in flight per
// thread), then the rows are computed and stored.

// token shift and mixes (backbone.py:316-323):
//   xx = shift(x) - x;  x_m = x + xx * mix_m
struct Out6 {
  bf16* p[6];
};
struct In6 {
  const bf16* p[6];
};

template <typename Tx>
__global__ void __launch_bounds__(1024) mix_fwd_kernel(const Tx* __restrict__ x,
                                                       const float* __restrict__ mix, Out6 out,
                                                       Shape S) {
  constexpr int U = 2;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  float m0[6], m1[6];
#pragma unroll
  for (int m = 0; m < 6; ++m) {
    m0[m] = mix[m * C + c];
    m1[m] = mix[m * C + c + 1];
  }
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    float2 xp = t0 > 0 ? ld2(x + (b * S.T + t0 - 1) * C + c) : make_float2(0.f, 0.f);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 xc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) xc[u] = ld2(x + o0 + (u < nu ? u : nu - 1) * C);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float dx0 = xp.x - xc[u].x, dx1 = xp.y - xc[u].y;
        if (u < nu)
#pragma unroll
          for (int m = 0; m < 6; ++m)
            st2(out.p[m] + o0 + u * C, xc[u].x + dx0 * m0[m], xc[u].y + dx1 * m1[m]);
        xp = xc[u];
      }
    }
  }
}

// dx[t] = sum_m dx_m[t] (1 - mix_m) + sum_m dx_m[t+1] mix_m;  dmix_m = sum_t dx_m[t] xx[t]
// Rows are walked downwards (dx_m[t+1] is the previous row's).
template <typename Tx>
__global__ void __launch_bounds__(1024) mix_bwd_kernel(const Tx* __restrict__ x,
                                                       const float* __restrict__ mix, In6 dout,
                                                       Tx* __restrict__ dx,
                                                       float* __restrict__ part, Shape S) {
  constexpr int U = 2;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  float a0[6], a1[6];
#pragma unroll
  for (int m = 0; m < 6; ++m) a0[m] = a1[m] = 0.f;
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    float2 dn[6];  // dx_m of the step after the current one
#pragma unroll
    for (int m = 0; m < 6; ++m)
      dn[m] = t1 < S.T ? ld2(dout.p[m] + (b * S.T + t1) * C + c) : make_float2(0.f, 0.f);
    float2 xc = ld2(x + (b * S.T + t1 - 1) * C + c);
    for (int64_t tb = t1 - 1; tb >= t0; tb -= U) {   // rows tb, tb - 1, ...
      const int nu = tb - t0 + 1 < U ? static_cast<int>(tb - t0 + 1) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 d[U][6], xp[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int uu = u < nu ? u : nu - 1;  // rows past the item repeat its last one
#pragma unroll
        for (int m = 0; m < 6; ++m) d[u][m] = ld2(dout.p[m] + o0 - uu * C);
        xp[u] = tb - uu > 0 ? ld2(x + o0 - (uu + 1) * C) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float on = u < nu ? 1.f : 0.f;
        const float xx0 = (xp[u].x - xc.x) * on, xx1 = (xp[u].y - xc.y) * on;
        float g0 = 0.f, g1 = 0.f;
#pragma unroll
        for (int m = 0; m < 6; ++m) {
          const float mx0 = __ldg(mix + m * C + c), mx1 = __ldg(mix + m * C + c + 1);
          g0 += d[u][m].x * (1.f - mx0) + dn[m].x * mx0;
          g1 += d[u][m].y * (1.f - mx1) + dn[m].y * mx1;
          a0[m] += d[u][m].x * xx0;
          a1[m] += d[u][m].y * xx1;
          dn[m] = d[u][m];
        }
        if (u < nu) st2(dx + o0 - u * C, g0, g1);
        xc = xp[u];
      }
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 6 * C;
#pragma unroll
  for (int m = 0; m < 6; ++m) st2(pp + m * C + c, a0[m], a1[m]);
}

// -------------------------------------------------------------------------
// op inputs (backbone.py:326-343, 347)
struct PrepFwd {
  const bf16 *wl, *k, *v, *vl, *al, *vf;
  const float* par;  // [5][C]: w0, v0, a0, k_k, k_a
  bf16 *w, *ko, *vo, *a, *b;
};

__global__ void __launch_bounds__(1024) prep_fwd_kernel(PrepFwd p, Shape S) {
  constexpr int U = 2;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 w0 = ld2(p.par + c), v0 = ld2(p.par + C + c), a0 = ld2(p.par + 2 * C + c);
  const float2 kk_ = ld2(p.par + 3 * C + c), ka = ld2(p.par + 4 * C + c);
  const bool vres = p.vl != nullptr;
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 wl[U], k[U], v[U], al[U], vl[U], vf[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t o = o0 + (u < nu ? u : nu - 1) * C;  // rows past the item repeat its last one
        wl[u] = ld2(p.wl + o); k[u] = ld2(p.k + o); v[u] = ld2(p.v + o); al[u] = ld2(p.al + o);
        vl[u] = vres ? ld2(p.vl + o) : make_float2(0.f, 0.f);
        vf[u] = vres ? ld2(p.vf + o) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        {
          const int64_t o = o0 + u * C;
          float2 vv = v[u];
          if (vres) {
            vv.x += (vf[u].x - vv.x) * sigm(v0.x + vl[u].x);
            vv.y += (vf[u].y - vv.y) * sigm(v0.y + vl[u].y);
          }
          const float a_0 = sigm(a0.x + al[u].x), a_1 = sigm(a0.y + al[u].y);
          const float kr0 = k[u].x * kk_.x, kr1 = k[u].y * kk_.y;
          const float inv = 1.0f / fmaxf(sqrtf(warp_sum(kr0 * kr0 + kr1 * kr1)), 1e-12f);
          const float kn0 = kr0 * inv, kn1 = kr1 * inv;
          if (u >= nu) continue;
          st2(p.w + o, -softplus(-(w0.x + wl[u].x)) - 0.5f, -softplus(-(w0.y + wl[u].y)) - 0.5f);
          st2(p.ko + o, k[u].x * (1.f + (a_0 - 1.f) * ka.x), k[u].y * (1.f + (a_1 - 1.f) * ka.y));
          st2(p.vo + o, vv.x, vv.y);
          st2(p.a + o, -kn0, -kn1);
          st2(p.b + o, kn0 * a_0, kn1 * a_1);
        }
      }
    }
  }
}

struct PrepBwd {
  const bf16 *dr_op, *dr_epi, *dw_op, *dk_op, *dk_epi, *dv_op, *dv_epi, *da_op, *db_op, *dvf_out;
  const bf16 *wl, *k, *v, *vl, *al, *vf;
  const float* par;
  bf16 *dr, *dwl, *dk, *dv, *dvl, *dal, *dvf;
};

__global__ void __launch_bounds__(1024) prep_bwd_kernel(PrepBwd p, float* __restrict__ part, Shape S) {
  constexpr int U = 1;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 w0 = ld2(p.par + c), v0 = ld2(p.par + C + c), a0 = ld2(p.par + 2 * C + c);
  const float2 kk_ = ld2(p.par + 3 * C + c), ka = ld2(p.par + 4 * C + c);
  const bool vres = p.vl != nullptr;
  float acc[5][2] = {};  // w0, v0, a0, k_k, k_a
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 gr[U], gw[U], gk[U], gv[U], ga[U], gb[U], gf[U], wl[U], k[U], al[U], v[U], vl[U], vf[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        {
          const int64_t o = o0 + (u < nu ? u : nu - 1) * C;  // rows past the item repeat its last one
          const float2 r1 = ld2(p.dr_op + o), r2 = ld2(p.dr_epi + o);
          const float2 k1 = ld2(p.dk_op + o), k2 = ld2(p.dk_epi + o);
          const float2 v1 = ld2(p.dv_op + o), v2 = ld2(p.dv_epi + o);
          gr[u] = make_float2(r1.x + r2.x, r1.y + r2.y);
          gk[u] = make_float2(k1.x + k2.x, k1.y + k2.y);
          gv[u] = make_float2(v1.x + v2.x, v1.y + v2.y);
          gw[u] = ld2(p.dw_op + o); ga[u] = ld2(p.da_op + o); gb[u] = ld2(p.db_op + o);
          wl[u] = ld2(p.wl + o); k[u] = ld2(p.k + o); al[u] = ld2(p.al + o); v[u] = ld2(p.v + o);
          vl[u] = vres ? ld2(p.vl + o) : make_float2(0.f, 0.f);
          vf[u] = vres ? ld2(p.vf + o) : make_float2(0.f, 0.f);
          gf[u] = (!vres && p.dvf_out != nullptr) ? ld2(p.dvf_out + o) : make_float2(0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t o = o0 + u * C;
        const bool live = u < nu;
        const float on = live ? 1.f : 0.f;  // weight of this row in the parameter sums
        if (live) st2(p.dr + o, gr[u].x, gr[u].y);
        const float gkv[2] = {gk[u].x * on, gk[u].y * on}, gvv[2] = {gv[u].x * on, gv[u].y * on};
        const float kv[2] = {k[u].x, k[u].y}, kkv[2] = {kk_.x, kk_.y}, kav[2] = {ka.x, ka.y};
        // decay input: w = -softplus(-u) - 1/2, dw/du = sigmoid(-u) (1 above torch's threshold)
        float dwl[2];
        {
          const float uu[2] = {w0.x + wl[u].x, w0.y + wl[u].y}, g[2] = {gw[u].x * on, gw[u].y * on};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            dwl[e] = -uu[e] > 20.f ? g[e] : g[e] * sigm(-uu[e]);
            acc[0][e] += dwl[e];
          }
        }
        const float a[2] = {sigm(a0.x + al[u].x), sigm(a0.y + al[u].y)};
        const float kr[2] = {kv[0] * kkv[0], kv[1] * kkv[1]};
        const float nrm = sqrtf(warp_sum(kr[0] * kr[0] + kr[1] * kr[1]));
        const float den = fmaxf(nrm, 1e-12f);
        const float kn[2] = {kr[0] / den, kr[1] / den};
        const float gav[2] = {ga[u].x * on, ga[u].y * on}, gbv[2] = {gb[u].x * on, gb[u].y * on};
        float dkn[2], da[2], dk[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          dkn[e] = -gav[e] + gbv[e] * a[e];                    // a_op = -kk, b_op = kk a
          da[e] = gbv[e] * kn[e] + gkv[e] * kv[e] * kav[e];    // k' = k (1 + (a - 1) k_a)
          dk[e] = gkv[e] * (1.f + (a[e] - 1.f) * kav[e]);
          acc[4][e] += gkv[e] * kv[e] * (a[e] - 1.f);
        }
        // kk = kr / max(|kr|, eps): dkr = (dkk - kk <dkk, kk>) / |kr|
        const float dot = warp_sum(dkn[0] * kn[0] + dkn[1] * kn[1]);
        float dal[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float dkr = nrm > 1e-12f ? (dkn[e] - kn[e] * dot) / den : dkn[e] / den;
          dk[e] += dkr * kkv[e];
          acc[3][e] += dkr * kv[e];
          dal[e] = da[e] * a[e] * (1.f - a[e]);
          acc[2][e] += dal[e];
        }
        if (!live) continue;
        st2(p.dwl + o, dwl[0], dwl[1]);
        st2(p.dk + o, dk[0], dk[1]);
        st2(p.dal + o, dal[0], dal[1]);
        if (vres) {
          const float s0 = sigm(v0.x + vl[u].x), s1 = sigm(v0.y + vl[u].y);
          const float dvl0 = gvv[0] * (vf[u].x - v[u].x) * s0 * (1.f - s0);
          const float dvl1 = gvv[1] * (vf[u].y - v[u].y) * s1 * (1.f - s1);
          acc[1][0] += dvl0;
          acc[1][1] += dvl1;
          st2(p.dv + o, gvv[0] * (1.f - s0), gvv[1] * (1.f - s1));
          st2(p.dvf + o, gvv[0] * s0, gvv[1] * s1);
          st2(p.dvl + o, dvl0, dvl1);
        } else {  // layer 0: v_first = v
          st2(p.dv + o, gvv[0] + gf[u].x, gvv[1] + gf[u].y);
        }
      }
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 5 * C;
#pragma unroll
  for (int q = 0; q < 5; ++q) st2(pp + q * C + c, acc[q][0], acc[q][1]);
}

// -------------------------------------------------------------------------
// epilogue (backbone.py:359-367): GroupNorm per head (eps 64e-5), bonus, gate
struct Post {
  const bf16 *y, *r, *ko, *vo, *g;
  const float *rk, *gamma, *beta;
};

__global__ void __launch_bounds__(1024) post_fwd_kernel(Post p, bf16* __restrict__ z, Shape S) {
  constexpr int U = 4;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 gm = ld2(p.gamma + c), bt = ld2(p.beta + c), rk = ld2(p.rk + c);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 y[U], r[U], ko[U], vo[U], g[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t o = o0 + (u < nu ? u : nu - 1) * C;  // rows past the item repeat its last one
        y[u] = ld2(p.y + o); r[u] = ld2(p.r + o); ko[u] = ld2(p.ko + o); vo[u] = ld2(p.vo + o);
        g[u] = ld2(p.g + o);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        {
          const float mean = warp_sum(y[u].x + y[u].y) * (1.f / 64.f);
          const float d0 = y[u].x - mean, d1 = y[u].y - mean;
          const float rstd = rsqrtf(warp_sum(d0 * d0 + d1 * d1) * (1.f / 64.f) + 64e-5f);
          const float s = warp_sum(r[u].x * ko[u].x * rk.x + r[u].y * ko[u].y * rk.y);
          const float x0 = d0 * rstd * gm.x + bt.x + s * vo[u].x;
          const float x1 = d1 * rstd * gm.y + bt.y + s * vo[u].y;
          if (u < nu) st2(z + o0 + u * C, x0 * g[u].x, x1 * g[u].y);
        }
      }
    }
  }
}

struct PostBwd {
  const bf16* dz;
  bf16 *dy, *dr, *dk, *dv, *dg;
};

__global__ void __launch_bounds__(1024) post_bwd_kernel(Post p, PostBwd q, float* __restrict__ part,
                                                        Shape S) {
  constexpr int U = 2;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 gm = ld2(p.gamma + c), bt = ld2(p.beta + c), rk = ld2(p.rk + c);
  float acc[3][2] = {};  // gamma, beta, r_k
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 y[U], r[U], ko[U], vo[U], g[U], dz[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t o = o0 + (u < nu ? u : nu - 1) * C;  // rows past the item repeat its last one
        y[u] = ld2(p.y + o); r[u] = ld2(p.r + o); ko[u] = ld2(p.ko + o); vo[u] = ld2(p.vo + o);
        g[u] = ld2(p.g + o);
        dz[u] = ld2(q.dz + o);
        if (u >= nu) dz[u] = make_float2(0.f, 0.f);  // contributes nothing to the parameter sums
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t o = o0 + u * C;
        const bool live = u < nu;
        const float mean = warp_sum(y[u].x + y[u].y) * (1.f / 64.f);
        const float d0 = y[u].x - mean, d1 = y[u].y - mean;
        const float rstd = rsqrtf(warp_sum(d0 * d0 + d1 * d1) * (1.f / 64.f) + 64e-5f);
        const float s = warp_sum(r[u].x * ko[u].x * rk.x + r[u].y * ko[u].y * rk.y);
        const float yn0 = d0 * rstd, yn1 = d1 * rstd;
        const float xa0 = yn0 * gm.x + bt.x + s * vo[u].x, xa1 = yn1 * gm.y + bt.y + s * vo[u].y;
        const float dx0 = dz[u].x * g[u].x, dx1 = dz[u].y * g[u].y;  // d x_att
        if (live) st2(q.dg + o, dz[u].x * xa0, dz[u].y * xa1);
        acc[0][0] += dx0 * yn0;
        acc[0][1] += dx1 * yn1;
        acc[1][0] += dx0;
        acc[1][1] += dx1;
        const float dn0 = dx0 * gm.x, dn1 = dx1 * gm.y;  // d yn
        const float m1 = warp_sum(dn0 + dn1) * (1.f / 64.f);
        const float m2 = warp_sum(dn0 * yn0 + dn1 * yn1) * (1.f / 64.f);
        const float ds = warp_sum(dx0 * vo[u].x + dx1 * vo[u].y);
        if (live) {
          st2(q.dy + o, rstd * (dn0 - m1 - yn0 * m2), rstd * (dn1 - m1 - yn1 * m2));
          // bonus s v': dv' = dx s, ds = <dx, v'>, s = sum r k' r_k
          st2(q.dv + o, dx0 * s, dx1 * s);
          st2(q.dr + o, ds * ko[u].x * rk.x, ds * ko[u].y * rk.y);
          st2(q.dk + o, ds * r[u].x * rk.x, ds * r[u].y * rk.y);
        }
        acc[2][0] += ds * r[u].x * ko[u].x;
        acc[2][1] += ds * r[u].y * ko[u].y;
      }
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 3 * C;
#pragma unroll
  for (int k = 0; k < 3; ++k) st2(pp + k * C + c, acc[k][0], acc[k][1]);
}

// -------------------------------------------------------------------------
// state representation (backbone.py:348): LayerNorm over C, eps 1e-5.  The
// U rows of an iteration share each CTA-wide reduction (one barrier for all).
template <int U>
__device__ __forceinline__ void block_sum_rows(float (&v)[U][2], float (*red)[32][U][2], int& buf) {
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    v[u][0] = warp_sum(v[u][0]);
    v[u][1] = warp_sum(v[u][1]);
  }
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      red[buf][warp][u][0] = v[u][0];
      red[buf][warp][u][1] = v[u][1];
    }
  __syncthreads();
  // lane l takes warp l's partials (nw <= 32), then one more warp sum
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const float2 x = lane < nw ? *reinterpret_cast<const float2*>(&red[buf][lane][u][0])
                               : make_float2(0.f, 0.f);
    v[u][0] = warp_sum(x.x);
    v[u][1] = warp_sum(x.y);
  }
  buf ^= 1;
}

__global__ void __launch_bounds__(1024) lnsa_fwd_kernel(const float* __restrict__ sa,
                                                        const float* __restrict__ wt,
                                                        const float* __restrict__ bs,
                                                        float* __restrict__ out, Shape S) {
  constexpr int U = 4;
  __shared__ __align__(8) float red[2][32][U][2];
  int buf = 0;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float invC = 1.0f / static_cast<float>(C);
  const float2 w = ld2(wt + c), bb = ld2(bs + c);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 x[U];
      float s[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        x[u] = u < nu ? ld2(sa + o0 + u * C) : make_float2(0.f, 0.f);
        s[u][0] = x[u].x + x[u].y;
        s[u][1] = 0.f;
      }
      block_sum_rows<U>(s, red, buf);  // mean, then the variance about it (two passes)
      float d[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float mean = s[u][0] * invC;
        d[u][0] = x[u].x - mean;
        d[u][1] = x[u].y - mean;
        s[u][0] = d[u][0] * d[u][0] + d[u][1] * d[u][1];
        s[u][1] = 0.f;
      }
      block_sum_rows<U>(s, red, buf);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (u < nu) {
          const float rstd = rsqrtf(s[u][0] * invC + 1e-5f);
          st2(out + o0 + u * C, d[u][0] * rstd * w.x + bb.x, d[u][1] * rstd * w.y + bb.y);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(1024) lnsa_bwd_kernel(const float* __restrict__ dout,
                                                        const float* __restrict__ sa,
                                                        const float* __restrict__ wt,
                                                        float* __restrict__ dsa,
                                                        float* __restrict__ part, Shape S) {
  constexpr int U = 4;
  __shared__ __align__(8) float red[2][32][U][2];
  int buf = 0;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float invC = 1.0f / static_cast<float>(C);
  const float2 w = ld2(wt + c);
  float acc[2][2] = {};  // weight, bias
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      const int nu = t1 - tb < U ? static_cast<int>(t1 - tb) : U;
      const int64_t o0 = (b * S.T + tb) * C + c;
      float2 x[U], g[U];
      float s[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        x[u] = u < nu ? ld2(sa + o0 + u * C) : make_float2(0.f, 0.f);
        g[u] = u < nu ? ld2(dout + o0 + u * C) : make_float2(0.f, 0.f);
        s[u][0] = x[u].x + x[u].y;
        s[u][1] = 0.f;
      }
      block_sum_rows<U>(s, red, buf);  // mean
      float d[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float mean = s[u][0] * invC;
        d[u][0] = x[u].x - mean;
        d[u][1] = x[u].y - mean;
        s[u][0] = d[u][0] * d[u][0] + d[u][1] * d[u][1];
        s[u][1] = 0.f;
      }
      block_sum_rows<U>(s, red, buf);  // variance
      float xn[U][2], dn[U][2], rstd[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        rstd[u] = rsqrtf(s[u][0] * invC + 1e-5f);
        xn[u][0] = d[u][0] * rstd[u];
        xn[u][1] = d[u][1] * rstd[u];
        dn[u][0] = g[u].x * w.x;
        dn[u][1] = g[u].y * w.y;
        acc[0][0] += g[u].x * xn[u][0];   // rows past nu have g = 0
        acc[0][1] += g[u].y * xn[u][1];
        acc[1][0] += g[u].x;
        acc[1][1] += g[u].y;
        s[u][0] = dn[u][0] + dn[u][1];
        s[u][1] = dn[u][0] * xn[u][0] + dn[u][1] * xn[u][1];
      }
      block_sum_rows<U>(s, red, buf);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (u < nu) {
          const float m1 = s[u][0] * invC, m2 = s[u][1] * invC;
          st2(dsa + o0 + u * C, rstd[u] * (dn[u][0] - m1 - xn[u][0] * m2),
              rstd[u] * (dn[u][1] - m1 - xn[u][1] * m2));
        }
      }
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 2 * C;
  st2(pp + c, acc[0][0], acc[0][1]);
  st2(pp + C + c, acc[1][0], acc[1][1]);
}

// out[i] = sum over g < G of part[g * n + i].  Block (32, 8): 32 consecutive
// columns, 8 row strides; each thread sums g = ty, ty + 8, ..., then the 8
// partial sums are added in order of ty (deterministic).
__global__ void __launch_bounds__(256) partial_reduce_kernel(const float* __restrict__ part, int G,
                                                             int64_t n, float* __restrict__ out) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t i = blockIdx.x * 32LL + tx;
  float s = 0.f;
  if (i < n)
    for (int g = ty; g < G; g += 8) s += part[g * n + i];
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && i < n) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][tx];
    out[i] = t;
  }
}

// ---------------------------------------------------------------------------
// host side

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int64_t B, int64_t T, int64_t C) {
  if (B < 0 || T < 0) return 1;              // CAMOE_ERR_INVALID_ARG
  if (C < 64 || C > 2048 || C % 64 != 0) return 2;  // CAMOE_ERR_UNSUPPORTED
  return 0;
}

// CTAs to launch: as many as fit on the device at once (CTAs of C/2 threads),
// at most one per work item and kMaxGrid
template <typename K>
int grid_for(K kernel, const Shape& S) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, static_cast<int>(S.C / 2), 0) !=
          cudaSuccess || per_sm < 1)
    per_sm = 1;
  int64_t g = static_cast<int64_t>(sms) * per_sm;
  if (g > kMaxGrid) g = kMaxGrid;
  if (g > S.items()) g = S.items();
  return static_cast<int>(g < 1 ? 1 : g);
}

size_t work_bytes(const Shape& S) {
  const int64_t g = S.items() < kMaxGrid ? S.items() : kMaxGrid;
  return static_cast<size_t>(g < 1 ? 1 : g) * kMaxParams * S.C * sizeof(float);
}

int status(cudaError_t e) {
  if (e == cudaSuccess) return 0;
  set_last_cuda_error(static_cast<int>(e));
  return 6;  // CAMOE_ERR_CUDA
}

int reduce(const float* part, int G, int64_t n, float* out, cudaStream_t st) {
  const int64_t blocks = (n + 31) / 32;
  partial_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(part, G, n, out);
  return status(cudaGetLastError());
}

}  // namespace tm
}  // namespace camoe

using camoe::bf16;
using camoe::tm::Shape;

namespace {

Shape make_shape(int64_t B, int64_t T, int64_t C) {
  return Shape{B, T, C, (T + camoe::tm::kRows - 1) / camoe::tm::kRows};
}

bool all_aligned(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p != nullptr && !camoe::tm::aligned16(p)) return false;
  return true;
}

bool any_null(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p == nullptr) return true;
  return false;
}

// common argument checks; 0 = go on, -1 = nothing to do, else a status code
int precheck(int64_t B, int64_t T, int64_t C, std::initializer_list<const void*> required,
             std::initializer_list<const void*> optional) {
  const int st = camoe::tm::check_shape(B, T, C);
  if (st != 0) return st;
  if (B == 0 || T == 0) return -1;
  if (any_null(required)) return 1;
  if (!all_aligned(required) || !all_aligned(optional)) return 4;  // CAMOE_ERR_ALIGNMENT
  return 0;
}

int check_work(const Shape& S, const void* work, size_t work_bytes) {
  if (work == nullptr) return 1;
  if (!camoe::tm::aligned16(work)) return 4;
  if (work_bytes < camoe::tm::work_bytes(S)) return 5;  // CAMOE_ERR_WORKSPACE
  return 0;
}

}  // namespace

extern "C" {

size_t camoe_tm_work_bytes(int64_t B, int64_t T, int64_t C) {
  if (camoe::tm::check_shape(B, T, C) != 0) return 0;
  return camoe::tm::work_bytes(make_shape(B, T, C));
}

int camoe_tm_mix_fwd(const void* x, int x_dtype, const float* mix, void* const* out, int64_t B,
                     int64_t T, int64_t C, void* stream) {
  if (out == nullptr) return 1;
  int st = precheck(B, T, C, {x, mix, out[0], out[1], out[2], out[3], out[4], out[5]}, {});
  if (st != 0) return st < 0 ? 0 : st;
  if (x_dtype != 0 && x_dtype != 1) return 2;
  const Shape S = make_shape(B, T, C);
  camoe::tm::Out6 o;
  for (int m = 0; m < 6; ++m) o.p[m] = static_cast<bf16*>(out[m]);
  const int G = x_dtype == 0 ? camoe::tm::grid_for(camoe::tm::mix_fwd_kernel<bf16>, S)
                             : camoe::tm::grid_for(camoe::tm::mix_fwd_kernel<float>, S);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == 0)
    camoe::tm::mix_fwd_kernel<bf16><<<G, static_cast<unsigned>(C / 2), 0, s>>>(static_cast<const bf16*>(x), mix, o, S);
  else
    camoe::tm::mix_fwd_kernel<float><<<G, static_cast<unsigned>(C / 2), 0, s>>>(static_cast<const float*>(x), mix, o, S);
  return camoe::tm::status(cudaGetLastError());
}

int camoe_tm_mix_bwd(const void* x, int x_dtype, const float* mix, const void* const* dout,
                     void* dx, float* dmix, void* work, size_t work_bytes, int64_t B, int64_t T,
                     int64_t C, void* stream) {
  if (dout == nullptr) return 1;
  int st = precheck(B, T, C, {x, mix, dx, dmix, dout[0], dout[1], dout[2], dout[3], dout[4], dout[5]}, {});
  if (st != 0) {
    if (st > 0) return st;
    if (dmix != nullptr && C >= 64) cudaMemsetAsync(dmix, 0, 6 * C * sizeof(float), static_cast<cudaStream_t>(stream));
    return 0;
  }
  if (x_dtype != 0 && x_dtype != 1) return 2;
  const Shape S = make_shape(B, T, C);
  if ((st = check_work(S, work, work_bytes)) != 0) return st;
  camoe::tm::In6 d;
  for (int m = 0; m < 6; ++m) d.p[m] = static_cast<const bf16*>(dout[m]);
  const int G = x_dtype == 0 ? camoe::tm::grid_for(camoe::tm::mix_bwd_kernel<bf16>, S)
                             : camoe::tm::grid_for(camoe::tm::mix_bwd_kernel<float>, S);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == 0)
    camoe::tm::mix_bwd_kernel<bf16><<<G, static_cast<unsigned>(C / 2), 0, s>>>(
        static_cast<const bf16*>(x), mix, d, static_cast<bf16*>(dx), part, S);
  else
    camoe::tm::mix_bwd_kernel<float><<<G, static_cast<unsigned>(C / 2), 0, s>>>(
        static_cast<const float*>(x), mix, d, static_cast<float*>(dx), part, S);
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 6 * C, dmix, s);
}

int camoe_tm_prep_fwd(const void* wl, const void* k, const void* v, const void* vl,
                      const void* al, const void* v_first, const float* params, void* w_op,
                      void* k_op, void* v_op, void* a_op, void* b_op, int64_t B, int64_t T,
                      int64_t C, void* stream) {
  if ((vl == nullptr) != (v_first == nullptr)) return 1;
  int st = precheck(B, T, C, {wl, k, v, al, params, w_op, k_op, v_op, a_op, b_op}, {vl, v_first});
  if (st != 0) return st < 0 ? 0 : st;
  const Shape S = make_shape(B, T, C);
  camoe::tm::PrepFwd p;
  p.wl = static_cast<const bf16*>(wl); p.k = static_cast<const bf16*>(k);
  p.v = static_cast<const bf16*>(v); p.vl = static_cast<const bf16*>(vl);
  p.al = static_cast<const bf16*>(al); p.vf = static_cast<const bf16*>(v_first);
  p.par = params;
  p.w = static_cast<bf16*>(w_op); p.ko = static_cast<bf16*>(k_op); p.vo = static_cast<bf16*>(v_op);
  p.a = static_cast<bf16*>(a_op); p.b = static_cast<bf16*>(b_op);
  camoe::tm::prep_fwd_kernel<<<camoe::tm::grid_for(camoe::tm::prep_fwd_kernel, S), static_cast<unsigned>(C / 2), 0,
                               static_cast<cudaStream_t>(stream)>>>(p, S);
  return camoe::tm::status(cudaGetLastError());
}

int camoe_tm_prep_bwd(const void* dr_op, const void* dr_epi, const void* dw_op,
                      const void* dk_op, const void* dk_epi, const void* dv_op,
                      const void* dv_epi, const void* da_op, const void* db_op,
                      const void* dv_first_out, const void* wl, const void* k, const void* v,
                      const void* vl, const void* al, const void* v_first, const float* params,
                      void* dr, void* dwl, void* dk, void* dv, void* dvl, void* dal,
                      void* dv_first, float* dparams, void* work, size_t work_bytes, int64_t B,
                      int64_t T, int64_t C, void* stream) {
  const bool vres = vl != nullptr;
  if (vres != (v_first != nullptr) || vres != (dvl != nullptr) || vres != (dv_first != nullptr))
    return 1;
  if (vres && dv_first_out != nullptr) return 1;  // v_first is an input there, not an output
  int st = precheck(B, T, C,
                    {dr_op, dr_epi, dw_op, dk_op, dk_epi, dv_op, dv_epi, da_op, db_op, wl, k, v, al,
                     params, dr, dwl, dk, dv, dal, dparams},
                    {dv_first_out, vl, v_first, dvl, dv_first});
  if (st != 0) {
    if (st > 0) return st;
    if (dparams != nullptr && C >= 64) cudaMemsetAsync(dparams, 0, 5 * C * sizeof(float), static_cast<cudaStream_t>(stream));
    return 0;
  }
  const Shape S = make_shape(B, T, C);
  if ((st = check_work(S, work, work_bytes)) != 0) return st;
  camoe::tm::PrepBwd p;
  p.dr_op = static_cast<const bf16*>(dr_op); p.dr_epi = static_cast<const bf16*>(dr_epi);
  p.dw_op = static_cast<const bf16*>(dw_op); p.dk_op = static_cast<const bf16*>(dk_op);
  p.dk_epi = static_cast<const bf16*>(dk_epi); p.dv_op = static_cast<const bf16*>(dv_op);
  p.dv_epi = static_cast<const bf16*>(dv_epi); p.da_op = static_cast<const bf16*>(da_op);
  p.db_op = static_cast<const bf16*>(db_op); p.dvf_out = static_cast<const bf16*>(dv_first_out);
  p.wl = static_cast<const bf16*>(wl); p.k = static_cast<const bf16*>(k);
  p.v = static_cast<const bf16*>(v); p.vl = static_cast<const bf16*>(vl);
  p.al = static_cast<const bf16*>(al); p.vf = static_cast<const bf16*>(v_first);
  p.par = params;
  p.dr = static_cast<bf16*>(dr); p.dwl = static_cast<bf16*>(dwl); p.dk = static_cast<bf16*>(dk);
  p.dv = static_cast<bf16*>(dv); p.dvl = static_cast<bf16*>(dvl); p.dal = static_cast<bf16*>(dal);
  p.dvf = static_cast<bf16*>(dv_first);
  const int G = camoe::tm::grid_for(camoe::tm::prep_bwd_kernel, S);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  camoe::tm::prep_bwd_kernel<<<G, static_cast<unsigned>(C / 2), 0, s>>>(p, part, S);
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 5 * C, dparams, s);
}

int camoe_tm_post_fwd(const void* y, const void* r, const void* k_op, const void* v_op,
                      const void* g, const float* r_k, const float* gamma, const float* beta,
                      void* z, int64_t B, int64_t T, int64_t C, void* stream) {
  int st = precheck(B, T, C, {y, r, k_op, v_op, g, r_k, gamma, beta, z}, {});
  if (st != 0) return st < 0 ? 0 : st;
  const Shape S = make_shape(B, T, C);
  camoe::tm::Post p{static_cast<const bf16*>(y), static_cast<const bf16*>(r),
                    static_cast<const bf16*>(k_op), static_cast<const bf16*>(v_op),
                    static_cast<const bf16*>(g), r_k, gamma, beta};
  camoe::tm::post_fwd_kernel<<<camoe::tm::grid_for(camoe::tm::post_fwd_kernel, S), static_cast<unsigned>(C / 2), 0,
                               static_cast<cudaStream_t>(stream)>>>(p, static_cast<bf16*>(z), S);
  return camoe::tm::status(cudaGetLastError());
}

int camoe_tm_post_bwd(const void* dz, const void* y, const void* r, const void* k_op,
                      const void* v_op, const void* g, const float* r_k, const float* gamma,
                      const float* beta, void* dy, void* dr_epi, void* dk_epi, void* dv_epi,
                      void* dg, float* dparams, void* work, size_t work_bytes, int64_t B,
                      int64_t T, int64_t C, void* stream) {
  int st = precheck(B, T, C, {dz, y, r, k_op, v_op, g, r_k, gamma, beta, dy, dr_epi, dk_epi,
                              dv_epi, dg, dparams}, {});
  if (st != 0) {
    if (st > 0) return st;
    if (dparams != nullptr && C >= 64) cudaMemsetAsync(dparams, 0, 3 * C * sizeof(float), static_cast<cudaStream_t>(stream));
    return 0;
  }
  const Shape S = make_shape(B, T, C);
  if ((st = check_work(S, work, work_bytes)) != 0) return st;
  camoe::tm::Post p{static_cast<const bf16*>(y), static_cast<const bf16*>(r),
                    static_cast<const bf16*>(k_op), static_cast<const bf16*>(v_op),
                    static_cast<const bf16*>(g), r_k, gamma, beta};
  camoe::tm::PostBwd q{static_cast<const bf16*>(dz), static_cast<bf16*>(dy),
                       static_cast<bf16*>(dr_epi), static_cast<bf16*>(dk_epi),
                       static_cast<bf16*>(dv_epi), static_cast<bf16*>(dg)};
  const int G = camoe::tm::grid_for(camoe::tm::post_bwd_kernel, S);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  camoe::tm::post_bwd_kernel<<<G, static_cast<unsigned>(C / 2), 0, s>>>(p, q, part, S);
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 3 * C, dparams, s);
}

int camoe_tm_lnsa_fwd(const float* sa, const float* weight, const float* bias, float* out,
                      int64_t B, int64_t T, int64_t C, void* stream) {
  int st = precheck(B, T, C, {sa, weight, bias, out}, {});
  if (st != 0) return st < 0 ? 0 : st;
  const Shape S = make_shape(B, T, C);
  camoe::tm::lnsa_fwd_kernel<<<camoe::tm::grid_for(camoe::tm::lnsa_fwd_kernel, S), static_cast<unsigned>(C / 2), 0,
                               static_cast<cudaStream_t>(stream)>>>(sa, weight, bias, out, S);
  return camoe::tm::status(cudaGetLastError());
}

int camoe_tm_lnsa_bwd(const float* dout, const float* sa, const float* weight, float* dsa,
                      float* dparams, void* work, size_t work_bytes, int64_t B, int64_t T,
                      int64_t C, void* stream) {
  int st = precheck(B, T, C, {dout, sa, weight, dsa, dparams}, {});
  if (st != 0) {
    if (st > 0) return st;
    if (dparams != nullptr && C >= 64) cudaMemsetAsync(dparams, 0, 2 * C * sizeof(float), static_cast<cudaStream_t>(stream));
    return 0;
  }
  const Shape S = make_shape(B, T, C);
  if ((st = check_work(S, work, work_bytes)) != 0) return st;
  const int G = camoe::tm::grid_for(camoe::tm::lnsa_bwd_kernel, S);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  camoe::tm::lnsa_bwd_kernel<<<G, static_cast<unsigned>(C / 2), 0, s>>>(dout, sa, weight, dsa, part, S);
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 2 * C, dparams, s);
}

}  // extern "C"
