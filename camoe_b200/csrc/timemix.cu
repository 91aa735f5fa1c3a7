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

constexpr int kRows = 16;     // time steps per work item
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

// sum over the CTA (all threads get it); `buf` alternates between calls so
// one barrier per call suffices (see lnsa kernels)
__device__ __forceinline__ float2 block_sum2(float2 v, float2 (*red)[32], int& buf) {
  v.x = warp_sum(v.x);
  v.y = warp_sum(v.y);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[buf][warp] = v;
  __syncthreads();
  float2 s = make_float2(0.f, 0.f);
  for (int w = 0; w < nw; ++w) {
    s.x += red[buf][w].x;
    s.y += red[buf][w].y;
  }
  buf ^= 1;
  return s;
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
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 xc = ld2(x + o);
      const float dx0 = xp.x - xc.x, dx1 = xp.y - xc.y;
#pragma unroll
      for (int m = 0; m < 6; ++m) st2(out.p[m] + o, xc.x + dx0 * m0[m], xc.y + dx1 * m1[m]);
      xp = xc;
    }
  }
}

// dx[t] = sum_m dx_m[t] (1 - mix_m) + sum_m dx_m[t+1] mix_m;  dmix_m = sum_t dx_m[t] xx[t]
template <typename Tx>
__global__ void __launch_bounds__(1024) mix_bwd_kernel(const Tx* __restrict__ x,
                                                       const float* __restrict__ mix, In6 dout,
                                                       Tx* __restrict__ dx,
                                                       float* __restrict__ part, Shape S) {
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  float m0[6], m1[6], a0[6], a1[6];
#pragma unroll
  for (int m = 0; m < 6; ++m) {
    m0[m] = mix[m * C + c];
    m1[m] = mix[m * C + c + 1];
    a0[m] = a1[m] = 0.f;
  }
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    float2 dn[6];  // dx_m of the step after the current one
#pragma unroll
    for (int m = 0; m < 6; ++m)
      dn[m] = t1 < S.T ? ld2(dout.p[m] + (b * S.T + t1) * C + c) : make_float2(0.f, 0.f);
    float2 xc = ld2(x + (b * S.T + t1 - 1) * C + c);
    for (int64_t t = t1 - 1; t >= t0; --t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 xp = t > 0 ? ld2(x + o - C) : make_float2(0.f, 0.f);
      const float xx0 = xp.x - xc.x, xx1 = xp.y - xc.y;
      float g0 = 0.f, g1 = 0.f;
#pragma unroll
      for (int m = 0; m < 6; ++m) {
        const float2 d = ld2(dout.p[m] + o);
        g0 += d.x * (1.f - m0[m]) + dn[m].x * m0[m];
        g1 += d.y * (1.f - m1[m]) + dn[m].y * m1[m];
        a0[m] += d.x * xx0;
        a1[m] += d.y * xx1;
        dn[m] = d;
      }
      st2(dx + o, g0, g1);
      xc = xp;
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
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 w0 = ld2(p.par + c), v0 = ld2(p.par + C + c), a0 = ld2(p.par + 2 * C + c);
  const float2 kk_ = ld2(p.par + 3 * C + c), ka = ld2(p.par + 4 * C + c);
  const bool vres = p.vl != nullptr;
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 wl = ld2(p.wl + o), k = ld2(p.k + o), al = ld2(p.al + o);
      float2 v = ld2(p.v + o);
      const float w_0 = -softplus(-(w0.x + wl.x)) - 0.5f, w_1 = -softplus(-(w0.y + wl.y)) - 0.5f;
      if (vres) {
        const float2 vl = ld2(p.vl + o), vf = ld2(p.vf + o);
        v.x += (vf.x - v.x) * sigm(v0.x + vl.x);
        v.y += (vf.y - v.y) * sigm(v0.y + vl.y);
      }
      const float a_0 = sigm(a0.x + al.x), a_1 = sigm(a0.y + al.y);
      const float kr0 = k.x * kk_.x, kr1 = k.y * kk_.y;
      const float inv = 1.0f / fmaxf(sqrtf(warp_sum(kr0 * kr0 + kr1 * kr1)), 1e-12f);
      const float kn0 = kr0 * inv, kn1 = kr1 * inv;
      st2(p.w + o, w_0, w_1);
      st2(p.ko + o, k.x * (1.f + (a_0 - 1.f) * ka.x), k.y * (1.f + (a_1 - 1.f) * ka.y));
      st2(p.vo + o, v.x, v.y);
      st2(p.a + o, -kn0, -kn1);
      st2(p.b + o, kn0 * a_0, kn1 * a_1);
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
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 w0 = ld2(p.par + c), v0 = ld2(p.par + C + c), a0 = ld2(p.par + 2 * C + c);
  const float2 kk_ = ld2(p.par + 3 * C + c), ka = ld2(p.par + 4 * C + c);
  const bool vres = p.vl != nullptr;
  float acc[5][2] = {};  // w0, v0, a0, k_k, k_a
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      {
        const float2 x = ld2(p.dr_op + o), y = ld2(p.dr_epi + o);
        st2(p.dr + o, x.x + y.x, x.y + y.y);
      }
      const float2 gw = ld2(p.dw_op + o), gk1 = ld2(p.dk_op + o), gk2 = ld2(p.dk_epi + o);
      const float2 gv1 = ld2(p.dv_op + o), gv2 = ld2(p.dv_epi + o);
      const float2 ga = ld2(p.da_op + o), gb = ld2(p.db_op + o);
      const float2 wl = ld2(p.wl + o), k = ld2(p.k + o), al = ld2(p.al + o), v = ld2(p.v + o);
      const float gk[2] = {gk1.x + gk2.x, gk1.y + gk2.y}, gvv[2] = {gv1.x + gv2.x, gv1.y + gv2.y};
      const float kv[2] = {k.x, k.y}, kkv[2] = {kk_.x, kk_.y}, kav[2] = {ka.x, ka.y};
      // decay input: w = -softplus(-u) - 1/2, dw/du = sigmoid(-u) (1 above torch's threshold)
      float dwl[2];
      {
        const float u[2] = {w0.x + wl.x, w0.y + wl.y}, g[2] = {gw.x, gw.y};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          dwl[e] = -u[e] > 20.f ? g[e] : g[e] * sigm(-u[e]);
          acc[0][e] += dwl[e];
        }
      }
      const float a[2] = {sigm(a0.x + al.x), sigm(a0.y + al.y)};
      const float kr[2] = {kv[0] * kkv[0], kv[1] * kkv[1]};
      const float nrm = sqrtf(warp_sum(kr[0] * kr[0] + kr[1] * kr[1]));
      const float den = fmaxf(nrm, 1e-12f);
      const float kn[2] = {kr[0] / den, kr[1] / den};
      const float gav[2] = {ga.x, ga.y}, gbv[2] = {gb.x, gb.y};
      float dkn[2], da[2], dk[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        dkn[e] = -gav[e] + gbv[e] * a[e];                      // a_op = -kk, b_op = kk a
        da[e] = gbv[e] * kn[e] + gk[e] * kv[e] * kav[e];       // k' = k (1 + (a - 1) k_a)
        dk[e] = gk[e] * (1.f + (a[e] - 1.f) * kav[e]);
        acc[4][e] += gk[e] * kv[e] * (a[e] - 1.f);
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
      st2(p.dwl + o, dwl[0], dwl[1]);
      st2(p.dk + o, dk[0], dk[1]);
      st2(p.dal + o, dal[0], dal[1]);
      if (vres) {
        const float2 vl = ld2(p.vl + o), vf = ld2(p.vf + o);
        const float s0 = sigm(v0.x + vl.x), s1 = sigm(v0.y + vl.y);
        const float dvl0 = gvv[0] * (vf.x - v.x) * s0 * (1.f - s0);
        const float dvl1 = gvv[1] * (vf.y - v.y) * s1 * (1.f - s1);
        acc[1][0] += dvl0;
        acc[1][1] += dvl1;
        st2(p.dv + o, gvv[0] * (1.f - s0), gvv[1] * (1.f - s1));
        st2(p.dvf + o, gvv[0] * s0, gvv[1] * s1);
        st2(p.dvl + o, dvl0, dvl1);
      } else {
        float2 gf = make_float2(0.f, 0.f);
        if (p.dvf_out != nullptr) gf = ld2(p.dvf_out + o);  // layer 0: v_first = v
        st2(p.dv + o, gvv[0] + gf.x, gvv[1] + gf.y);
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
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 gm = ld2(p.gamma + c), bt = ld2(p.beta + c), rk = ld2(p.rk + c);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 y = ld2(p.y + o), r = ld2(p.r + o), ko = ld2(p.ko + o), vo = ld2(p.vo + o);
      const float2 g = ld2(p.g + o);
      const float mean = warp_sum(y.x + y.y) * (1.f / 64.f);
      const float d0 = y.x - mean, d1 = y.y - mean;
      const float rstd = rsqrtf(warp_sum(d0 * d0 + d1 * d1) * (1.f / 64.f) + 64e-5f);
      const float s = warp_sum(r.x * ko.x * rk.x + r.y * ko.y * rk.y);
      const float x0 = d0 * rstd * gm.x + bt.x + s * vo.x;
      const float x1 = d1 * rstd * gm.y + bt.y + s * vo.y;
      st2(z + o, x0 * g.x, x1 * g.y);
    }
  }
}

struct PostBwd {
  const bf16* dz;
  bf16 *dy, *dr, *dk, *dv, *dg;
};

__global__ void __launch_bounds__(1024) post_bwd_kernel(Post p, PostBwd q, float* __restrict__ part,
                                                        Shape S) {
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float2 gm = ld2(p.gamma + c), bt = ld2(p.beta + c), rk = ld2(p.rk + c);
  float acc[3][2] = {};  // gamma, beta, r_k
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 y = ld2(p.y + o), r = ld2(p.r + o), ko = ld2(p.ko + o), vo = ld2(p.vo + o);
      const float2 g = ld2(p.g + o), dz = ld2(q.dz + o);
      const float mean = warp_sum(y.x + y.y) * (1.f / 64.f);
      const float d0 = y.x - mean, d1 = y.y - mean;
      const float rstd = rsqrtf(warp_sum(d0 * d0 + d1 * d1) * (1.f / 64.f) + 64e-5f);
      const float s = warp_sum(r.x * ko.x * rk.x + r.y * ko.y * rk.y);
      const float yn0 = d0 * rstd, yn1 = d1 * rstd;
      const float xa0 = yn0 * gm.x + bt.x + s * vo.x, xa1 = yn1 * gm.y + bt.y + s * vo.y;
      const float dx0 = dz.x * g.x, dx1 = dz.y * g.y;  // d x_att
      st2(q.dg + o, dz.x * xa0, dz.y * xa1);
      acc[0][0] += dx0 * yn0;
      acc[0][1] += dx1 * yn1;
      acc[1][0] += dx0;
      acc[1][1] += dx1;
      const float dn0 = dx0 * gm.x, dn1 = dx1 * gm.y;  // d yn
      const float m1 = warp_sum(dn0 + dn1) * (1.f / 64.f);
      const float m2 = warp_sum(dn0 * yn0 + dn1 * yn1) * (1.f / 64.f);
      st2(q.dy + o, rstd * (dn0 - m1 - yn0 * m2), rstd * (dn1 - m1 - yn1 * m2));
      // bonus s v': dv' = dx s, ds = <dx, v'>, s = sum r k' r_k
      st2(q.dv + o, dx0 * s, dx1 * s);
      const float ds = warp_sum(dx0 * vo.x + dx1 * vo.y);
      st2(q.dr + o, ds * ko.x * rk.x, ds * ko.y * rk.y);
      st2(q.dk + o, ds * r.x * rk.x, ds * r.y * rk.y);
      acc[2][0] += ds * r.x * ko.x;
      acc[2][1] += ds * r.y * ko.y;
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 3 * C;
#pragma unroll
  for (int k = 0; k < 3; ++k) st2(pp + k * C + c, acc[k][0], acc[k][1]);
}

// -------------------------------------------------------------------------
// state representation (backbone.py:348): LayerNorm over C, eps 1e-5
__global__ void __launch_bounds__(1024) lnsa_fwd_kernel(const float* __restrict__ sa,
                                                        const float* __restrict__ wt,
                                                        const float* __restrict__ bs,
                                                        float* __restrict__ out, Shape S) {
  __shared__ float2 red[2][32];
  int buf = 0;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float invC = 1.0f / static_cast<float>(C);
  const float2 w = ld2(wt + c), bb = ld2(bs + c);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 x = ld2(sa + o);
      const float mean = block_sum2(make_float2(x.x + x.y, 0.f), red, buf).x * invC;
      const float d0 = x.x - mean, d1 = x.y - mean;
      const float rstd = rsqrtf(block_sum2(make_float2(d0 * d0 + d1 * d1, 0.f), red, buf).x * invC + 1e-5f);
      st2(out + o, d0 * rstd * w.x + bb.x, d1 * rstd * w.y + bb.y);
    }
  }
}

__global__ void __launch_bounds__(1024) lnsa_bwd_kernel(const float* __restrict__ dout,
                                                        const float* __restrict__ sa,
                                                        const float* __restrict__ wt,
                                                        float* __restrict__ dsa,
                                                        float* __restrict__ part, Shape S) {
  __shared__ float2 red[2][32];
  int buf = 0;
  const int c = 2 * threadIdx.x;
  const int64_t C = S.C;
  const float invC = 1.0f / static_cast<float>(C);
  const float2 w = ld2(wt + c);
  float acc[2][2] = {};  // weight, bias
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const float2 x = ld2(sa + o), g = ld2(dout + o);
      const float mean = block_sum2(make_float2(x.x + x.y, 0.f), red, buf).x * invC;
      const float d0 = x.x - mean, d1 = x.y - mean;
      const float rstd = rsqrtf(block_sum2(make_float2(d0 * d0 + d1 * d1, 0.f), red, buf).x * invC + 1e-5f);
      const float xn0 = d0 * rstd, xn1 = d1 * rstd;
      acc[0][0] += g.x * xn0;
      acc[0][1] += g.y * xn1;
      acc[1][0] += g.x;
      acc[1][1] += g.y;
      const float dn0 = g.x * w.x, dn1 = g.y * w.y;
      const float2 m = block_sum2(make_float2(dn0 + dn1, dn0 * xn0 + dn1 * xn1), red, buf);
      const float m1 = m.x * invC, m2 = m.y * invC;
      st2(dsa + o, rstd * (dn0 - m1 - xn0 * m2), rstd * (dn1 - m1 - xn1 * m2));
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 2 * C;
  st2(pp + c, acc[0][0], acc[0][1]);
  st2(pp + C + c, acc[1][0], acc[1][1]);
}

// out[i] = sum over g < G of part[g * n + i], in order of g
__global__ void partial_reduce_kernel(const float* __restrict__ part, int G, int64_t n,
                                      float* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int g = 0; g < G; ++g) s += part[g * n + i];
    out[i] = s;
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

int grid_for(const Shape& S) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per_sm = 2048 / (S.C / 2);  // CTAs of C/2 threads resident per SM
  int64_t g = sms * per_sm;
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
  const int64_t blocks = (n + 255) / 256;
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
  const int G = camoe::tm::grid_for(S);
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
  const int G = camoe::tm::grid_for(S);
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
  camoe::tm::prep_fwd_kernel<<<camoe::tm::grid_for(S), static_cast<unsigned>(C / 2), 0,
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
  const int G = camoe::tm::grid_for(S);
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
  camoe::tm::post_fwd_kernel<<<camoe::tm::grid_for(S), static_cast<unsigned>(C / 2), 0,
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
  const int G = camoe::tm::grid_for(S);
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
  camoe::tm::lnsa_fwd_kernel<<<camoe::tm::grid_for(S), static_cast<unsigned>(C / 2), 0,
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
  const int G = camoe::tm::grid_for(S);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  camoe::tm::lnsa_bwd_kernel<<<G, static_cast<unsigned>(C / 2), 0, s>>>(dout, sa, weight, dsa, part, S);
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 2 * C, dparams, s);
}

}  // extern "C"
