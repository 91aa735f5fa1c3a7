// Fused elementwise kernels of RWKV-7's time mix around the WKV-7 op
// (camoe/backbone.py:296-373), declared in include/camoe_timemix.h.
//
// Each kernel is one pass over HBM for what the reference runs as chains of
// eager PyTorch ops (each a separate read and write of [B, T, C] tensors).
// Layout: one CTA owns one row (one time step of one sequence) at a time.
// In mix_fwd, post and lnsa the CTA has C/8 threads and thread i holds
// columns 8i..8i+7 (one 16-byte access per bf16 tensor, two per fp32 one), so
// a head (64 columns) is 8 adjacent threads and a per-head sum (GroupNorm,
// the bonus term) is three xor-shuffles; the LayerNorm over C adds one
// shared-memory step (lnsa for C > 1024; up to C = 1024 it runs one warp per
// row, shuffles only, lnsa_*_rows_kernel).  mix_bwd and prep, which keep the most values live per
// column (six mixes and their gradient sums; fifteen input tensors), use C/2
// threads of two columns each (warp = head) so that they fit in 64 registers
// at full occupancy: measured faster than eight columns on B200.
// CTAs walk work items of kRows consecutive steps of one sequence (the token
// shift takes the neighbouring step from registers), U rows in flight per
// thread: the loads of U rows are issued before any of them is used.
// Per-column parameters too many for registers live in shared memory.
// Parameter gradients are summed over a CTA's rows in registers, written as
// one partial row per CTA and added by partial_reduce_kernel in a fixed
// order (deterministic).  All arithmetic is fp32; activations are bf16.
#include <initializer_list>
#include <type_traits>

#include "camoe_timemix.h"
#include "wkv7_common.cuh"
#include "wkv7_sync.cuh"

namespace camoe {
void set_last_cuda_error(int e);  // wkv7_capi.cu: reported by camoe_wkv7_last_cuda_error()

namespace tm {

constexpr int kRows = 4;       // time steps per work item (small items balance the one wave)
constexpr int kMaxGrid = 1024;
constexpr int kMaxParams = 6;  // parameter vectors of the backward with the most (mix)
constexpr int V = 8;           // columns per thread

struct Shape {
  int64_t B, T, C;
  int64_t nblk;  // ceil(T / kRows)
  __host__ __device__ int64_t items() const { return B * nblk; }
};

// 8 bf16 <-> 8 floats
__device__ __forceinline__ uint4 ldv(const bf16* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[V]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void ld8(const bf16* p, float (&f)[V]) { unpack(ldv(p), f); }
__device__ __forceinline__ void ld8(const float* p, float (&f)[V]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void st8(bf16* p, const float (&f)[V]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void st8(float* p, const float (&f)[V]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// lanes of this thread's warp that exist (the last warp of a CTA of C/8 < 32
// threads, or of C/8 not a multiple of 32, is partial)
__device__ __forceinline__ unsigned warp_lanes() {
  const unsigned n = blockDim.x - (threadIdx.x & ~31u);
  return n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
}
// sum over the 8 threads of a head
__device__ __forceinline__ float head_sum(float x, unsigned m) {
  x += __shfl_xor_sync(m, x, 1);
  x += __shfl_xor_sync(m, x, 2);
  x += __shfl_xor_sync(m, x, 4);
  return x;
}
__device__ __forceinline__ float sum8(const float (&a)[V]) {
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// The gates and the decay input end in bf16 (8 significant bits), so they
// use the hardware's base-2 exponential and logarithm (__expf, __logf: a few
// ulp) and an approximate reciprocal (__fdividef): an IEEE division or log1pf
// takes ten to twenty instructions each, which left prep_fwd issue-bound at
// about half of HBM bandwidth.  1 / (1 + inf) is 0, as the limit wants.
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
// torch's softplus with threshold 20; its error (a few ulp of __expf and
// __logf, and below z = -16.6 a result of 0 where e^z < 6e-8) stays below
// 1e-5 of the decay input -softplus(-u) - 1/2, which is rounded to bf16
__device__ __forceinline__ float softplus(float z) { return z > 20.0f ? z : __logf(1.0f + __expf(z)); }
// 1 / max(sqrt(ss), 1e-12): F.normalize's divisor, as one reciprocal square root
__device__ __forceinline__ float inv_norm(float ss) { return rsqrtf(fmaxf(ss, 1e-24f)); }

// rows [t0, t1) of sequence b for work item `item`
__device__ __forceinline__ void item_rows(const Shape& S, int64_t item, int64_t& b, int64_t& t0,
                                          int64_t& t1) {
  b = item / S.nblk;
  t0 = (item - b * S.nblk) * kRows;
  t1 = t0 + kRows < S.T ? t0 + kRows : S.T;
}

// Two-columns-per-thread kernels (CTA of C/2 threads, warp = head): the
// layout of the kernels with the most live values per column, where eight
// columns per thread would cost occupancy.
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
__device__ __forceinline__ float2 f2(const __nv_bfloat162& v) { return __bfloat1622float2(v); }
__device__ __forceinline__ float2 f2(const float2& v) { return v; }
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
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

// x_prev (nullable): [B, C], the step before step 0 of each sequence (the
// token-shift state of a stateful call); zero when null, as in the reference
template <typename Tx>
__global__ void __launch_bounds__(256) mix_fwd_kernel(const Tx* __restrict__ x,
                                                      const Tx* __restrict__ x_prev,
                                                      const float* __restrict__ mix, Out6 out,
                                                      Shape S) {
  const int c = V * threadIdx.x;
  const int64_t C = S.C;
  float mx[6][V];
#pragma unroll
  for (int m = 0; m < 6; ++m) ld8(mix + m * C + c, mx[m]);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    float xp[V];
    if (t0 > 0) {
      ld8(x + (b * S.T + t0 - 1) * C + c, xp);
    } else if (x_prev != nullptr) {
      ld8(x_prev + b * C + c, xp);
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) xp[e] = 0.f;
    }
    float xc[kRows][V];
#pragma unroll
    for (int u = 0; u < kRows; ++u) {  // rows past the item repeat its last one
      const int64_t t = t0 + u < t1 ? t0 + u : t1 - 1;
      ld8(x + (b * S.T + t) * C + c, xc[u]);
    }
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      float d[V];
#pragma unroll
      for (int e = 0; e < V; ++e) d[e] = xp[e] - xc[u][e];
      if (t0 + u < t1) {
        const int64_t o = (b * S.T + t0 + u) * C + c;
#pragma unroll
        for (int m = 0; m < 6; ++m) {
          float y[V];
#pragma unroll
          for (int e = 0; e < V; ++e) y[e] = xc[u][e] + d[e] * mx[m][e];
          st8(out.p[m] + o, y);
        }
      }
#pragma unroll
      for (int e = 0; e < V; ++e) xp[e] = xc[u][e];
    }
  }
}

// dx[t] = sum_m dx_m[t] (1 - mix_m) + sum_m dx_m[t+1] mix_m;  dmix_m = sum_t dx_m[t] xx[t]
// With s[t] = sum_m dx_m[t] and q[t] = sum_m dx_m[t] mix_m this is
// dx[t] = s[t] - q[t] + q[t+1]: rows are walked downwards carrying one q per
// column instead of the six dx_m of the next row.  Each CTA takes a contiguous
// range of work items (the walk goes down through it, so q carries from item to
// item and is loaded only for the row after the range), which leaves the
// registers for a whole item's rows, all of whose loads are issued before the
// first is used.  The mixes sit in shared memory, each thread reading back its
// own columns.
template <typename Tx>
__global__ void __launch_bounds__(1024) mix_bwd_kernel(const Tx* __restrict__ x,
                                                       const float* __restrict__ mix, In6 dout,
                                                       Tx* __restrict__ dx,
                                                       float* __restrict__ part, Shape S) {
  using X2 = typename std::conditional<std::is_same<Tx, float>::value, float2, __nv_bfloat162>::type;
  extern __shared__ float2 mxs[];  // [6][C / 2]: the mixes of each thread's columns
  const int c = 2 * threadIdx.x, nt = blockDim.x;
  const int64_t C = S.C;
  float2 acc[6];
#pragma unroll
  for (int m = 0; m < 6; ++m) {
    mxs[m * nt + threadIdx.x] = ld2(mix + m * C + c);
    acc[m] = make_float2(0.f, 0.f);
  }
  const float2* mx = mxs + threadIdx.x;  // mx[m * nt]: read back by this thread only
  const int64_t n = S.items();
  const int64_t i0 = blockIdx.x * n / gridDim.x, i1 = (blockIdx.x + 1) * n / gridDim.x;
  float2 qn = make_float2(0.f, 0.f);  // q of the row after the current item
  for (int64_t item = i1 - 1; item >= i0; --item) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    const int64_t o = (b * S.T + t0) * C + c;  // row t0, this thread's columns
    if (t1 == S.T) {
      qn = make_float2(0.f, 0.f);  // past the sequence's end
    } else if (item == i1 - 1) {   // the row after the range: another CTA's
      const int64_t on = o + (t1 - t0) * C;
#pragma unroll
      for (int m = 0; m < 6; ++m) {
        const float2 g = ld2(dout.p[m] + on), w = mx[m * nt];
        qn.x += g.x * w.x;
        qn.y += g.y * w.y;
      }
    }  // else qn is the q of row t1, the last row walked in item + 1
    __nv_bfloat162 d[kRows][6];  // rows past the item repeat its last one
    X2 xr[kRows + 1];            // x[t0 - 1 + u], as loaded
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      const int64_t ou = o + (t0 + u < t1 ? u : t1 - 1 - t0) * C;
#pragma unroll
      for (int m = 0; m < 6; ++m) d[u][m] = *reinterpret_cast<const __nv_bfloat162*>(dout.p[m] + ou);
      xr[u + 1] = *reinterpret_cast<const X2*>(x + ou);
    }
    if (t0 > 0) xr[0] = *reinterpret_cast<const X2*>(x + o - C);
#pragma unroll
    for (int u = kRows - 1; u >= 0; --u) {
      if (t0 + u >= t1) continue;  // the same for the whole CTA
      float2 s = make_float2(0.f, 0.f), q = make_float2(0.f, 0.f);
      const float2 xa = u > 0 || t0 > 0 ? f2(xr[u]) : make_float2(0.f, 0.f), xb = f2(xr[u + 1]);
      const float2 xx = make_float2(xa.x - xb.x, xa.y - xb.y);
#pragma unroll
      for (int m = 0; m < 6; ++m) {
        const float2 g = __bfloat1622float2(d[u][m]), w = mx[m * nt];
        s.x += g.x;
        s.y += g.y;
        q.x += g.x * w.x;
        q.y += g.y * w.y;
        acc[m].x += g.x * xx.x;
        acc[m].y += g.y * xx.y;
      }
      st2(dx + o + u * C, s.x - q.x + qn.x, s.y - q.y + qn.y);
      qn = q;
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 6 * C;
#pragma unroll
  for (int m = 0; m < 6; ++m) st2(pp + m * C + c, acc[m].x, acc[m].y);
}

// mix_bwd for bf16 x and C <= 1024 with its rows streamed through shared
// memory: one producer thread copies each work item's rows (the six mix
// gradients' rows t0..t1-1 and x's rows t0-1..t1-1, each a contiguous run of
// one sequence) into a ring of kRingStages stages with 1-D bulk copies behind
// mbarriers, and the C/2 consumer threads (two columns each, as in
// mix_bwd_kernel) compute from there.  The loads in flight then no longer
// need registers (the register-staged kernel waits on load latency with one
// item per thread in flight); same arithmetic and item order as
// mix_bwd_kernel.  Waits are bounded (wkv7_sync.cuh).
constexpr int kRingStages = 3;

__host__ __device__ inline size_t ring_stage_elems(int64_t C) {  // bf16 elements of a stage
  return static_cast<size_t>(6 * kRows + kRows + 1) * static_cast<size_t>(C);
}
inline size_t ring_smem(int64_t C) {
  return 6 * static_cast<size_t>(C) * sizeof(float) + kRingStages * ring_stage_elems(C) * sizeof(bf16) +
         2 * kRingStages * sizeof(uint64_t);
}

__global__ void __launch_bounds__(544) mix_bwd_ring_kernel(const bf16* __restrict__ x,
                                                           const float* __restrict__ mix, In6 dout,
                                                           bf16* __restrict__ dx,
                                                           float* __restrict__ part, Shape S) {
  extern __shared__ __align__(16) unsigned char ring_raw[];
  const int64_t C = S.C;
  const int nt = static_cast<int>(C / 2), tid = threadIdx.x, lane = tid & 31;
  const size_t se = ring_stage_elems(C);
  float2* mxs = reinterpret_cast<float2*>(ring_raw);  // [6][nt]
  bf16* stages = reinterpret_cast<bf16*>(ring_raw + 6 * C * sizeof(float));
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kRingStages * se);
  uint64_t* empty = full + kRingStages;
  if (tid == 0) {
    for (int s = 0; s < kRingStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], static_cast<uint32_t>(nt / 32));  // one arrival per consumer warp
    }
    mbar_fence_init();
  }
  if (tid < nt)
#pragma unroll
    for (int m = 0; m < 6; ++m) mxs[m * nt + tid] = ld2(mix + m * C + 2 * tid);
  __syncthreads();
  const int64_t n = S.items();
  const int64_t i0 = blockIdx.x * n / gridDim.x, i1 = (blockIdx.x + 1) * n / gridDim.x;
  const uint32_t rowb = static_cast<uint32_t>(C * sizeof(bf16));

  if (tid >= nt) {  // the producer warp: its first thread copies, item by item (downwards)
    if (tid == nt) {
      int64_t k = 0;
      for (int64_t item = i1 - 1; item >= i0; --item, ++k) {
        const int s = static_cast<int>(k % kRingStages);
        if (k >= kRingStages &&
            !mbar_wait(&empty[s], static_cast<uint32_t>((k / kRingStages - 1) & 1)))
          break;
        int64_t b, t0, t1;
        item_rows(S, item, b, t0, t1);
        const uint32_t rows = static_cast<uint32_t>(t1 - t0);
        const int64_t row0 = b * S.T + t0;
        mbar_arrive_expect_tx(&full[s], 6 * rows * rowb + (rows + (t0 > 0 ? 1u : 0u)) * rowb);
        bf16* st = stages + s * se;
#pragma unroll
        for (int m = 0; m < 6; ++m)
          bulk_g2s(st + m * kRows * C, dout.p[m] + row0 * C, rows * rowb, &full[s]);
        if (t0 > 0)  // x[t0 - 1 .. t1 - 1] at rows 0 .. rows of the x block
          bulk_g2s(st + 6 * kRows * C, x + (row0 - 1) * C, (rows + 1) * rowb, &full[s]);
        else         // x[-1] is zero: rows 1 .. rows
          bulk_g2s(st + (6 * kRows + 1) * C, x + row0 * C, rows * rowb, &full[s]);
      }
      // keep the CTA alive until every copy it issued has landed
      for (int64_t j = k - 1; j >= 0 && j >= k - kRingStages; --j)
        mbar_wait(&full[j % kRingStages], static_cast<uint32_t>((j / kRingStages) & 1));
    }
    return;
  }

  const int c = 2 * tid;
  const float2* mx = mxs + tid;  // mx[m * nt]
  float2 acc[6];
#pragma unroll
  for (int m = 0; m < 6; ++m) acc[m] = make_float2(0.f, 0.f);
  float2 qn = make_float2(0.f, 0.f);  // q of the row after the current item
  int64_t k = 0;
  for (int64_t item = i1 - 1; item >= i0; --item, ++k) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    const int64_t row0 = b * S.T + t0;
    const int rows = static_cast<int>(t1 - t0);
    if (t1 == S.T) {
      qn = make_float2(0.f, 0.f);
    } else if (item == i1 - 1) {  // the row after the range: another CTA's
#pragma unroll
      for (int m = 0; m < 6; ++m) {
        const float2 g = ld2(dout.p[m] + (row0 + rows) * C + c), w = mx[m * nt];
        qn.x += g.x * w.x;
        qn.y += g.y * w.y;
      }
    }
    const int s = static_cast<int>(k % kRingStages);
    if (!mbar_wait(&full[s], static_cast<uint32_t>((k / kRingStages) & 1))) break;
    const bf16* st = stages + s * se;
#pragma unroll
    for (int u = kRows - 1; u >= 0; --u) {
      if (u >= rows) continue;  // the same for the whole CTA
      const float2 xa = u > 0 || t0 > 0 ? ld2(st + (6 * kRows + u) * C + c) : make_float2(0.f, 0.f);
      const float2 xb = ld2(st + (6 * kRows + u + 1) * C + c);
      const float2 xx = make_float2(xa.x - xb.x, xa.y - xb.y);
      float2 sm = make_float2(0.f, 0.f), q = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 6; ++m) {
        const float2 g = ld2(st + (m * kRows + u) * C + c), w = mx[m * nt];
        sm.x += g.x;
        sm.y += g.y;
        q.x += g.x * w.x;
        q.y += g.y * w.y;
        acc[m].x += g.x * xx.x;
        acc[m].y += g.y * xx.y;
      }
      st2(dx + (row0 + u) * C + c, sm.x - q.x + qn.x, sm.y - q.y + qn.y);
      qn = q;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 6 * C;
#pragma unroll
  for (int m = 0; m < 6; ++m) st2(pp + m * C + c, acc[m].x, acc[m].y);
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
          const float inv = inv_norm(warp_sum(kr0 * kr0 + kr1 * kr1));
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
        const float ss = warp_sum(kr[0] * kr[0] + kr[1] * kr[1]);
        const float inv = inv_norm(ss);  // 1 / max(|kr|, 1e-12)
        const float kn[2] = {kr[0] * inv, kr[1] * inv};
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
          const float dkr = (ss > 1e-24f ? dkn[e] - kn[e] * dot : dkn[e]) * inv;
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

__global__ void __launch_bounds__(256) post_fwd_kernel(Post p, bf16* __restrict__ z, Shape S) {
  constexpr int U = 2;
  const int c = V * threadIdx.x;
  const int64_t C = S.C;
  const unsigned lanes = warp_lanes();
  float gm[V], bt[V], rk[V];
  ld8(p.gamma + c, gm);
  ld8(p.beta + c, bt);
  ld8(p.rk + c, rk);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      uint4 y[U], r[U], ko[U], vo[U], g[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {  // rows past the item repeat its last one
        const int64_t o = (b * S.T + (tb + u < t1 ? tb + u : t1 - 1)) * C + c;
        y[u] = ldv(p.y + o); r[u] = ldv(p.r + o); ko[u] = ldv(p.ko + o); vo[u] = ldv(p.vo + o);
        g[u] = ldv(p.g + o);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float yf[V], rf[V], kf[V], sr = 0.f;
        unpack(y[u], yf);
        unpack(r[u], rf);
        unpack(ko[u], kf);
#pragma unroll
        for (int e = 0; e < V; ++e) sr += rf[e] * kf[e] * rk[e];
        const float mean = head_sum(sum8(yf), lanes) * (1.f / 64.f);
        float vs = 0.f;
#pragma unroll
        for (int e = 0; e < V; ++e) {
          yf[e] -= mean;
          vs += yf[e] * yf[e];
        }
        const float rstd = rsqrtf(head_sum(vs, lanes) * (1.f / 64.f) + 64e-5f);
        const float s = head_sum(sr, lanes);
        if (tb + u >= t1) continue;
        float vf[V], gf[V];
        unpack(vo[u], vf);
        unpack(g[u], gf);
#pragma unroll
        for (int e = 0; e < V; ++e) yf[e] = (yf[e] * rstd * gm[e] + bt[e] + s * vf[e]) * gf[e];
        st8(z + (b * S.T + tb + u) * C + c, yf);
      }
    }
  }
}

struct PostBwd {
  const bf16* dz;
  bf16 *dy, *dr, *dk, *dv, *dg;
};

__global__ void __launch_bounds__(256) post_bwd_kernel(Post p, PostBwd q, float* __restrict__ part,
                                                       Shape S) {
  const int c = V * threadIdx.x;
  const int64_t C = S.C;
  const unsigned lanes = warp_lanes();
  float gm[V], rk[V];
  ld8(p.gamma + c, gm);
  ld8(p.rk + c, rk);
  float acc[3][V];  // gamma, beta, r_k
#pragma unroll
  for (int k = 0; k < 3; ++k)
#pragma unroll
    for (int e = 0; e < V; ++e) acc[k][e] = 0.f;
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t o = (b * S.T + t) * C + c;
      const uint4 yp = ldv(p.y + o), rp = ldv(p.r + o), kp = ldv(p.ko + o), vp = ldv(p.vo + o);
      const uint4 gp = ldv(p.g + o), dzp = ldv(q.dz + o);
      float yn[V], rf[V], kf[V], sr = 0.f;
      unpack(yp, yn);
      unpack(rp, rf);
      unpack(kp, kf);
#pragma unroll
      for (int e = 0; e < V; ++e) sr += rf[e] * kf[e] * rk[e];
      const float mean = head_sum(sum8(yn), lanes) * (1.f / 64.f);
      float vs = 0.f;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        yn[e] -= mean;
        vs += yn[e] * yn[e];
      }
      const float rstd = rsqrtf(head_sum(vs, lanes) * (1.f / 64.f) + 64e-5f);
      const float s = head_sum(sr, lanes);
      float vf[V], gf[V], dz[V], bt[V];
      unpack(vp, vf);
      unpack(gp, gf);
      unpack(dzp, dz);
      ld8(p.beta + c, bt);
      float dxa[V], m1 = 0.f, m2 = 0.f, dsv = 0.f;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        yn[e] *= rstd;
        const float xa = yn[e] * gm[e] + bt[e] + s * vf[e];
        dxa[e] = dz[e] * gf[e];             // d x_att
        gf[e] = dz[e] * xa;                 // dg (gf reused)
        acc[0][e] += dxa[e] * yn[e];
        acc[1][e] += dxa[e];
        const float dn = dxa[e] * gm[e];    // d yn
        m1 += dn;
        m2 += dn * yn[e];
        dsv += dxa[e] * vf[e];
      }
      st8(q.dg + o, gf);
      m1 = head_sum(m1, lanes) * (1.f / 64.f);
      m2 = head_sum(m2, lanes) * (1.f / 64.f);
      const float ds = head_sum(dsv, lanes);  // bonus s v': ds = <dx, v'>, s = sum r k' r_k
#pragma unroll
      for (int e = 0; e < V; ++e) {
        dz[e] = rstd * (dxa[e] * gm[e] - m1 - yn[e] * m2);  // dy (dz reused)
        vf[e] = dxa[e] * s;                                 // dv'
        acc[2][e] += ds * rf[e] * kf[e];
      }
      st8(q.dy + o, dz);
      st8(q.dv + o, vf);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const float dr = ds * kf[e] * rk[e], dk = ds * rf[e] * rk[e];
        rf[e] = dr;
        kf[e] = dk;
      }
      st8(q.dr + o, rf);
      st8(q.dk + o, kf);
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 3 * C;
#pragma unroll
  for (int k = 0; k < 3; ++k) st8(pp + k * C + c, acc[k]);
}

// -------------------------------------------------------------------------
// state representation (backbone.py:348): LayerNorm over C, eps 1e-5.  The
// CTA is the row; the U rows of an iteration share each CTA-wide sum.
template <int U>
__device__ __forceinline__ void row_sums(float (&v)[U][2], float2 (*red)[8][U], int& buf,
                                         unsigned lanes) {
  const int warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;  // nw <= 8 (C <= 2048)
  const int lane = threadIdx.x & 31, n = __popc(lanes);  // a partial last warp has n < 32 lanes
  // lane 0 of each warp collects its warp's sum (shuffles from lanes past n are not used)
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_down_sync(lanes, v[u][j], o);
        if (lane + o < n) v[u][j] += t;
      }
  if (lane == 0)
#pragma unroll
    for (int u = 0; u < U; ++u) red[buf][warp][u] = make_float2(v[u][0], v[u][1]);
  __syncthreads();
#pragma unroll
  for (int u = 0; u < U; ++u) {
    float2 t = red[buf][0][u];
    for (int w = 1; w < nw; ++w) {
      const float2 x = red[buf][w][u];
      t.x += x.x;
      t.y += x.y;
    }
    v[u][0] = t.x;
    v[u][1] = t.y;
  }
  buf ^= 1;
}

__global__ void __launch_bounds__(256) lnsa_fwd_kernel(const float* __restrict__ sa,
                                                       const float* __restrict__ wt,
                                                       const float* __restrict__ bs,
                                                       float* __restrict__ out, Shape S) {
  constexpr int U = kRows;
  __shared__ float2 red[2][8][U];
  int buf = 0;
  const int c = V * threadIdx.x;
  const int64_t C = S.C;
  const unsigned lanes = warp_lanes();
  const float invC = 1.0f / static_cast<float>(C);
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    float x[U][V], s[U][2];
#pragma unroll
    for (int u = 0; u < U; ++u) {  // rows past the item repeat its last one
      ld8(sa + (b * S.T + (t0 + u < t1 ? t0 + u : t1 - 1)) * C + c, x[u]);
      s[u][0] = sum8(x[u]);
      s[u][1] = 0.f;
    }
    row_sums<U>(s, red, buf, lanes);  // mean
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float mean = s[u][0] * invC;
      float q = 0.f;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        x[u][e] -= mean;
        q += x[u][e] * x[u][e];
      }
      s[u][0] = q;
    }
    row_sums<U>(s, red, buf, lanes);  // variance about the mean (two passes)
    float w[V], bb[V];
    ld8(wt + c, w);
    ld8(bs + c, bb);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (t0 + u >= t1) continue;
      const float rstd = rsqrtf(s[u][0] * invC + 1e-5f);
      float y[V];
#pragma unroll
      for (int e = 0; e < V; ++e) y[e] = x[u][e] * rstd * w[e] + bb[e];
      st8(out + (b * S.T + t0 + u) * C + c, y);
    }
  }
}

__global__ void __launch_bounds__(256) lnsa_bwd_kernel(const float* __restrict__ dout,
                                                       const float* __restrict__ sa,
                                                       const float* __restrict__ wt,
                                                       float* __restrict__ dsa,
                                                       float* __restrict__ part, Shape S) {
  constexpr int U = 4;
  __shared__ float2 red[2][8][U];
  int buf = 0;
  const int c = V * threadIdx.x;
  const int64_t C = S.C;
  const unsigned lanes = warp_lanes();
  const float invC = 1.0f / static_cast<float>(C);
  float w[V], acc[2][V];  // weight, bias
  ld8(wt + c, w);
#pragma unroll
  for (int e = 0; e < V; ++e) acc[0][e] = acc[1][e] = 0.f;
  for (int64_t item = blockIdx.x; item < S.items(); item += gridDim.x) {
    int64_t b, t0, t1;
    item_rows(S, item, b, t0, t1);
    for (int64_t tb = t0; tb < t1; tb += U) {
      float x[U][V], g[U][V], s[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {  // rows past the item repeat its last one, with g = 0
        const int64_t o = (b * S.T + (tb + u < t1 ? tb + u : t1 - 1)) * C + c;
        ld8(sa + o, x[u]);
        ld8(dout + o, g[u]);
        if (tb + u >= t1)
#pragma unroll
          for (int e = 0; e < V; ++e) g[u][e] = 0.f;
        s[u][0] = sum8(x[u]);
        s[u][1] = 0.f;
      }
      row_sums<U>(s, red, buf, lanes);  // mean
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float mean = s[u][0] * invC;
        float q = 0.f;
#pragma unroll
        for (int e = 0; e < V; ++e) {
          x[u][e] -= mean;
          q += x[u][e] * x[u][e];
        }
        s[u][0] = q;
      }
      row_sums<U>(s, red, buf, lanes);  // variance
      float rstd[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        rstd[u] = rsqrtf(s[u][0] * invC + 1e-5f);
        float m1 = 0.f, m2 = 0.f;
#pragma unroll
        for (int e = 0; e < V; ++e) {
          x[u][e] *= rstd[u];                  // xn
          acc[0][e] += g[u][e] * x[u][e];
          acc[1][e] += g[u][e];
          g[u][e] *= w[e];                     // d xn
          m1 += g[u][e];
          m2 += g[u][e] * x[u][e];
        }
        s[u][0] = m1;
        s[u][1] = m2;
      }
      row_sums<U>(s, red, buf, lanes);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (tb + u >= t1) continue;
        const float m1 = s[u][0] * invC, m2 = s[u][1] * invC;
        float d[V];
#pragma unroll
        for (int e = 0; e < V; ++e) d[e] = rstd[u] * (g[u][e] - m1 - x[u][e] * m2);
        st8(dsa + (b * S.T + tb + u) * C + c, d);
      }
    }
  }
  float* pp = part + static_cast<int64_t>(blockIdx.x) * 2 * C;
  st8(pp + c, acc[0]);
  st8(pp + C + c, acc[1]);
}

// LayerNorm of sa for C <= 1024 (C = 64 J): one warp per row, the CTA's eight
// warps taking rows in turn (grid-strided), lane l holding the column pairs
// 2(l + 32 j), j < J, so each load and store of a row is J coalesced 256-byte
// warp accesses and every sum over the row is five xor-shuffles: no CTA
// barrier couples the warps, which the C/8-thread layout above needs for each
// of its row sums.  Weight and bias are staged once in shared memory.  Same
// arithmetic as lnsa_fwd_kernel (two-pass variance, eps 1e-5).
constexpr int kRowWarps = 8;  // warps of a row kernel's CTA

template <int J>
__global__ void __launch_bounds__(32 * kRowWarps) lnsa_fwd_rows_kernel(
    const float* __restrict__ sa, const float* __restrict__ wt, const float* __restrict__ bs,
    float* __restrict__ out, int64_t rows) {
  constexpr int C = 64 * J, P = 32 * J;  // columns, column pairs
  __shared__ float2 pw[P], pb[P];
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    pw[i] = reinterpret_cast<const float2*>(wt)[i];
    pb[i] = reinterpret_cast<const float2*>(bs)[i];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kRowWarps;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5); r < rows;
       r += step) {
    const float2* src = reinterpret_cast<const float2*>(sa + r * C) + lane;
    float2 x[J];
#pragma unroll
    for (int j = 0; j < J; ++j) x[j] = src[32 * j];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) s += x[j].x + x[j].y;
    const float mean = warp_sum(s) * (1.0f / static_cast<float>(C));
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      x[j].x -= mean;
      x[j].y -= mean;
      q += x[j].x * x[j].x + x[j].y * x[j].y;
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / static_cast<float>(C)) + 1e-5f);
    float2* dst = reinterpret_cast<float2*>(out + r * C) + lane;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float2 w = pw[lane + 32 * j], b = pb[lane + 32 * j];
      dst[32 * j] = make_float2(x[j].x * rstd * w.x + b.x, x[j].y * rstd * w.y + b.y);
    }
  }
}

// Backward of lnsa_fwd_rows_kernel, same layout.  Each warp adds its rows'
// weight and bias gradients into its own slice of shared memory (a lane
// touches only its own columns, so no barrier is needed per row); at the end
// the CTA adds its eight slices in warp order into one partial row of part,
// [weight C | bias C] as lnsa_bwd_kernel writes it.
// Dynamic shared memory: lnsa_rows_smem(J) bytes.
template <int J>
__global__ void __launch_bounds__(32 * kRowWarps) lnsa_bwd_rows_kernel(
    const float* __restrict__ dout, const float* __restrict__ sa, const float* __restrict__ wt,
    float* __restrict__ dsa, float* __restrict__ part, int64_t rows) {
  constexpr int C = 64 * J, P = 32 * J;
  extern __shared__ float2 rsm[];  // weight [P], then per warp [weight grad P | bias grad P]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float2* pw = rsm;
  float2* acc = rsm + P + warp * 2 * P;
  for (int i = threadIdx.x; i < P; i += blockDim.x) pw[i] = reinterpret_cast<const float2*>(wt)[i];
  for (int i = threadIdx.x; i < kRowWarps * 2 * P; i += blockDim.x) rsm[P + i] = make_float2(0.f, 0.f);
  __syncthreads();
  const int64_t step = static_cast<int64_t>(gridDim.x) * kRowWarps;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp; r < rows; r += step) {
    const float2* xs = reinterpret_cast<const float2*>(sa + r * C) + lane;
    const float2* gs = reinterpret_cast<const float2*>(dout + r * C) + lane;
    float2 x[J], g[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      x[j] = xs[32 * j];
      g[j] = gs[32 * j];
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) s += x[j].x + x[j].y;
    const float mean = warp_sum(s) * (1.0f / static_cast<float>(C));
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      x[j].x -= mean;
      x[j].y -= mean;
      q += x[j].x * x[j].x + x[j].y * x[j].y;
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / static_cast<float>(C)) + 1e-5f);
    float m1 = 0.f, m2 = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = lane + 32 * j;
      x[j].x *= rstd;  // xn
      x[j].y *= rstd;
      float2 aw = acc[i], ab = acc[P + i];
      aw.x += g[j].x * x[j].x;
      aw.y += g[j].y * x[j].y;
      ab.x += g[j].x;
      ab.y += g[j].y;
      acc[i] = aw;
      acc[P + i] = ab;
      const float2 w = pw[i];
      g[j].x *= w.x;  // d xn
      g[j].y *= w.y;
      m1 += g[j].x + g[j].y;
      m2 += g[j].x * x[j].x + g[j].y * x[j].y;
    }
    m1 = warp_sum(m1) * (1.0f / static_cast<float>(C));
    m2 = warp_sum(m2) * (1.0f / static_cast<float>(C));
    float2* dst = reinterpret_cast<float2*>(dsa + r * C) + lane;
#pragma unroll
    for (int j = 0; j < J; ++j)
      dst[32 * j] = make_float2(rstd * (g[j].x - m1 - x[j].x * m2),
                                rstd * (g[j].y - m1 - x[j].y * m2));
  }
  __syncthreads();
  float2* pp = reinterpret_cast<float2*>(part) + static_cast<int64_t>(blockIdx.x) * 2 * P;
  for (int i = threadIdx.x; i < 2 * P; i += blockDim.x) {
    float2 t = rsm[P + i];
#pragma unroll
    for (int w = 1; w < kRowWarps; ++w) {
      const float2 u = rsm[P + w * 2 * P + i];
      t.x += u.x;
      t.y += u.y;
    }
    pp[i] = t;
  }
}

constexpr size_t lnsa_rows_smem(int J) {
  return static_cast<size_t>(32 * J) * (1 + 2 * kRowWarps) * sizeof(float2);
}

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}

// out[i] = sum over g < G of part[g * n + i], n a multiple of 4 (n4 = n / 4
// float4 columns).  A block of 256 threads covers four float4 columns (16
// floats) with 64 row strides: thread (c, r) adds rows r, r + 64, ... into four
// accumulators (one per row stride of a 256-row pass, so four loads are in
// flight), adds them in a fixed order, and the 64 row strides are then added
// by a fixed tree in shared memory (deterministic for a given G).  n / 16
// blocks keep every SM busy where one block of 32 columns per 32 floats left
// most of them idle for the G ~ 1000 partial rows of a backward kernel.
__global__ void __launch_bounds__(256) partial_reduce_kernel(const float4* __restrict__ part, int G,
                                                             int64_t n4, float4* __restrict__ out) {
  __shared__ float4 red[64][4];
  const int c = threadIdx.x & 3, r = threadIdx.x >> 2;
  const int64_t i = blockIdx.x * 4LL + c;
  float4 a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (i < n4) {
    int g = r;
    for (; g + 192 < G; g += 256)
#pragma unroll
      for (int k = 0; k < 4; ++k) add4(a[k], part[static_cast<int64_t>(g + 64 * k) * n4 + i]);
    // fewer than four strides left (g + 192 >= G)
    if (g < G) add4(a[0], part[static_cast<int64_t>(g) * n4 + i]);
    if (g + 64 < G) add4(a[1], part[static_cast<int64_t>(g + 64) * n4 + i]);
    if (g + 128 < G) add4(a[2], part[static_cast<int64_t>(g + 128) * n4 + i]);
  }
  add4(a[0], a[1]);
  add4(a[2], a[3]);
  add4(a[0], a[2]);
  red[r][c] = a[0];
  __syncthreads();
#pragma unroll
  for (int h = 32; h > 0; h >>= 1) {
    if (r < h) {
      float4 t = red[r][c];
      add4(t, red[r + h][c]);
      red[r][c] = t;
    }
    __syncthreads();
  }
  if (r == 0 && i < n4) out[i] = red[0][c];
}

// ---------------------------------------------------------------------------
// host side

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int64_t B, int64_t T, int64_t C) {
  if (B < 0 || T < 0) return 1;              // CAMOE_ERR_INVALID_ARG
  if (C < 64 || C > 2048 || C % 64 != 0) return 2;  // CAMOE_ERR_UNSUPPORTED
  return 0;
}

// CTAs to launch: as many as fit on the device at once (CTAs of `threads`,
// C/8 by default),
// at most one per work item and kMaxGrid
template <typename K>
int grid_for(K kernel, const Shape& S, size_t smem = 0, int threads = 0) {
  if (threads == 0) threads = static_cast<int>(S.C / V);
  // launches above the default 48 KiB of dynamic shared memory need the opt-in
  if (smem > (48u << 10))
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
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

// n is k * C, a multiple of 64; part (the workspace) and out are 16-byte aligned
int reduce(const float* part, int G, int64_t n, float* out, cudaStream_t st) {
  const int64_t n4 = n / 4, blocks = (n4 + 3) / 4;
  partial_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      reinterpret_cast<const float4*>(part), G, n4, reinterpret_cast<float4*>(out));
  return status(cudaGetLastError());
}

// f(std::integral_constant<int, J>) for J = C / 64 in 1..16 (C <= 1024); false
// for wider rows, which the C/8-thread kernels take
template <typename F>
bool with_pairs(int64_t C, F&& f) {
  switch (C / 64) {
#define CAMOE_TM_PAIRS(J) \
    case J:               \
      f(std::integral_constant<int, J>{}); \
      return true;
    CAMOE_TM_PAIRS(1) CAMOE_TM_PAIRS(2) CAMOE_TM_PAIRS(3) CAMOE_TM_PAIRS(4)
    CAMOE_TM_PAIRS(5) CAMOE_TM_PAIRS(6) CAMOE_TM_PAIRS(7) CAMOE_TM_PAIRS(8)
    CAMOE_TM_PAIRS(9) CAMOE_TM_PAIRS(10) CAMOE_TM_PAIRS(11) CAMOE_TM_PAIRS(12)
    CAMOE_TM_PAIRS(13) CAMOE_TM_PAIRS(14) CAMOE_TM_PAIRS(15) CAMOE_TM_PAIRS(16)
#undef CAMOE_TM_PAIRS
    default:
      return false;
  }
}

}  // namespace tm

unsigned int tm_timeouts() {  // the bounded waits of this file's ring kernel
  unsigned int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_wkv7_timeouts, sizeof(n)) != cudaSuccess) return ~0u;
  return n;
}
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
  return camoe_tm_mix_fwd_prev(x, x_dtype, nullptr, mix, out, B, T, C, stream);
}

int camoe_tm_mix_fwd_prev(const void* x, int x_dtype, const void* x_prev, const float* mix,
                          void* const* out, int64_t B, int64_t T, int64_t C, void* stream) {
  if (out == nullptr) return 1;
  int st = precheck(B, T, C, {x, mix, out[0], out[1], out[2], out[3], out[4], out[5]}, {x_prev});
  if (st != 0) return st < 0 ? 0 : st;
  if (x_dtype != 0 && x_dtype != 1) return 2;
  const Shape S = make_shape(B, T, C);
  camoe::tm::Out6 o;
  for (int m = 0; m < 6; ++m) o.p[m] = static_cast<bf16*>(out[m]);
  const int G = x_dtype == 0 ? camoe::tm::grid_for(camoe::tm::mix_fwd_kernel<bf16>, S)
                             : camoe::tm::grid_for(camoe::tm::mix_fwd_kernel<float>, S);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == 0)
    camoe::tm::mix_fwd_kernel<bf16><<<G, static_cast<unsigned>(C / camoe::tm::V), 0, s>>>(
        static_cast<const bf16*>(x), static_cast<const bf16*>(x_prev), mix, o, S);
  else
    camoe::tm::mix_fwd_kernel<float><<<G, static_cast<unsigned>(C / camoe::tm::V), 0, s>>>(
        static_cast<const float*>(x), static_cast<const float*>(x_prev), mix, o, S);
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
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == 0 && C <= 1024) {  // rows streamed through shared memory
    const int threads = static_cast<int>(C / 2) + 32;
    const size_t smem = camoe::tm::ring_smem(C);
    const int G = camoe::tm::grid_for(camoe::tm::mix_bwd_ring_kernel, S, smem, threads);
    camoe::tm::mix_bwd_ring_kernel<<<G, threads, smem, s>>>(
        static_cast<const bf16*>(x), mix, d, static_cast<bf16*>(dx), part, S);
    if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
    return camoe::tm::reduce(part, G, 6 * C, dmix, s);
  }
  const int threads = static_cast<int>(C / 2);  // two columns per thread
  const size_t smem = 6 * static_cast<size_t>(C) * sizeof(float);  // the mixes, <= 48 KiB
  const int G = x_dtype == 0 ? camoe::tm::grid_for(camoe::tm::mix_bwd_kernel<bf16>, S, smem, threads)
                             : camoe::tm::grid_for(camoe::tm::mix_bwd_kernel<float>, S, smem, threads);
  if (x_dtype == 0)
    camoe::tm::mix_bwd_kernel<bf16><<<G, threads, smem, s>>>(
        static_cast<const bf16*>(x), mix, d, static_cast<bf16*>(dx), part, S);
  else
    camoe::tm::mix_bwd_kernel<float><<<G, threads, smem, s>>>(
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
  const int threads = static_cast<int>(C / 2);  // two columns per thread
  camoe::tm::prep_fwd_kernel<<<camoe::tm::grid_for(camoe::tm::prep_fwd_kernel, S, 0, threads),
                               threads, 0,
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
  const int threads = static_cast<int>(C / 2);  // two columns per thread
  const int G = camoe::tm::grid_for(camoe::tm::prep_bwd_kernel, S, 0, threads);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  camoe::tm::prep_bwd_kernel<<<G, threads, 0, s>>>(p, part, S);
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
  camoe::tm::post_fwd_kernel<<<camoe::tm::grid_for(camoe::tm::post_fwd_kernel, S), static_cast<unsigned>(C / camoe::tm::V), 0,
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
  camoe::tm::post_bwd_kernel<<<G, static_cast<unsigned>(C / camoe::tm::V), 0, s>>>(p, q, part, S);
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 3 * C, dparams, s);
}

int camoe_tm_lnsa_fwd(const float* sa, const float* weight, const float* bias, float* out,
                      int64_t B, int64_t T, int64_t C, void* stream) {
  int st = precheck(B, T, C, {sa, weight, bias, out}, {});
  if (st != 0) return st < 0 ? 0 : st;
  const Shape S = make_shape(B, T, C);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool rows = camoe::tm::with_pairs(C, [&](auto pairs) {
    constexpr int J = decltype(pairs)::value;
    const auto k = camoe::tm::lnsa_fwd_rows_kernel<J>;
    const int G = camoe::tm::grid_for(k, S, 0, 32 * camoe::tm::kRowWarps);
    k<<<G, 32 * camoe::tm::kRowWarps, 0, s>>>(sa, weight, bias, out, B * T);
  });
  if (!rows)
    camoe::tm::lnsa_fwd_kernel<<<camoe::tm::grid_for(camoe::tm::lnsa_fwd_kernel, S),
                                 static_cast<unsigned>(C / camoe::tm::V), 0, s>>>(sa, weight, bias, out, S);
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
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int G = 0;
  const bool rows = camoe::tm::with_pairs(C, [&](auto pairs) {
    constexpr int J = decltype(pairs)::value;
    const auto k = camoe::tm::lnsa_bwd_rows_kernel<J>;
    const size_t smem = camoe::tm::lnsa_rows_smem(J);
    G = camoe::tm::grid_for(k, S, smem, 32 * camoe::tm::kRowWarps);
    k<<<G, 32 * camoe::tm::kRowWarps, smem, s>>>(dout, sa, weight, dsa, part, B * T);
  });
  if (!rows) {
    G = camoe::tm::grid_for(camoe::tm::lnsa_bwd_kernel, S);
    camoe::tm::lnsa_bwd_kernel<<<G, static_cast<unsigned>(C / camoe::tm::V), 0, s>>>(dout, sa, weight, dsa, part, S);
  }
  if ((st = camoe::tm::status(cudaGetLastError())) != 0) return st;
  return camoe::tm::reduce(part, G, 2 * C, dparams, s);
}

}  // extern "C"
