// Shared definitions of the WKV-7 ClampW kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace camoe {

constexpr int kN = 64;      // head size (state is kN x kN)
constexpr int kChunk = 16;  // steps per chunk / checkpoint interval
// -exp(-1/2): the ClampW decay is w = exp(kWScale * sigmoid(w_in)),
// camoe/cuda/rwkv7_clampw.cu:16,42.
constexpr float kWScale = -0.6065306597126334f;

// Decay transforms w = exp(lw(w_in)) of the two reference ops:
//   ClampW             lw = -e^{-1/2} sigmoid(w_in)   camoe/cuda/rwkv7_clampw.cu:42
//   wind_backstepping  lw = -exp(w_in)                camoe/cuda/wkv7_cuda.cu:21,66-67
enum : int { kDecayClampW = 0, kDecayWind = 1 };

__device__ __forceinline__ float log_decay(float x, int kind) {
  return kind == kDecayWind ? -expf(x) : kWScale / (1.0f + expf(-x));
}
// fast-math form, for the chunked kernels (bf16 operands)
__device__ __forceinline__ float log_decay_fast(float x, int kind) {
  return kind == kDecayWind ? -__expf(x) : kWScale * __fdividef(1.0f, 1.0f + __expf(-x));
}
// d lw / d w_in, written in terms of lw: ClampW kWScale s (1 - s) with
// s = lw / kWScale; wind -exp(w_in) = lw
__device__ __forceinline__ float dlog_decay(float lw, int kind) {
  return kind == kDecayWind ? lw : lw * (1.0f - lw * (1.0f / kWScale));
}

using bf16 = __nv_bfloat16;

// Geometry of one call: heads [h0, h0 + hc) of [B, T, H, kN] arrays, and
// the decay transform (kDecayClampW or kDecayWind) the call applies.
struct Geom {
  int64_t B, T, H, h0, hc;
  int64_t nchunk;  // ceil(T / kChunk)
  int decay = kDecayClampW;
  __host__ __device__ int64_t chains() const { return B * hc; }
  // offset of element (t, i) of chain `ch`
  __device__ __forceinline__ int64_t off(int64_t ch, int64_t t, int i) const {
    const int64_t b = ch / hc, h = h0 + ch % hc;
    return ((b * T + t) * H + h) * kN + i;
  }
  // offset of element (0, 0) of chain `ch`; element (t, i) is at base + t * tstride() + i
  __device__ __forceinline__ int64_t base(int64_t ch) const {
    const int64_t b = ch / hc, h = h0 + ch % hc;
    return (b * T * H + h) * kN;
  }
  // stride between consecutive time steps of one chain, in elements
  __host__ __device__ int64_t tstride() const { return H * kN; }
  // offset of element (0, 0) of chain `ch`'s N x N state in a [B, H, N, N] array
  __host__ __device__ int64_t state_off(int64_t ch) const {
    return ((ch / hc) * H + h0 + ch % hc) * kN * kN;
  }
};

// Position of a grid-stride walk over the (chain, chunk) items of a call,
// item = ch * nchunk + c with ch = b * hc + hm.  The divisions happen once, in
// init(); next() advances by the stride with one carry per level, so a loop
// over items pays a few integer adds per item instead of 64-bit divisions.
struct ItemWalk {
  int64_t ch, c, b, hm;      // the current item
  int64_t dch, dc, db, dhm;  // the stride in the same terms
  __device__ __forceinline__ void init(const Geom& g, int64_t item, int64_t stride) {
    ch = item / g.nchunk;
    c = item - ch * g.nchunk;
    b = ch / g.hc;
    hm = ch - b * g.hc;
    dch = stride / g.nchunk;
    dc = stride - dch * g.nchunk;
    db = dch / g.hc;
    dhm = dch - db * g.hc;
  }
  __device__ __forceinline__ void next(const Geom& g) {
    c += dc;
    const int64_t carry = c >= g.nchunk ? 1 : 0;  // c, dc < nchunk: at most one wrap
    c -= carry * g.nchunk;
    ch += dch + carry;
    hm += dhm + carry;
    b += db;
    if (hm >= g.hc) {  // hm, dhm < hc: at most one wrap
      hm -= g.hc;
      b += 1;
    }
  }
  __device__ __forceinline__ int head(const Geom& g) const { return static_cast<int>(g.h0 + hm); }
  // offset of element (0, 0) of the current chain, as Geom::base
  __device__ __forceinline__ int64_t base(const Geom& g) const { return (b * g.T * g.H + g.h0 + hm) * kN; }
};

struct FwdArgs {
  const void *r, *w, *k, *v, *a, *b;
  void* y;
  float* sa;
  float* ckpt;  // may be null
  Geom g;
  // start state (null = zero) and final state (null = not stored) of every
  // chain, fp32 [B, H, N, N] with element ((b*H + h)*N + i)*N + j = S[i][j];
  // sT may equal s0 (each element is read before it is overwritten, by the
  // same thread).  The inference forward (ckpt == null) and the carried
  // training forward take them.
  const float* s0 = nullptr;
  float* sT = nullptr;
  // inference forward only: with a workspace the chunked path runs as two
  // kernels (key-side records into `work`, then the value pass), else fused
  void* work = nullptr;
  // chunked training forward: the key-side records in ckpt were written by an
  // earlier forward of the same r, w, k, a, b and geometry; run the value pass only
  bool records_ready = false;
};

struct BwdArgs {
  const void *r, *w, *k, *v, *a, *b, *dy;
  const float* dsa;   // may be null
  const float* ckpt;  // written by the matching forward
  void *dr, *dw, *dk, *dv, *da, *db;
  Geom g;
  // a sequence carried in from a previous call (T a multiple of kChunk): the
  // start state the forward was given (null = zero), the gradient of the final
  // state (null = zero), and where to write the gradient of the start state
  // (null = not wanted); [B, H, N, N] fp32 like FwdArgs::s0
  const float* s0 = nullptr;
  const float* dsT = nullptr;
  float* ds0 = nullptr;
};

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(bf16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ bf16 from_f32<bf16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// ---- cp.async (16-byte, L2-only) helpers ----------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int n = pred ? 16 : 0;  // n == 0 zero-fills the destination
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

}  // namespace camoe
