// Joins the time segments of a chain cut into P pieces (the time-segmented
// long-context path, camoe_b200/segmented.py).  The WKV-7 state map of one
// segment is affine, S_end = S_start A + C, with A the segment's transition
// (its final state from an identity start and v = 0) and C its final state
// from a zero start.  Given A and C of every segment, the start states follow
// from S_0 by P - 1 64x64 products, S_g = S_{g-1} A_{g-1} + C_{g-1}; the
// backward runs the same chain the other way on gradients,
// E_{g-1} = E_g A_g^T + D_g, with E_g the gradient of segment g's final state
// and D_g its start-state gradient when E_g = 0.
//
// Rows of the running matrix evolve independently (row i of S_g is row i of
// S_{g-1} times A, plus row i of C), so each chain is split over four CTAs of
// 16 rows that walk the P segments; the rows and the transition stay in shared
// memory (fp32, rows padded to 65 floats so that the row and column reads of
// the product are free of bank conflicts).
#include "camoe_wkv7.h"
#include "wkv7_common.cuh"

namespace camoe {
void set_last_cuda_error(int e);

namespace seg {

constexpr int kThreads = 256;  // 16 rows x 16 column groups, 4 outputs per thread
constexpr int kRows = 16;      // rows of the running matrix per CTA
constexpr int kSplit = kN / kRows;
constexpr int kLd = kN + 1;

__global__ void __launch_bounds__(kThreads) chain_kernel(float* states, const float* trans,
                                                        const float* local, int64_t P, int64_t H,
                                                        int64_t h0, int64_t hc, int backward) {
  __shared__ float run[kRows * kLd];  // this CTA's rows of the running state (or gradient)
  __shared__ float tm[kN * kLd];      // A (forward) or A^T (backward) of the current segment
  const int64_t chain = blockIdx.x / kSplit;
  const int i0 = kRows * static_cast<int>(blockIdx.x % kSplit);
  const int64_t b = chain / hc, h = h0 + chain % hc;
  const int tid = threadIdx.x, il = tid >> 4, jb = tid & 15;  // row i0 + il, columns jb + 16 m
  auto block = [&](int64_t g) { return ((b * P + g) * H + h) * kN * kN; };

  const int64_t first = backward ? P - 1 : 0;
  for (int e = tid; e < kRows * kN; e += kThreads)
    run[(e >> 6) * kLd + (e & 63)] = states[block(first) + i0 * kN + e];
  for (int64_t step = 1; step < P; ++step) {
    // forward: S_g from S_{g-1}, A_{g-1}, C_{g-1}; backward: E_{g-1} from E_g, A_g, D_g
    const int64_t src = backward ? P - step : step - 1;   // segment whose A and C / D are used
    const int64_t dst = backward ? P - 1 - step : step;   // segment whose start (end) is written
    const float* A = trans + block(src);
    for (int e = tid; e < kN * kN; e += kThreads) {
      const int r = e >> 6, c = e & 63;
      if (backward)
        tm[c * kLd + r] = A[e];  // tm[k][j] = A[j][k]
      else
        tm[r * kLd + c] = A[e];
    }
    __syncthreads();
    float acc[4];
    const float* loc = local + block(src) + (i0 + il) * kN;
#pragma unroll
    for (int m = 0; m < 4; ++m) acc[m] = loc[jb + 16 * m];
#pragma unroll 8
    for (int k = 0; k < kN; ++k) {
      const float s = run[il * kLd + k];
#pragma unroll
      for (int m = 0; m < 4; ++m) acc[m] = fmaf(s, tm[k * kLd + jb + 16 * m], acc[m]);
    }
    __syncthreads();  // every read of run and tm done
    float* out = states + block(dst) + (i0 + il) * kN;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      run[il * kLd + jb + 16 * m] = acc[m];
      out[jb + 16 * m] = acc[m];
    }
    __syncthreads();
  }
}

}  // namespace seg
}  // namespace camoe

extern "C" {

int camoe_wkv7_seg_chain(float* states, const float* trans, const float* local, int64_t B,
                         int64_t P, int64_t H_total, int64_t h0, int64_t h_count, int backward,
                         void* stream) {
  if (B < 0 || P < 1 || H_total < 0 || h0 < 0 || h_count < 0 || h0 + h_count > H_total)
    return CAMOE_ERR_INVALID_ARG;
  if (backward != 0 && backward != 1) return CAMOE_ERR_INVALID_ARG;
  if (B * h_count == 0 || P == 1) return CAMOE_OK;
  if (B * h_count * camoe::seg::kSplit > 0x7fffffffLL) return CAMOE_ERR_INVALID_ARG;
  const void* ptrs[] = {states, trans, local};
  for (const void* p : ptrs) {
    if (p == nullptr) return CAMOE_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return CAMOE_ERR_ALIGNMENT;
  }
  camoe::seg::chain_kernel<<<static_cast<unsigned>(B * h_count * camoe::seg::kSplit),
                             camoe::seg::kThreads, 0,
                             static_cast<cudaStream_t>(stream)>>>(states, trans, local, P, H_total,
                                                                  h0, h_count, backward);
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return CAMOE_OK;
  camoe::set_last_cuda_error(static_cast<int>(e));
  return CAMOE_ERR_CUDA;
}

}  // extern "C"
