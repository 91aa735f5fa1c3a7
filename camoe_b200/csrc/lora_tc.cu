// Weight gradients of the time mix's LoRA products on the 5th-generation
// tensor cores (tcgen05), declared in include/camoe_timemix.h.
//
// The reference gets these from autograd through cuBLAS (camoe/backbone.py:
// 326-341: x @ w1 and h @ w2 per LoRA, four LoRAs per layer): with R = B T
// rows, C = 1024 and a rank D of 64 or 160,
//   T[c][d] = sum over r of big[r][c] thin[r][d]
// (big = x, thin = dh for w1's [C][D] gradient; big = dy, thin = h for w2's
// [D][C] one).  The reduction runs over all R rows and the output is small, a
// shape cuBLAS runs at a fifth of HBM bandwidth with a few warps per SM bound
// by dependent warp-level MMA latency.  Here one thread per CTA issues the
// products (tcgen05.mma kind::f16, bf16 operands, fp32 accumulator in tensor
// memory):
//   * a CTA takes 128 columns of big (the MMA's M, one TMEM lane each) and all
//     D columns of thin (the MMA's N, D rounded up to a multiple of 64 with
//     zero columns), for one slice of the rows;
//   * a producer thread streams the slice's rows through a ring of stages by
//     TMA, 64 rows per stage: big as two and thin as N/64 boxes of 64 columns,
//     each landing as 64 rows of 128 bytes with the 128-byte swizzle, the
//     canonical MN-major layout the MMA reads (both operands are stored with
//     M or N contiguous);
//   * an MMA thread issues four K = 16 products per stage and commits each
//     stage back to the producer through an mbarrier;
//   * all four warps then read the accumulator rows of their TMEM lane
//     quarter (tcgen05.ld) and write the slice's fp32 tile to a row of
//     partial sums, which slice_sum_kernel adds in a fixed order
//     (deterministic).
// Every mbarrier wait is bounded (wkv7_sync.cuh); a wait that runs out is
// counted in camoe_wkv7_device_errors().
#include "camoe_timemix.h"
#include "wkv7_common.cuh"
#include "wkv7_sync.cuh"
#include "wkv7_tma.cuh"

namespace camoe {
void set_last_cuda_error(int e);  // wkv7_capi.cu
namespace tm {
int status(cudaError_t e);  // timemix.cu
}  // namespace tm

namespace lora {

constexpr int kM = 128;      // big columns per CTA: the MMA's M
constexpr int kKR = 64;      // rows per stage: four K = 16 products
constexpr int kThreads = 128;
constexpr int kSlices = 16;  // row slices at most (partial-sum rows)
constexpr uint32_t kAtomBytes = kKR * 128;  // one 64-column box of a stage

// stages of the ring: four (64 rows each; with at most one CTA per SM at the
// layer's shapes, the ring is what keeps loads in flight)
template <int NA>
__host__ __device__ constexpr int stages() { return 4; }

template <int NA>  // N = 64 NA
struct alignas(1024) TcSmem {
  static constexpr int S = stages<NA>();
  bf16 a[S][2][kKR * 64];   // big: two boxes of 64 columns per stage
  bf16 b[S][NA][kKR * 64];  // thin: NA boxes
  uint64_t full[S], empty[S], done;
  uint32_t tmem;
};

// Shared-memory matrix descriptor of an MN-major operand with the 128-byte
// swizzle: start address, leading byte offset = bytes between 64-element
// blocks along M (or N), stride byte offset = 1024 bytes between groups of 8
// rows along K, descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>(1024u >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), bf16
// A and B (bits 7-9, 10-12 = 1), both MN-major (bits 15, 16), N / 8 at bit 17,
// M / 16 at bit 24.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc,
                                       bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   sm_addr(bar))
               : "memory");
}
// 16 consecutive accumulator columns of this thread's TMEM lane
__device__ __forceinline__ void tc_ld16(uint32_t (&v)[16], uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int NA>
__global__ void __launch_bounds__(kThreads) wgrad_tc_kernel(const __grid_constant__ CUtensorMap mbig,
                                                            const __grid_constant__ CUtensorMap mthin,
                                                            float* __restrict__ part, int64_t R,
                                                            int64_t C, int D, int64_t slice_rows,
                                                            int out_cd) {
  constexpr int N = 64 * NA, S = stages<NA>();
  constexpr uint32_t kCols = N <= 64 ? 64 : (N <= 128 ? 128 : 256);  // TMEM columns: a power of two
  extern __shared__ __align__(128) unsigned char tc_raw[];
  TcSmem<NA>& sm =
      *reinterpret_cast<TcSmem<NA>*>(tc_raw + ((1024u - (sm_addr(tc_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kM;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * slice_rows;
  const int64_t r1 = r0 + slice_rows < R ? r0 + slice_rows : R;
  const int nch = r1 > r0 ? static_cast<int>((r1 - r0 + kKR - 1) / kKR) : 0;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.done, 1);
    mbar_fence_init();
  }
  if (warp == 0) {  // the whole warp allocates the accumulator's columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sm_addr(&sm.tmem)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;

  if (warp == 0 && lane == 0) {  // producer: the slice's rows, stage by stage
    for (int i = 0; i < nch; ++i) {
      const int s = i % S;
      if (i >= S && !mbar_wait(&sm.empty[s], static_cast<uint32_t>((i / S - 1) & 1))) break;
      mbar_arrive_expect_tx(&sm.full[s], (2 + NA) * kAtomBytes);
      const int row = static_cast<int>(r0 + static_cast<int64_t>(i) * kKR);
      tma::load_2d(sm.a[s][0], &mbig, static_cast<int>(c0), row, &sm.full[s]);
      tma::load_2d(sm.a[s][1], &mbig, static_cast<int>(c0) + 64, row, &sm.full[s]);
#pragma unroll
      for (int j = 0; j < NA; ++j) tma::load_2d(sm.b[s][j], &mthin, 64 * j, row, &sm.full[s]);
    }
  } else if (warp == 1 && lane == 0) {  // MMA issue
    constexpr uint32_t idesc = instr_desc(kM, N);
    bool issued = false;
    for (int i = 0; i < nch; ++i) {
      const int s = i % S;
      if (!mbar_wait(&sm.full[s], static_cast<uint32_t>((i / S) & 1))) break;
      tc_fence_after();
      const uint32_t a0 = sm_addr(sm.a[s][0]), b0 = sm_addr(sm.b[s][0]);
#pragma unroll
      for (int kk = 0; kk < kKR / 16; ++kk)  // 16 rows = 2048 bytes of each box
        tc_mma(tmem, smem_desc(a0 + 2048u * kk, kAtomBytes), smem_desc(b0 + 2048u * kk, kAtomBytes),
               idesc, i > 0 || kk > 0);
      tc_commit(&sm.empty[s]);  // the stage is free once these products are done
      issued = true;
    }
    if (issued)
      tc_commit(&sm.done);
    else
      mbar_arrive(&sm.done);
  }
  __syncwarp();

  // epilogue: warp w holds accumulator rows 32w..32w+31 (TMEM lanes), one per thread
  const bool ok = mbar_wait(&sm.done, 0);
  tc_fence_after();
  const bool have = ok && nch > 0;
  float* pp = part + static_cast<int64_t>(blockIdx.y) * C * D;
  const int64_t c = c0 + 32 * warp + lane;
  for (int col = 0; col < D; col += 16) {  // D is a multiple of 32
    uint32_t v[16];
    if (have) {
      tc_ld16(v, tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(col));
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = 0u;
    }
    if (out_cd) {
      float4* dst = reinterpret_cast<float4*>(pp + c * D + col);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                             __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) pp[static_cast<int64_t>(col + e) * C + c] = __uint_as_float(v[e]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols)
                 : "memory");
}

// out[i] = sum over g < G of part[g n + i] in the order g = 0, 1, ..., one
// float4 column per thread: the few (<= kSlices) partial rows of this kernel
// need no cross-thread tree.
__global__ void __launch_bounds__(256) slice_sum_kernel(const float4* __restrict__ part, int G,
                                                        int64_t n4, float4* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n4) return;
  float4 t = part[i];
  for (int g = 1; g < G; ++g) {
    const float4 v = part[static_cast<int64_t>(g) * n4 + i];
    t.x += v.x;
    t.y += v.y;
    t.z += v.z;
    t.w += v.w;
  }
  out[i] = t;
}

inline int slices(int64_t R) {
  const int64_t chunks = (R + kKR - 1) / kKR;
  return static_cast<int>(chunks < kSlices ? (chunks < 1 ? 1 : chunks) : kSlices);
}

template <typename F>
bool with_boxes(int64_t D, F&& f) {  // f(integral_constant<NA>) with N = 64 NA >= D
  switch ((D + 63) / 64) {
    case 1: f(std::integral_constant<int, 1>{}); return true;
    case 2: f(std::integral_constant<int, 2>{}); return true;
    case 3: f(std::integral_constant<int, 3>{}); return true;
    case 4: f(std::integral_constant<int, 4>{}); return true;
    default: return false;
  }
}

}  // namespace lora

unsigned int lora_timeouts() {
  unsigned int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_wkv7_timeouts, sizeof(n)) != cudaSuccess) return ~0u;
  return n;
}

}  // namespace camoe

extern "C" {

size_t camoe_tm_lora_work_bytes(int64_t R, int64_t C, int64_t D) {
  if (R < 0 || C < 0 || D < 0) return 0;
  return static_cast<size_t>(camoe::lora::slices(R)) * static_cast<size_t>(C) *
         static_cast<size_t>(D) * sizeof(float);
}

int camoe_tm_lora_wgrad(const void* big, const void* thin, float* dw, int out_cd, void* work,
                        size_t work_bytes, int64_t R, int64_t C, int64_t D, void* stream) {
  using namespace camoe;
  if (R < 0 || (out_cd != 0 && out_cd != 1)) return 1;                       // CAMOE_ERR_INVALID_ARG
  if (C < 128 || C % 128 != 0 || D < 64 || D > 256 || D % 32 != 0) return 2;  // CAMOE_ERR_UNSUPPORTED
  if (R > (1ll << 31) - 1 || C > (1ll << 31) - 1) return 3;                   // CAMOE_ERR_SHAPE
  if (big == nullptr || thin == nullptr || dw == nullptr) return 1;
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(big) || !a16(thin) || !a16(dw)) return 4;  // CAMOE_ERR_ALIGNMENT
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (R == 0) return camoe::tm::status(cudaMemsetAsync(dw, 0, static_cast<size_t>(C * D) * sizeof(float), s));
  if (work == nullptr) return 1;
  if (!a16(work)) return 4;
  if (work_bytes < camoe_tm_lora_work_bytes(R, C, D)) return 5;  // CAMOE_ERR_WORKSPACE
  if (!tma::bind_context()) return camoe::tm::status(cudaErrorNoDevice);
  CUtensorMap mbig, mthin;
  if (!tma::encode_2d_sw128(&mbig, big, C, R, lora::kKR) ||
      !tma::encode_2d_sw128(&mthin, thin, D, R, lora::kKR))
    return camoe::tm::status(cudaErrorInvalidValue);
  const int S = lora::slices(R);
  const int64_t chunks = (R + lora::kKR - 1) / lora::kKR;
  const int64_t slice_rows = (chunks + S - 1) / S * lora::kKR;
  float* part = static_cast<float*>(work);
  int st = 0;
  lora::with_boxes(D, [&](auto boxes) {
    constexpr int NA = decltype(boxes)::value;
    const auto k = lora::wgrad_tc_kernel<NA>;
    const int smem = static_cast<int>(sizeof(lora::TcSmem<NA>)) + 1024;  // + alignment slack
    if ((st = camoe::tm::status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) != 0)
      return;
    k<<<dim3(static_cast<unsigned>(C / lora::kM), static_cast<unsigned>(S)), lora::kThreads, smem, s>>>(
        mbig, mthin, part, R, C, static_cast<int>(D), slice_rows, out_cd);
    st = camoe::tm::status(cudaGetLastError());
  });
  if (st != 0) return st;
  const int64_t n4 = C * D / 4;  // C D is a multiple of 4
  lora::slice_sum_kernel<<<static_cast<unsigned>((n4 + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const float4*>(part), S, n4, reinterpret_cast<float4*>(dw));
  return camoe::tm::status(cudaGetLastError());
}

}  // extern "C"
