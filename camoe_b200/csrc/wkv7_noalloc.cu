// Allocation-free forward + backward of the WKV-7 ClampW operator.
//
// Who needs it: hosts that hand this library device buffers they own but
// cannot, or must not, create device allocations themselves — an FFI/JNI host
// whose process memory is managed by another runtime's pooled allocator (a
// cudaMalloc behind that pool's back breaks its accounting and its memory
// caps), and latency-critical training loops where cudaMalloc/cudaFree would
// synchronise the device in the middle of a step.  Such callers still pass
// every input and output; only the state checkpoint, which a forward normally
// writes into a caller-allocated buffer for the backward, lives here in a
// fixed device array owned by the library.
//
// The scratch is a file-scope __device__ array of CAMOE_WKV7_NOALLOC_SCRATCH_BYTES
// (64 MiB): every GPU that loads the library holds it until the process exits.
// A call first validates its arguments (including that the checkpoint of the
// problem fits the array; otherwise CAMOE_ERR_WORKSPACE), then, on its first
// call on a device, looks up the array's device address with
// cudaGetSymbolAddress while that device is current (make that first call
// before any stream capture; the address is kept for the life of the process,
// so it is stale after a cudaDeviceReset of that device), then launches the
// existing forward and backward kernels on `stream` with the array as their
// checkpoint.
//
// The array is shared by every call and keeps the last call's contents.
// Nothing in it needs to start at zero: the forward writes every checkpoint
// record that the backward of the same call reads, and the backward writes
// its workspace records before reading them.  Calls whose work overlaps
// on the GPU (different streams, or several host threads) race on the array.
#include <mutex>

#include "camoe_wkv7.h"
#include "wkv7_common.cuh"

namespace camoe {
void set_last_cuda_error(int e);
namespace scan {
template <typename Tin>
cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream);
template <typename Tin>
cudaError_t launch_bwd(const BwdArgs& p, cudaStream_t stream);
}  // namespace scan
namespace chunked {
cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream);
cudaError_t launch_bwd(const BwdArgs& p, void* work, cudaStream_t stream);
}  // namespace chunked
}  // namespace camoe

namespace {

static __device__ __align__(256) unsigned char g_ckpt_scratch[CAMOE_WKV7_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 128;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_ckpt_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    camoe::set_last_cuda_error(static_cast<int>(e));
    return CAMOE_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return CAMOE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ckpt_scratch);
    if (e != cudaSuccess || p == nullptr) {
      camoe::set_last_cuda_error(static_cast<int>(e));
      return CAMOE_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return CAMOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int camoe_wkv7_fwd_bwd_noalloc(
    const void* r, const void* w, const void* k, const void* v, const void* a, const void* b,
    const void* dy, const float* dsa, void* y, float* sa, void* dr, void* dw, void* dk,
    void* dv, void* da, void* db, int64_t B, int64_t T, int64_t H_total, int64_t h0,
    int64_t h_count, int N, int dtype, int algo, void* stream) {
  if (N != camoe::kN) return CAMOE_ERR_UNSUPPORTED;
  if (B < 0 || T < 0 || H_total < 0 || h0 < 0 || h_count < 0 || h0 + h_count > H_total ||
      B * h_count > 0x7fffffffLL)
    return CAMOE_ERR_INVALID_ARG;
  if (dtype != CAMOE_DTYPE_BF16 && dtype != CAMOE_DTYPE_FP32) return CAMOE_ERR_UNSUPPORTED;
  int al = algo;
  if (al == CAMOE_ALGO_AUTO) al = dtype == CAMOE_DTYPE_BF16 ? CAMOE_ALGO_CHUNKED : CAMOE_ALGO_SCAN;
  if (al != CAMOE_ALGO_SCAN && al != CAMOE_ALGO_CHUNKED) return CAMOE_ERR_UNSUPPORTED;
  if (al == CAMOE_ALGO_CHUNKED && dtype != CAMOE_DTYPE_BF16) return CAMOE_ERR_UNSUPPORTED;
  if (B * h_count == 0 || T == 0) return CAMOE_OK;
  const void* ptrs[] = {r, w, k, v, a, b, dy, y, sa, dr, dw, dk, dv, da, db};
  for (const void* p : ptrs) {
    if (p == nullptr) return CAMOE_ERR_INVALID_ARG;
    if (!aligned16(p)) return CAMOE_ERR_ALIGNMENT;
  }
  if (dsa != nullptr && !aligned16(dsa)) return CAMOE_ERR_ALIGNMENT;
  // Every algorithm needs more than 4 KiB per chain and 16-step chunk, so a
  // problem with more chain-chunks than the scratch holds 4 KiB pieces cannot
  // fit.  Rejecting those first keeps the byte counts below from overflowing
  // (B * h_count < 2^31 and nchunk <= 2^14 / chains bound every product).
  const int64_t chains = B * h_count;
  const int64_t nchunk = T / camoe::kChunk + (T % camoe::kChunk != 0 ? 1 : 0);
  if (nchunk > static_cast<int64_t>(CAMOE_WKV7_NOALLOC_SCRATCH_BYTES / 4096) / chains)
    return CAMOE_ERR_WORKSPACE;
  // the scratch holds the checkpoint, then the backward workspace
  const size_t need = camoe_wkv7_ckpt_bytes(B, T, h_count, N, dtype, al);
  const size_t wneed = camoe_wkv7_work_bytes(B, T, h_count, N, dtype, al);
  const size_t wofs = (need + 255) & ~static_cast<size_t>(255);
  if (wofs + wneed > CAMOE_WKV7_NOALLOC_SCRATCH_BYTES) return CAMOE_ERR_WORKSPACE;

  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != CAMOE_OK) return st;

  const camoe::Geom g{B, T, H_total, h0, h_count, (T + camoe::kChunk - 1) / camoe::kChunk};
  camoe::FwdArgs f;
  f.r = r; f.w = w; f.k = k; f.v = v; f.a = a; f.b = b;
  f.y = y; f.sa = sa; f.ckpt = static_cast<float*>(scratch); f.g = g;
  camoe::BwdArgs p;
  p.r = r; p.w = w; p.k = k; p.v = v; p.a = a; p.b = b; p.dy = dy; p.dsa = dsa;
  p.ckpt = static_cast<const float*>(scratch);
  p.dr = dr; p.dw = dw; p.dk = dk; p.dv = dv; p.da = da; p.db = db; p.g = g;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (al == CAMOE_ALGO_CHUNKED) {
    e = camoe::chunked::launch_fwd(f, s);
    if (e == cudaSuccess) e = camoe::chunked::launch_bwd(p, static_cast<char*>(scratch) + wofs, s);
  } else if (dtype == CAMOE_DTYPE_BF16) {
    e = camoe::scan::launch_fwd<camoe::bf16>(f, s);
    if (e == cudaSuccess) e = camoe::scan::launch_bwd<camoe::bf16>(p, s);
  } else {
    e = camoe::scan::launch_fwd<float>(f, s);
    if (e == cudaSuccess) e = camoe::scan::launch_bwd<float>(p, s);
  }
  if (e != cudaSuccess) {
    camoe::set_last_cuda_error(static_cast<int>(e));
    return CAMOE_ERR_CUDA;
  }
  return CAMOE_OK;
}
