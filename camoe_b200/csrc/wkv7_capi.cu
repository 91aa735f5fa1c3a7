// C ABI of the WKV-7 ClampW operator (declared in include/camoe_wkv7.h):
// argument validation, algorithm selection and kernel dispatch.  Nothing here
// allocates or synchronises; every launch goes to the caller's stream.
#include <initializer_list>

#include "camoe_wkv7.h"
#include "wkv7_common.cuh"

namespace camoe {
namespace scan {
template <typename Tin>
cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream);
template <typename Tin>
cudaError_t launch_bwd(const BwdArgs& p, cudaStream_t stream);
}  // namespace scan
unsigned int lora_timeouts();  // lora_tc.cu
unsigned int tm_timeouts();    // timemix.cu
namespace chunked {
unsigned int fwd_timeouts();
unsigned int bwd_timeouts();
cudaError_t fwd_test_hooks(long long wait_limit_cycles, int skip_pair);
cudaError_t bwd_test_hooks(long long wait_limit_cycles);
cudaError_t launch_fwd(const FwdArgs& p, cudaStream_t stream);
cudaError_t launch_bwd(const BwdArgs& p, void* work, cudaStream_t stream);
size_t ckpt_bytes(int64_t chains, int64_t T);
size_t work_bytes(int64_t chains, int64_t T);
size_t infer_bytes(int64_t chains, int64_t T);
}  // namespace chunked
}  // namespace camoe

namespace {

thread_local int g_last_cuda_error = 0;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// AUTO -> CHUNKED for bf16, SCAN for fp32; -1 for an invalid combination.
int resolve_algo(int dtype, int algo) {
  if (dtype != CAMOE_DTYPE_BF16 && dtype != CAMOE_DTYPE_FP32) return -1;
  if (algo == CAMOE_ALGO_AUTO) return dtype == CAMOE_DTYPE_BF16 ? CAMOE_ALGO_CHUNKED : CAMOE_ALGO_SCAN;
  if (algo == CAMOE_ALGO_SCAN) return algo;
  if (algo == CAMOE_ALGO_CHUNKED) return dtype == CAMOE_DTYPE_BF16 ? algo : -1;
  return -1;
}

// algorithm of a stateful forward: AUTO picks the decode-step kernel for T <= 16
int resolve_state_algo(int dtype, int algo, int64_t T) {
  const int al = resolve_algo(dtype, algo);
  if (al >= 0 && algo == CAMOE_ALGO_AUTO && T <= camoe::kChunk) return CAMOE_ALGO_SCAN;
  return al;
}

size_t required_ckpt(int64_t B, int64_t T, int64_t hc, int algo) {
  const int64_t chains = B * hc;
  if (algo == CAMOE_ALGO_CHUNKED) return camoe::chunked::ckpt_bytes(chains, T);
  const int64_t nchunk = (T + camoe::kChunk - 1) / camoe::kChunk;
  return static_cast<size_t>(chains * nchunk) * camoe::kN * camoe::kN * sizeof(float);
}

size_t required_work(int64_t B, int64_t T, int64_t hc, int algo) {
  return algo == CAMOE_ALGO_CHUNKED ? camoe::chunked::work_bytes(B * hc, T) : 0;
}

int check_geometry(int64_t B, int64_t T, int64_t H, int64_t h0, int64_t hc, int N) {
  if (N != camoe::kN) return CAMOE_ERR_UNSUPPORTED;
  if (B < 0 || T < 0 || H < 0 || h0 < 0 || hc < 0 || h0 + hc > H) return CAMOE_ERR_INVALID_ARG;
  if (B * hc > 0x7fffffffLL) return CAMOE_ERR_INVALID_ARG;  // grid size
  return CAMOE_OK;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return CAMOE_OK;
  g_last_cuda_error = static_cast<int>(e);
  return CAMOE_ERR_CUDA;
}

}  // namespace

namespace camoe {
// lets other translation units of the library report a CUDA error through
// camoe_wkv7_last_cuda_error()
void set_last_cuda_error(int e) { g_last_cuda_error = e; }
}  // namespace camoe

extern "C" {

int camoe_wkv7_version(void) { return 10100; }

const char* camoe_wkv7_strerror(int code) {
  switch (code) {
    case CAMOE_OK: return "ok";
    case CAMOE_ERR_INVALID_ARG: return "invalid argument (null pointer, negative size or head range outside H_total)";
    case CAMOE_ERR_UNSUPPORTED: return "unsupported configuration (N must be 64; CHUNKED needs bf16)";
    case CAMOE_ERR_SHAPE: return "unsupported shape";
    case CAMOE_ERR_ALIGNMENT: return "a pointer is not 16-byte aligned";
    case CAMOE_ERR_WORKSPACE: return "checkpoint buffer too small (see camoe_wkv7_ckpt_bytes)";
    case CAMOE_ERR_CUDA: return "CUDA launch failed (see camoe_wkv7_last_cuda_error)";
    default: return "unknown status code";
  }
}

int camoe_wkv7_last_cuda_error(void) { return g_last_cuda_error; }

unsigned int camoe_wkv7_device_errors(void) {
  const unsigned int a = camoe::chunked::fwd_timeouts(), b = camoe::chunked::bwd_timeouts();
  const unsigned int c = camoe::lora_timeouts(), d = camoe::tm_timeouts();
  if (a == ~0u || b == ~0u || c == ~0u || d == ~0u) return ~0u;
  return a + b + c + d;
}

int camoe_wkv7_test_hooks(long long wait_limit_cycles, int skip_pair) {
  // at most the kernels' default limit (kWaitLimitCycles of wkv7_sync.cuh)
  if (wait_limit_cycles < 1000 || wait_limit_cycles > 2000000000LL || skip_pair < -1)
    return CAMOE_ERR_INVALID_ARG;
  cudaError_t e = camoe::chunked::fwd_test_hooks(wait_limit_cycles, skip_pair);
  if (e == cudaSuccess) e = camoe::chunked::bwd_test_hooks(wait_limit_cycles);
  return cuda_status(e);
}

size_t camoe_wkv7_ckpt_bytes(int64_t B, int64_t T, int64_t h_count, int N, int dtype, int algo) {
  const int al = resolve_algo(dtype, algo);
  if (al < 0 || N != camoe::kN || B < 0 || T < 0 || h_count < 0) return 0;
  return required_ckpt(B, T, h_count, al);
}

size_t camoe_wkv7_work_bytes(int64_t B, int64_t T, int64_t h_count, int N, int dtype, int algo) {
  const int al = resolve_algo(dtype, algo);
  if (al < 0 || N != camoe::kN || B < 0 || T < 0 || h_count < 0) return 0;
  return required_work(B, T, h_count, al);
}

}  // extern "C"

namespace {

// the [B, H_total, N, N] state arrays of a call, when given, must be aligned
// and the sequence a whole number of chunks (a ragged last chunk would put
// the final state mid-chunk)
int check_carry(int64_t T, std::initializer_list<const void*> states) {
  bool any = false;
  for (const void* p : states) {
    if (p == nullptr) continue;
    any = true;
    if (!aligned16(p)) return CAMOE_ERR_ALIGNMENT;
  }
  if (any && T % camoe::kChunk != 0) return CAMOE_ERR_SHAPE;
  return CAMOE_OK;
}

int fwd_impl(const void* r, const void* w, const void* k, const void* v, const void* a,
             const void* b, void* y, float* sa, void* ckpt, size_t ckpt_bytes, int64_t B,
             int64_t T, int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
             void* stream, int decay, const float* s0 = nullptr, float* sT = nullptr,
             bool records_ready = false) {
  int st = check_geometry(B, T, H_total, h0, h_count, N);
  if (st != CAMOE_OK) return st;
  const int al = resolve_algo(dtype, algo);
  if (al < 0) return CAMOE_ERR_UNSUPPORTED;
  if (B * h_count == 0 || T == 0) return CAMOE_OK;
  const void* ptrs[] = {r, w, k, v, a, b, y, sa};
  for (const void* p : ptrs) {
    if (p == nullptr) return CAMOE_ERR_INVALID_ARG;
    if (!aligned16(p)) return CAMOE_ERR_ALIGNMENT;
  }
  if (ckpt != nullptr) {
    if (!aligned16(ckpt)) return CAMOE_ERR_ALIGNMENT;
    if (ckpt_bytes < required_ckpt(B, T, h_count, al)) return CAMOE_ERR_WORKSPACE;
  }
  if ((st = check_carry(T, {s0, sT})) != CAMOE_OK) return st;
  camoe::FwdArgs p;
  p.r = r; p.w = w; p.k = k; p.v = v; p.a = a; p.b = b;
  p.y = y; p.sa = sa; p.ckpt = static_cast<float*>(ckpt);
  p.s0 = s0; p.sT = sT;
  p.records_ready = records_ready;
  p.g = camoe::Geom{B, T, H_total, h0, h_count, (T + camoe::kChunk - 1) / camoe::kChunk, decay};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (al == CAMOE_ALGO_CHUNKED) return cuda_status(camoe::chunked::launch_fwd(p, s));
  if (dtype == CAMOE_DTYPE_BF16) return cuda_status(camoe::scan::launch_fwd<camoe::bf16>(p, s));
  return cuda_status(camoe::scan::launch_fwd<float>(p, s));
}

}  // namespace

extern "C" {

int camoe_wkv7_fwd(const void* r, const void* w, const void* k, const void* v, const void* a,
                   const void* b, void* y, float* sa, void* ckpt, size_t ckpt_bytes, int64_t B,
                   int64_t T, int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype,
                   int algo, void* stream) {
  return fwd_impl(r, w, k, v, a, b, y, sa, ckpt, ckpt_bytes, B, T, H_total, h0, h_count, N, dtype,
                  algo, stream, camoe::kDecayClampW);
}

int camoe_wkv7_wind_fwd(const void* w, const void* q, const void* k, const void* v,
                        const void* z, const void* a, void* y, float* sa, void* ckpt,
                        size_t ckpt_bytes, int64_t B, int64_t T, int64_t H_total, int64_t h0,
                        int64_t h_count, int N, int dtype, int algo, void* stream) {
  // the wind op's (w, q, z, a) are the ClampW op's (w, r, a, b)
  return fwd_impl(q, w, k, v, z, a, y, sa, ckpt, ckpt_bytes, B, T, H_total, h0, h_count, N, dtype,
                  algo, stream, camoe::kDecayWind);
}

size_t camoe_wkv7_state_work_bytes(int64_t B, int64_t T, int64_t h_count, int N, int dtype,
                                   int algo) {
  const int al = resolve_state_algo(dtype, algo, T);
  if (al != CAMOE_ALGO_CHUNKED || N != camoe::kN || B < 0 || T < 0 || h_count < 0) return 0;
  return camoe::chunked::infer_bytes(B * h_count, T);
}

int camoe_wkv7_fwd_state(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, void* y, float* sa, const float* s0,
                         float* s_out, void* work, size_t work_bytes, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
                         void* stream) {
  int st = check_geometry(B, T, H_total, h0, h_count, N);
  if (st != CAMOE_OK) return st;
  const int al = resolve_state_algo(dtype, algo, T);
  if (al < 0) return CAMOE_ERR_UNSUPPORTED;
  if (B * h_count == 0) return CAMOE_OK;
  if (work != nullptr && al == CAMOE_ALGO_CHUNKED) {
    if (!aligned16(work)) return CAMOE_ERR_ALIGNMENT;
    if (work_bytes < camoe::chunked::infer_bytes(B * h_count, T)) return CAMOE_ERR_WORKSPACE;
  }
  if ((s0 != nullptr && !aligned16(s0)) || (s_out != nullptr && !aligned16(s_out)))
    return CAMOE_ERR_ALIGNMENT;
  if (s0 != nullptr && s_out != nullptr && s0 != s_out) {
    // the two [B, H_total, N, N] arrays must be the same or disjoint
    const size_t bytes = static_cast<size_t>(B * H_total) * camoe::kN * camoe::kN * sizeof(float);
    const uintptr_t x = reinterpret_cast<uintptr_t>(s0), z = reinterpret_cast<uintptr_t>(s_out);
    if (x < z + bytes && z < x + bytes) return CAMOE_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) {  // no step: the final state is the start state
    if (s_out == nullptr || s_out == s0) return CAMOE_OK;
    const size_t nn = static_cast<size_t>(camoe::kN) * camoe::kN * sizeof(float);
    float* dst = s_out + h0 * camoe::kN * camoe::kN;
    const size_t pitch = static_cast<size_t>(H_total) * nn, width = static_cast<size_t>(h_count) * nn;
    if (s0 == nullptr)
      return cuda_status(cudaMemset2DAsync(dst, pitch, 0, width, static_cast<size_t>(B), s));
    return cuda_status(cudaMemcpy2DAsync(dst, pitch, s0 + h0 * camoe::kN * camoe::kN, pitch, width,
                                         static_cast<size_t>(B), cudaMemcpyDeviceToDevice, s));
  }
  const void* ptrs[] = {r, w, k, v, a, b, y, sa};
  for (const void* p : ptrs) {
    if (p == nullptr) return CAMOE_ERR_INVALID_ARG;
    if (!aligned16(p)) return CAMOE_ERR_ALIGNMENT;
  }
  camoe::FwdArgs p;
  p.r = r; p.w = w; p.k = k; p.v = v; p.a = a; p.b = b;
  p.y = y; p.sa = sa; p.ckpt = nullptr;
  p.s0 = s0; p.sT = s_out;
  p.work = al == CAMOE_ALGO_CHUNKED ? work : nullptr;
  p.g = camoe::Geom{B, T, H_total, h0, h_count, (T + camoe::kChunk - 1) / camoe::kChunk};
  if (al == CAMOE_ALGO_CHUNKED) return cuda_status(camoe::chunked::launch_fwd(p, s));
  if (dtype == CAMOE_DTYPE_BF16) return cuda_status(camoe::scan::launch_fwd<camoe::bf16>(p, s));
  return cuda_status(camoe::scan::launch_fwd<float>(p, s));
}

}  // extern "C"

namespace {

int bwd_impl(const void* r, const void* w, const void* k, const void* v, const void* a,
             const void* b, const void* dy, const float* dsa, const void* ckpt, size_t ckpt_bytes,
             void* work, size_t work_bytes, void* dr, void* dw, void* dk, void* dv, void* da,
             void* db, int64_t B, int64_t T, int64_t H_total, int64_t h0, int64_t h_count, int N,
             int dtype, int algo, void* stream, int decay, const float* s0 = nullptr,
             const float* dsT = nullptr, float* ds0 = nullptr) {
  int st = check_geometry(B, T, H_total, h0, h_count, N);
  if (st != CAMOE_OK) return st;
  const int al = resolve_algo(dtype, algo);
  if (al < 0) return CAMOE_ERR_UNSUPPORTED;
  if (B * h_count == 0 || T == 0) return CAMOE_OK;
  // dv and ds0 only: the chunked path with a start-state gradient may leave
  // the five key-side gradients null (its key-side pass is then skipped)
  const bool key_null = dr == nullptr && dw == nullptr && dk == nullptr && da == nullptr &&
                        db == nullptr;
  const bool ds0_only = key_null && ds0 != nullptr && al == CAMOE_ALGO_CHUNKED;
  const void* ptrs[] = {r, w, k, v, a, b, dy, dv, dr, dw, dk, da, db};
  for (int i = 0; i < (ds0_only ? 8 : 13); ++i) {
    if (ptrs[i] == nullptr) return CAMOE_ERR_INVALID_ARG;
    if (!aligned16(ptrs[i])) return CAMOE_ERR_ALIGNMENT;
  }
  if (dsa != nullptr && !aligned16(dsa)) return CAMOE_ERR_ALIGNMENT;
  const size_t need = required_ckpt(B, T, h_count, al);
  if (need > 0) {
    if (ckpt == nullptr) return CAMOE_ERR_INVALID_ARG;
    if (!aligned16(ckpt)) return CAMOE_ERR_ALIGNMENT;
    if (ckpt_bytes < need) return CAMOE_ERR_WORKSPACE;
  }
  const size_t wneed = required_work(B, T, h_count, al);
  if (wneed > 0) {
    if (work == nullptr) return CAMOE_ERR_INVALID_ARG;
    if (!aligned16(work)) return CAMOE_ERR_ALIGNMENT;
    if (work_bytes < wneed) return CAMOE_ERR_WORKSPACE;
  }
  if ((st = check_carry(T, {s0, dsT, ds0})) != CAMOE_OK) return st;
  camoe::BwdArgs p;
  p.r = r; p.w = w; p.k = k; p.v = v; p.a = a; p.b = b; p.dy = dy;
  p.dsa = dsa; p.ckpt = static_cast<const float*>(ckpt);
  p.dr = dr; p.dw = dw; p.dk = dk; p.dv = dv; p.da = da; p.db = db;
  p.s0 = s0; p.dsT = dsT; p.ds0 = ds0;
  p.g = camoe::Geom{B, T, H_total, h0, h_count, (T + camoe::kChunk - 1) / camoe::kChunk, decay};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (al == CAMOE_ALGO_CHUNKED) return cuda_status(camoe::chunked::launch_bwd(p, work, s));
  if (dtype == CAMOE_DTYPE_BF16) return cuda_status(camoe::scan::launch_bwd<camoe::bf16>(p, s));
  return cuda_status(camoe::scan::launch_bwd<float>(p, s));
}

}  // namespace

extern "C" {

int camoe_wkv7_fwd_carry(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, void* y, float* sa, const float* s0,
                         float* s_out, void* ckpt, size_t ckpt_bytes, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
                         void* stream) {
  // an empty sequence would have to pass the state through unchanged; the
  // carried calls want at least one chunk
  if (T == 0 && (s0 != nullptr || s_out != nullptr)) return CAMOE_ERR_SHAPE;
  return fwd_impl(r, w, k, v, a, b, y, sa, ckpt, ckpt_bytes, B, T, H_total, h0, h_count, N, dtype,
                  algo, stream, camoe::kDecayClampW, s0, s_out);
}

int camoe_wkv7_fwd_value(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, void* y, float* sa, const float* s0,
                         float* s_out, void* ckpt, size_t ckpt_bytes, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype,
                         void* stream) {
  if (T == 0 && (s0 != nullptr || s_out != nullptr)) return CAMOE_ERR_SHAPE;
  if (dtype != CAMOE_DTYPE_BF16) return CAMOE_ERR_UNSUPPORTED;
  if (ckpt == nullptr) return CAMOE_ERR_INVALID_ARG;
  return fwd_impl(r, w, k, v, a, b, y, sa, ckpt, ckpt_bytes, B, T, H_total, h0, h_count, N, dtype,
                  CAMOE_ALGO_CHUNKED, stream, camoe::kDecayClampW, s0, s_out, true);
}

int camoe_wkv7_bwd(const void* r, const void* w, const void* k, const void* v, const void* a,
                   const void* b, const void* dy, const float* dsa, const void* ckpt,
                   size_t ckpt_bytes, void* work, size_t work_bytes, void* dr, void* dw, void* dk,
                   void* dv, void* da, void* db, int64_t B, int64_t T, int64_t H_total,
                   int64_t h0, int64_t h_count, int N, int dtype, int algo, void* stream) {
  return bwd_impl(r, w, k, v, a, b, dy, dsa, ckpt, ckpt_bytes, work, work_bytes, dr, dw, dk, dv,
                  da, db, B, T, H_total, h0, h_count, N, dtype, algo, stream, camoe::kDecayClampW);
}

int camoe_wkv7_bwd_carry(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, const void* dy, const float* dsa,
                         const float* s0, const float* ds_out, float* ds0, const void* ckpt,
                         size_t ckpt_bytes, void* work, size_t work_bytes, void* dr, void* dw,
                         void* dk, void* dv, void* da, void* db, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
                         void* stream) {
  if (T == 0 && (s0 != nullptr || ds_out != nullptr || ds0 != nullptr)) return CAMOE_ERR_SHAPE;
  return bwd_impl(r, w, k, v, a, b, dy, dsa, ckpt, ckpt_bytes, work, work_bytes, dr, dw, dk, dv,
                  da, db, B, T, H_total, h0, h_count, N, dtype, algo, stream, camoe::kDecayClampW,
                  s0, ds_out, ds0);
}

int camoe_wkv7_wind_bwd(const void* w, const void* q, const void* k, const void* v,
                        const void* z, const void* a, const void* dy, const float* dsa,
                        const void* ckpt, size_t ckpt_bytes, void* work, size_t work_bytes,
                        void* dw, void* dq, void* dk, void* dv, void* dz, void* da, int64_t B,
                        int64_t T, int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype,
                        int algo, void* stream) {
  return bwd_impl(q, w, k, v, z, a, dy, dsa, ckpt, ckpt_bytes, work, work_bytes, dq, dw, dk, dv,
                  dz, da, B, T, H_total, h0, h_count, N, dtype, algo, stream, camoe::kDecayWind);
}

}  // extern "C"
