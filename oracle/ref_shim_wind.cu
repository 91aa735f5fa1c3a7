// C-ABI shim over the reference's wind_backstepping host launchers, so the
// GPU parity tests can call that op (built from camoe/cuda/wkv7_cuda.cu and
// wkv7_cuda_fp32.cu by oracle/Makefile) with plain device pointers.  Test
// infrastructure only.
//
// The launchers' prototypes are those of camoe/cuda/wkv7_op.cpp:5,13: they
// launch on the legacy default stream and check nothing, so the caller
// synchronises and validates shapes (T % 16 == 0) itself.
#include <cuda_runtime.h>
#ifdef _FP32_
using elem_t = float;
#else
#include <cuda_bf16.h>
using elem_t = __nv_bfloat16;
#endif

void cuda_forward(int B, int T, int H, elem_t* w, elem_t* q, elem_t* k, elem_t* v, elem_t* z,
                  elem_t* a, elem_t* y, float* s, float* sa);
void cuda_backward(int B, int T, int H, elem_t* w, elem_t* q, elem_t* k, elem_t* v, elem_t* z,
                   elem_t* a, elem_t* dy, float* s, float* sa, elem_t* dw, elem_t* dq,
                   elem_t* dk, elem_t* dv, elem_t* dz, elem_t* da);

extern "C" int ref_wind_fwd(int B, int T, int H, void* w, void* q, void* k, void* v, void* z,
                            void* a, void* y, float* s, float* sa) {
  cuda_forward(B, T, H, (elem_t*)w, (elem_t*)q, (elem_t*)k, (elem_t*)v, (elem_t*)z,
               (elem_t*)a, (elem_t*)y, s, sa);
  return (int)cudaGetLastError();
}

extern "C" int ref_wind_bwd(int B, int T, int H, void* w, void* q, void* k, void* v, void* z,
                            void* a, void* dy, float* s, float* sa, void* dw, void* dq,
                            void* dk, void* dv, void* dz, void* da) {
  cuda_backward(B, T, H, (elem_t*)w, (elem_t*)q, (elem_t*)k, (elem_t*)v, (elem_t*)z,
                (elem_t*)a, (elem_t*)dy, s, sa, (elem_t*)dw, (elem_t*)dq, (elem_t*)dk,
                (elem_t*)dv, (elem_t*)dz, (elem_t*)da);
  return (int)cudaGetLastError();
}
