// C-ABI shim over the reference's ClampW host launchers, so the GPU parity
// tests can call the reference op (built from camoe/cuda/rwkv7_clampw.cu by
// oracle/Makefile) with plain device pointers.  Test infrastructure only.
//
// The launchers' prototypes are those of camoe/cuda/rwkv7_clampw.cpp:9,16:
// they launch on the legacy default stream and check nothing, so the caller
// synchronises and validates shapes (T % 16 == 0) itself.
#include <cuda_runtime.h>
#ifdef _FP32_
using elem_t = float;
#else
#include <cuda_bf16.h>
using elem_t = __nv_bfloat16;
#endif

void cuda_forward(int B, int T, int H, elem_t* r, elem_t* w, elem_t* k, elem_t* v, elem_t* a,
                  elem_t* b, elem_t* y, float* s, float* sa);
void cuda_backward(int B, int T, int H, elem_t* r, elem_t* w, elem_t* k, elem_t* v, elem_t* a,
                   elem_t* b, elem_t* dy, float* s, float* sa, elem_t* dr, elem_t* dw,
                   elem_t* dk, elem_t* dv, elem_t* da, elem_t* db);

extern "C" int ref_clampw_fwd(int B, int T, int H, void* r, void* w, void* k, void* v, void* a,
                              void* b, void* y, float* s, float* sa) {
  cuda_forward(B, T, H, (elem_t*)r, (elem_t*)w, (elem_t*)k, (elem_t*)v, (elem_t*)a,
               (elem_t*)b, (elem_t*)y, s, sa);
  return (int)cudaGetLastError();
}

extern "C" int ref_clampw_bwd(int B, int T, int H, void* r, void* w, void* k, void* v, void* a,
                              void* b, void* dy, float* s, float* sa, void* dr, void* dw,
                              void* dk, void* dv, void* da, void* db) {
  cuda_backward(B, T, H, (elem_t*)r, (elem_t*)w, (elem_t*)k, (elem_t*)v, (elem_t*)a,
                (elem_t*)b, (elem_t*)dy, s, sa, (elem_t*)dr, (elem_t*)dw, (elem_t*)dk,
                (elem_t*)dv, (elem_t*)da, (elem_t*)db);
  return (int)cudaGetLastError();
}
