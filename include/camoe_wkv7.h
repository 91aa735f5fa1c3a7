/*
 * camoe_wkv7.h — C ABI of the B200 (sm_100a) WKV-7 "ClampW" operator.
 *
 * The operator computes, independently for every (batch b, head h) chain,
 *     w_t  = exp(-exp(-1/2) * sigmoid(w_in_t))            (per element)
 *     sa_t = S_{t-1} a_t
 *     S_t  = S_{t-1} diag(w_t) + sa_t b_t^T + v_t k_t^T    (S_{-1} = 0, N x N, fp32)
 *     y_t  = S_t r_t
 * and the gradients of sum(dy*y) + sum(dsa*sa) with respect to r, w_in, k,
 * v, a and b.
 *
 * Every tensor argument is a [B, T, H_total, N] contiguous array (element
 * ((b*T + t)*H_total + h)*N + i), N = 64.  A call processes the heads
 * [h0, h0 + h_count) of those arrays in place, so a head-sharded launcher
 * passes slices without copies.  r, w, k, v, a, b, y, dy and the six
 * gradients have the element type `dtype` (bf16 or fp32); sa and dsa are
 * always fp32.  The caller owns every buffer; nothing is allocated.  All
 * pointers must be 16-byte aligned device pointers.
 *
 * The forward writes a per-chain checkpoint that the backward reads.  Its
 * size comes from camoe_wkv7_ckpt_bytes(); it never exceeds the reference's
 * [B, H, T/16, N, N] fp32 checkpoint tensor, so that tensor can be passed as
 * the buffer.  The forward and backward of one pair must use the same dtype,
 * algo and shape.  Passing ckpt = NULL to the forward skips the checkpoint
 * (inference).  The backward also takes a scratch workspace of
 * camoe_wkv7_work_bytes() bytes (0 for the scan algorithm); the checkpoint is
 * only read, so a backward can be repeated.
 *
 * Calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 * stream); all but camoe_wkv7_fwd_bwd_noalloc keep no global state and may
 * run concurrently on different streams.  They return CAMOE_OK or an error
 * code; no call aborts or traps.
 *
 * Reference interfaces these replace:
 *   torch.ops.rwkv7_clampw.forward(r,w,k,v,a,b,y,s,sa)
 *       camoe/cuda/rwkv7_clampw.cpp:12-15, launcher rwkv7_clampw.cu:76-79
 *   torch.ops.rwkv7_clampw.backward(r,w,k,v,a,b,dy,s,sa,dr,dw,dk,dv,da,db)
 *       camoe/cuda/rwkv7_clampw.cpp:19-23, launcher rwkv7_clampw.cu:172-176
 *   checkpoint tensor s = empty(B, H, T/16, N, N, fp32)   camoe/backbone.py:87
 */
#ifndef CAMOE_WKV7_H
#define CAMOE_WKV7_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define CAMOE_DTYPE_BF16 0
#define CAMOE_DTYPE_FP32 1

/* algorithms: AUTO = CHUNKED for bf16, SCAN for fp32 */
#define CAMOE_ALGO_AUTO 0
#define CAMOE_ALGO_SCAN 1    /* per-step fp32 SIMT scan, the fp32-exact path */
#define CAMOE_ALGO_CHUNKED 2 /* 16-step chunks on the tensor cores, bf16 only */

/* status codes */
#define CAMOE_OK 0
#define CAMOE_ERR_INVALID_ARG 1  /* NULL required pointer, negative size, bad head range */
#define CAMOE_ERR_UNSUPPORTED 2  /* N != 64, unknown dtype/algo, fp32 with CHUNKED */
#define CAMOE_ERR_SHAPE 3        /* T not a multiple of 16 */
#define CAMOE_ERR_ALIGNMENT 4    /* a pointer is not 16-byte aligned */
#define CAMOE_ERR_WORKSPACE 5    /* checkpoint or workspace smaller than required */
#define CAMOE_ERR_CUDA 6         /* a CUDA launch failed; see camoe_wkv7_last_cuda_error() */

/* Version of this ABI (major*10000 + minor*100 + patch). */
int camoe_wkv7_version(void);

/* Static description of a status code. */
const char* camoe_wkv7_strerror(int code);

/* The cudaError_t of the most recent CAMOE_ERR_CUDA on the calling thread. */
int camoe_wkv7_last_cuda_error(void);

/* Number of bounded device-side waits that timed out on the current device
 * since the library was loaded (0 in correct operation; a timed-out kernel
 * stops early and leaves its outputs incomplete).  Synchronises the device.
 * Returns UINT_MAX if the count cannot be read. */
unsigned int camoe_wkv7_device_errors(void);

/* Bytes of state checkpoint a forward/backward pair needs for B x h_count
 * chains of length T (0 when there is nothing to store).  Returns 0 for
 * invalid arguments as well; the fwd/bwd calls report those. */
size_t camoe_wkv7_ckpt_bytes(int64_t B, int64_t T, int64_t h_count, int N, int dtype,
                             int algo);

/* Bytes of backward workspace for the same problem (0 when none is needed). */
size_t camoe_wkv7_work_bytes(int64_t B, int64_t T, int64_t h_count, int N, int dtype,
                             int algo);

/* Forward.  Writes y (dtype) and sa (fp32) for heads [h0, h0+h_count) and,
 * when ckpt != NULL, the state checkpoint.  Replaces
 * torch.ops.rwkv7_clampw.forward (camoe/cuda/rwkv7_clampw.cpp:12-15). */
int camoe_wkv7_fwd(const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, void* y, float* sa, void* ckpt,
                   size_t ckpt_bytes, int64_t B, int64_t T, int64_t H_total, int64_t h0,
                   int64_t h_count, int N, int dtype, int algo, void* stream);

/* Backward.  Reads the checkpoint written by the matching forward, dy
 * (dtype) and, when non-NULL, dsa (fp32, the gradient of sa); writes the six
 * input gradients (dtype).  Replaces torch.ops.rwkv7_clampw.backward
 * (camoe/cuda/rwkv7_clampw.cpp:19-23), whose autograd wrapper took no sa
 * gradient (camoe/backbone.py:95). */
int camoe_wkv7_bwd(const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, const void* dy, const float* dsa,
                   const void* ckpt, size_t ckpt_bytes, void* work, size_t work_bytes,
                   void* dr, void* dw, void* dk, void* dv, void* da, void* db, int64_t B,
                   int64_t T, int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype,
                   int algo, void* stream);

/* Training across calls (a long sequence processed in pieces with the
 * state carried between them): camoe_wkv7_fwd and camoe_wkv7_bwd with the
 * state arrays of camoe_wkv7_fwd_state ([B, H_total, N, N] fp32, element
 * ((b*H_total + h)*N + i)*N + j = S[i][j]).  The forward starts every chain
 * from s0 (NULL = zero) and writes its final state to s_out (NULL = not
 * stored).  The backward takes the same s0, the gradient of the final state
 * ds_out (NULL = zero), and writes the gradient of the start state to ds0
 * (NULL = not wanted), besides the six input gradients; so the backward of a
 * later piece hands its ds0 to the earlier piece as ds_out.  With
 * CAMOE_ALGO_CHUNKED (or AUTO on bf16) and ds0 given, dr, dw, dk, da and db
 * may all be NULL: only dv and ds0 are then computed, and the key-side pass,
 * about 60% of the backward, is skipped.  T must be a
 * positive multiple of 16 when any state array is given (else
 * CAMOE_ERR_SHAPE).  No counterpart in the reference, whose op always starts
 * from the zero state (camoe/cuda/rwkv7_clampw.cu:28). */
int camoe_wkv7_fwd_carry(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, void* y, float* sa, const float* s0,
                         float* s_out, void* ckpt, size_t ckpt_bytes, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
                         void* stream);

/* The value pass of camoe_wkv7_fwd_carry alone (bf16, chunked): the
 * key-side records in ckpt (which depend on r, w, k, a and b only) were
 * written by an earlier camoe_wkv7_fwd_carry or camoe_wkv7_fwd of the same r,
 * w, k, a, b and geometry into the same ckpt, and are reused; v, s0 may
 * differ.  Writes y, sa, s_out and the checkpoint's states, so the ckpt then
 * serves the backward of this call.  Several forwards over one sequence that
 * differ only in v or the start state (camoe_b200/segmented.py) run the
 * key-side pass once. */
int camoe_wkv7_fwd_value(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, void* y, float* sa, const float* s0,
                         float* s_out, void* ckpt, size_t ckpt_bytes, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype,
                         void* stream);

int camoe_wkv7_bwd_carry(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, const void* dy, const float* dsa,
                         const float* s0, const float* ds_out, float* ds0, const void* ckpt,
                         size_t ckpt_bytes, void* work, size_t work_bytes, void* dr, void* dw,
                         void* dk, void* dv, void* da, void* db, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
                         void* stream);

/* Joins the segments of chains cut in time into P pieces of equal length.
 * states, trans and local are [B*P, H_total, N, N] fp32 arrays (segment g of
 * sequence b at index b*P + g, element as in camoe_wkv7_fwd_state); only the
 * heads [h0, h0 + h_count) are read or written.  trans holds every segment's
 * transition A (its final state from an identity start with v = 0).
 *   backward = 0: local = C, each segment's final state from a zero start;
 *     states[b, 0] is given and states[b, g] = states[b, g-1] A_{g-1} + C_{g-1}
 *     is written for g = 1 .. P-1 (the start state of every segment).
 *   backward = 1: local = D, each segment's start-state gradient with no
 *     gradient at its end; states[b, P-1] is given and
 *     states[b, g-1] = states[b, g] A_g^T + D_g is written for g = P-1 .. 1
 *     (the gradient of every segment's final state).
 * One launch on `stream`.  No counterpart in the reference, whose op runs each
 * chain from t = 0 to T in one sequential pass (camoe/cuda/rwkv7_clampw.cu:36). */
int camoe_wkv7_seg_chain(float* states, const float* trans, const float* local, int64_t B,
                         int64_t P, int64_t H_total, int64_t h0, int64_t h_count, int backward,
                         void* stream);

/* The reference's second WKV-7 op, wind_backstepping (camoe/cuda/wkv7_cuda.cu,
 * wkv7_cuda_fp32.cu; bound by camoe/cuda/wkv7_op.cpp:5-21), in its own
 * argument order: forward(w, q, k, v, z, a) with decay exp(-exp(w)) in place
 * of ClampW's exp(-e^{-1/2} sigmoid(w)); q, z, a play the roles of ClampW's
 * r, a, b.  Same shapes, dtypes, checkpoint and workspace sizes, algorithms
 * and status codes as camoe_wkv7_fwd / camoe_wkv7_bwd.  The decay is not
 * clamped: the chunked algorithm is exact for w <= -1/2 (decays >= 0.545,
 * as RWKV-7's time mix produces them) and stays finite while a 16-step
 * chunk's summed exp(w) stays below about 88; SCAN takes any w.  The
 * reference's backward reverses the state through 1/decay
 * (wkv7_cuda.cu:91-94); this one recomputes it forward from checkpoints. */
int camoe_wkv7_wind_fwd(const void* w, const void* q, const void* k, const void* v,
                        const void* z, const void* a, void* y, float* sa, void* ckpt,
                        size_t ckpt_bytes, int64_t B, int64_t T, int64_t H_total, int64_t h0,
                        int64_t h_count, int N, int dtype, int algo, void* stream);

int camoe_wkv7_wind_bwd(const void* w, const void* q, const void* k, const void* v,
                        const void* z, const void* a, const void* dy, const float* dsa,
                        const void* ckpt, size_t ckpt_bytes, void* work, size_t work_bytes,
                        void* dw, void* dq, void* dk, void* dv, void* dz, void* da, int64_t B,
                        int64_t T, int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype,
                        int algo, void* stream);

/* Stateful forward, for inference and decoding: camoe_wkv7_fwd without a
 * checkpoint, but every chain starts from the state s0 instead of zero and
 * its state after step T-1 is written to s_out.  s0 and s_out are fp32
 * [B, H_total, N, N] arrays, element ((b*H_total + h)*N + i)*N + j = S[i][j]
 * (i the value index, j the key index); the heads [h0, h0 + h_count) are
 * read and written in place.  s0 = NULL starts from the zero state (then
 * y and sa equal camoe_wkv7_fwd's), s_out = NULL skips the store, and
 * s_out == s0 updates the state in place (a partial overlap is
 * CAMOE_ERR_INVALID_ARG).  Any T >= 0: a forward over steps [0, T1) followed
 * by one over [T1, T) from its s_out gives the y and sa of one forward over
 * [0, T).  AUTO runs the per-step decode kernel for T <= 16 (any dtype),
 * else CHUNKED for bf16 and SCAN for fp32.  CHUNKED with work = NULL runs one
 * fused kernel per chain; with a workspace of camoe_wkv7_state_work_bytes()
 * bytes it runs the key-side pass over all SMs first (faster when there are
 * fewer chains than about 3/4 of the SM count); other algorithms ignore work.
 * No gradient flows through the states.  No counterpart in the reference,
 * which recomputes the whole prefix for every generated token (eval.py:212,
 * camoe/wrapper.py:203-223). */
int camoe_wkv7_fwd_state(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, void* y, float* sa, const float* s0,
                         float* s_out, void* work, size_t work_bytes, int64_t B, int64_t T,
                         int64_t H_total, int64_t h0, int64_t h_count, int N, int dtype, int algo,
                         void* stream);

/* Bytes of the optional workspace of camoe_wkv7_fwd_state (0 when its
 * algorithm takes none). */
size_t camoe_wkv7_state_work_bytes(int64_t B, int64_t T, int64_t h_count, int N, int dtype,
                                   int algo);

/* Test hook for the bounded device waits; no counterpart in the reference.
 * Every wait of the chunked kernels on a pipeline barrier gives up after a
 * limit (by default 2e9 clock cycles, about a second), counts the event in
 * camoe_wkv7_device_errors() and makes the kernel's roles return.  This call
 * sets that limit (1000 .. 2e9 cycles) for later launches on the current
 * device, and with skip_pair >= 0 makes the forward's value pass withhold
 * the loads of that pair of 16-step chunks, so that its waits run out: a test
 * that failure detection returns instead of hanging.  skip_pair = -1 with
 * the default limit restores normal operation.  Returns CAMOE_ERR_INVALID_ARG
 * for a limit or pair outside those ranges.  Not for production use. */
int camoe_wkv7_test_hooks(long long wait_limit_cycles, int skip_pair);

/* Size of the library-owned checkpoint scratch used by
 * camoe_wkv7_fwd_bwd_noalloc (64 MiB per GPU that loads the library). */
#define CAMOE_WKV7_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/* Forward and backward in one call that allocates nothing, for callers that
 * cannot allocate device memory (a host whose device memory belongs to
 * another runtime's pooled allocator, or a training step that must not let
 * cudaMalloc synchronise the device).  No counterpart in the reference.
 * Writes y, sa and the six gradients like camoe_wkv7_fwd followed by
 * camoe_wkv7_bwd, with the state checkpoint kept in a library-owned device
 * array of CAMOE_WKV7_NOALLOC_SCRATCH_BYTES instead of a caller buffer.
 * Returns CAMOE_ERR_WORKSPACE when camoe_wkv7_ckpt_bytes() plus
 * camoe_wkv7_work_bytes() of the problem exceed that size (about 1900 chains x
 * 16-step chunks for the chunked algorithm, 4096 for the scan).  The first
 * call on a device looks up the array's address (cudaGetSymbolAddress); make
 * it before any stream capture.  That address is cached for the life of the
 * process and does not survive a cudaDeviceReset of the device: do not call
 * this entry point on a device after resetting it.  All calls share the
 * array: calls whose work overlaps on the GPU race. */
int camoe_wkv7_fwd_bwd_noalloc(const void* r, const void* w, const void* k, const void* v,
                               const void* a, const void* b, const void* dy, const float* dsa,
                               void* y, float* sa, void* dr, void* dw, void* dk, void* dv,
                               void* da, void* db, int64_t B, int64_t T, int64_t H_total,
                               int64_t h0, int64_t h_count, int N, int dtype, int algo,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CAMOE_WKV7_H */
