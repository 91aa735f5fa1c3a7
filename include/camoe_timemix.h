/*
 * camoe_timemix.h — C ABI of the fused elementwise kernels around the WKV-7
 * op in RWKV-7's time mix (the reference's RWKV7_TimeMix.forward,
 * camoe/backbone.py:296-373).  The projections (receptance, key, value,
 * output and the LoRA products) are plain GEMMs and are not here.
 *
 * Every activation is a [B, T, C] contiguous array (C = H * 64, 64 <= C <=
 * 2048, C % 64 == 0), element (b*T + t)*C + c, bf16 unless stated; head h is
 * columns [64h, 64h + 64).  Parameters are fp32 vectors of C (r_k: [H, 64]).
 * All math is fp32.  Backward calls write parameter gradients (fp32, not
 * accumulated) and take a scratch workspace of camoe_tm_work_bytes() bytes
 * for their per-block partial sums.  All pointers 16-byte aligned; calls are
 * asynchronous on `stream`; status codes as in camoe_wkv7.h (0 = ok).
 *
 * Forward of one time mix with these kernels:
 *   mix:  xr..xg = x + (shift(x) - x) * x_{r,w,k,v,a,g}      (backbone.py:316-323)
 *   [GEMMs: r, k, v, wl = tanh(xw w1) w2, vl = xv v1 v2, al = xa a1 a2, g]
 *   prep: w = -softplus(-(w0 + wl)) - 1/2; v' = v + (v_first - v) sigmoid(v0 + vl)
 *         (layers > 0); a = sigmoid(a0 + al); kk = normalize_head(k k_k);
 *         k' = k (1 + (a - 1) k_a); op inputs (r, w, k', v', -kk, kk a)
 *                                                            (backbone.py:326-343)
 *   [WKV-7 op: y, sa]
 *   lnsa: state_representation = LayerNorm_C(sa)             (backbone.py:348)
 *   post: z = (GroupNorm_head(y) + sum_head(r k' r_k) v') g  (backbone.py:359-367)
 *   [GEMM: out = z W_o^T]
 */
#ifndef CAMOE_TIMEMIX_H
#define CAMOE_TIMEMIX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Bytes of backward workspace (partial sums) for a [B, T, C] problem. */
size_t camoe_tm_work_bytes(int64_t B, int64_t T, int64_t C);

/* Token shift and the six mixes.  x has element type x_dtype (0 bf16,
 * 1 fp32); mix is [6][C] (x_r, x_w, x_k, x_v, x_a, x_g); out[m] are six bf16
 * arrays. */
int camoe_tm_mix_fwd(const void* x, int x_dtype, const float* mix, void* const* out, int64_t B,
                     int64_t T, int64_t C, void* stream);

/* camoe_tm_mix_fwd with the step before step 0 of each sequence given:
 * x_prev is [B, C] of x_dtype (the last step of the previous call, for a
 * time mix carried across calls); NULL means zero, as camoe_tm_mix_fwd. */
int camoe_tm_mix_fwd_prev(const void* x, int x_dtype, const void* x_prev, const float* mix,
                          void* const* out, int64_t B, int64_t T, int64_t C, void* stream);

/* Backward of camoe_tm_mix_fwd: dout[m] (bf16) -> dx (x_dtype), dmix [6][C]. */
int camoe_tm_mix_bwd(const void* x, int x_dtype, const float* mix, const void* const* dout,
                     void* dx, float* dmix, void* work, size_t work_bytes, int64_t B, int64_t T,
                     int64_t C, void* stream);

/* Op inputs from the projections.  params is [5][C]: w0, v0, a0, k_k, k_a.
 * vl and v_first are NULL for layer 0 (no value residual; then v' = v).
 * Writes w, k', v', a = -kk and b = kk * a (bf16). */
int camoe_tm_prep_fwd(const void* wl, const void* k, const void* v, const void* vl,
                      const void* al, const void* v_first, const float* params, void* w_op,
                      void* k_op, void* v_op, void* a_op, void* b_op, int64_t B, int64_t T,
                      int64_t C, void* stream);

/* Backward of camoe_tm_prep_fwd and of the two uses of r, k', v' downstream:
 * g_r = dr_op + dr_epi, g_k' = dk_op + dk_epi, g_v' = dv_op + dv_epi (the op's
 * and the epilogue's gradients), g_w = dw_op, g_a = da_op, g_b = db_op, and
 * (layer 0) dv_first_out, the gradient of v_first = v.  Writes dr, dwl, dk,
 * dv, dal and, for layers > 0, dvl and dv_first (bf16); dparams [5][C]. */
int camoe_tm_prep_bwd(const void* dr_op, const void* dr_epi, const void* dw_op,
                      const void* dk_op, const void* dk_epi, const void* dv_op,
                      const void* dv_epi, const void* da_op, const void* db_op,
                      const void* dv_first_out, const void* wl, const void* k, const void* v,
                      const void* vl, const void* al, const void* v_first, const float* params,
                      void* dr, void* dwl, void* dk, void* dv, void* dvl, void* dal,
                      void* dv_first, float* dparams, void* work, size_t work_bytes, int64_t B,
                      int64_t T, int64_t C, void* stream);

/* Epilogue: z = (GroupNorm_head(y) * gamma + beta + sum_head(r k' r_k) v') * g
 * (GroupNorm eps 64e-5, camoe/backbone.py:217). */
int camoe_tm_post_fwd(const void* y, const void* r, const void* k_op, const void* v_op,
                      const void* g, const float* r_k, const float* gamma, const float* beta,
                      void* z, int64_t B, int64_t T, int64_t C, void* stream);

/* Backward of camoe_tm_post_fwd: dz -> dy, dr_epi, dk_epi, dv_epi, dg (bf16);
 * dparams [3][C]: gamma, beta, r_k. */
int camoe_tm_post_bwd(const void* dz, const void* y, const void* r, const void* k_op,
                      const void* v_op, const void* g, const float* r_k, const float* gamma,
                      const float* beta, void* dy, void* dr_epi, void* dk_epi, void* dv_epi,
                      void* dg, float* dparams, void* work, size_t work_bytes, int64_t B,
                      int64_t T, int64_t C, void* stream);

/* state_representation = LayerNorm over C of sa (fp32 in and out, eps 1e-5,
 * weight/bias [C]). */
int camoe_tm_lnsa_fwd(const float* sa, const float* weight, const float* bias, float* out,
                      int64_t B, int64_t T, int64_t C, void* stream);

/* Backward: dout -> dsa (fp32); dparams [2][C]: weight, bias. */
int camoe_tm_lnsa_bwd(const float* dout, const float* sa, const float* weight, float* dsa,
                      float* dparams, void* work, size_t work_bytes, int64_t B, int64_t T,
                      int64_t C, void* stream);

/* Weight gradient of one LoRA product (camoe/backbone.py:326-341, x @ w1 and
 * h @ w2, whose gradients the reference gets from autograd through cuBLAS):
 * T[c][d] = sum over the R rows of big[r][c] thin[r][d], big an [R, C] and thin
 * an [R, D] bf16 matrix (row-major, contiguous), written to dw (fp32) as [C][D]
 * (out_cd = 1: the gradient of w1 [C, D] from x and dh) or [D][C] (out_cd = 0:
 * the gradient of w2 [D, C] from h and dy).  C a multiple of 128, D a multiple
 * of 32 from 64 to 256; the workspace holds camoe_tm_lora_work_bytes(R, C, D)
 * bytes of per-slice partial sums, added in a fixed order (deterministic).
 * Runs on the tcgen05 tensor cores (lora_tc.cu).  R = 0 writes zeros. */
size_t camoe_tm_lora_work_bytes(int64_t R, int64_t C, int64_t D);
int camoe_tm_lora_wgrad(const void* big, const void* thin, float* dw, int out_cd, void* work,
                        size_t work_bytes, int64_t R, int64_t C, int64_t D, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CAMOE_TIMEMIX_H */
