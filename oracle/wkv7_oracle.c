/*
 * CPU oracle for the WKV-7 ClampW recurrence.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg compare
 * against it; nothing in the camoe_b200 product path links or calls it.
 *
 * Restated from the reference:
 *   decay        w = exp(W_SCALE * sigmoid(w_in)), W_SCALE = -exp(-1/2)
 *                (camoe/cuda/rwkv7_clampw.cu:16,42; camoe/backbone.py:20,272);
 *                with decay = 1, the wind_backstepping op's w = exp(-exp(w_in))
 *                (camoe/cuda/wkv7_cuda.cu:21,66-67), whose recurrence is the
 *                same with (q, z, a) in the roles of (r, a, b)
 *   forward      sa_t = S_{t-1} a_t
 *                S_t  = S_{t-1} diag(w_t) + sa_t b_t^T + v_t k_t^T
 *                y_t  = S_t r_t,  S_{-1} = 0
 *                (camoe/backbone.py:274-290; camoe/cuda/rwkv7_clampw.cu:36-74)
 *   backward     the per-element gradient formulas of
 *                camoe/cuda/rwkv7_clampw.cu:123-168 (dr, dw, dk, dv, db, the
 *                sa-gradient "dSb", da, and the dS propagation through
 *                diag(w) + a b^T), plus an optional external gradient of sa
 *                added to dSb.  Instead of reversing the state through 1/w
 *                (rwkv7_clampw.cu:133) the previous states are recomputed
 *                forward from checkpoints taken every `ckpt` steps, so the
 *                oracle's states are exactly the forward states.
 *
 * Layout: every tensor is [B, T, H, N] contiguous, element
 * ((b*T + t)*H + h)*N + i (rwkv7_clampw.cu:38).  Row index i of the state is
 * the value dimension, column j the key dimension.  Inputs and outputs are
 * float32; the arithmetic is done in REAL (double for the ground truth,
 * float for the reference-precision CPU baseline).  Chains (b, h) are
 * independent and are spread over OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define W_SCALE_D (-0.60653065971263342360)

#define ORACLE_OK 0
#define ORACLE_ERR_ARG 1
#define ORACLE_ERR_NOMEM 2

/* ------------------------------------------------------------------ */
/* Body, instantiated once for double (_f64) and once for float (_f32). */
/* ------------------------------------------------------------------ */
#define DEFINE_ORACLE(REAL, SUF, EXPF)                                                        \
/* log-decay lw(w_in): ClampW -e^{-1/2} sigmoid(w_in) (rwkv7_clampw.cu:42),                  \
 * wind_backstepping -exp(w_in) (wkv7_cuda.cu:21) */                                           \
static REAL logdecay_##SUF(REAL x, int decay)                                                  \
{                                                                                              \
    return decay ? -EXPF(x) : (REAL)W_SCALE_D / ((REAL)1 + EXPF(-x));                          \
}                                                                                              \
/* d lw / d w_in: ClampW W_SCALE s (1 - s) (rwkv7_clampw.cu:99-100,147),                      \
 * wind -exp(w_in) (wkv7_cuda.cu:66,108) */                                                    \
static REAL dlogdecay_##SUF(REAL x, int decay)                                                 \
{                                                                                              \
    if (decay) return -EXPF(x);                                                                \
    const REAL sg = (REAL)1 / ((REAL)1 + EXPF(-x));                                            \
    return (REAL)W_SCALE_D * sg * ((REAL)1 - sg);                                              \
}                                                                                              \
                                                                                               \
static void chain_fwd_##SUF(int64_t T, int64_t H, int64_t N, int64_t b, int64_t h,           \
        const float* r, const float* wi, const float* k, const float* v, const float* a,      \
        const float* bb, float* y, float* sa_out, REAL* S, REAL* sa, REAL* wv,                \
        const float* s0, float* sT, int decay)                                                 \
{                                                                                              \
    if (s0) for (int64_t e = 0; e < N * N; ++e) S[e] = (REAL)s0[e];                            \
    else memset(S, 0, sizeof(REAL) * N * N);                                                   \
    for (int64_t t = 0; t < T; ++t) {                                                          \
        const int64_t base = ((b * T + t) * H + h) * N;                                        \
        for (int64_t j = 0; j < N; ++j)                                                        \
            wv[j] = EXPF(logdecay_##SUF((REAL)wi[base + j], decay));            \
        for (int64_t i = 0; i < N; ++i) {                                                      \
            REAL acc = 0;                                                                      \
            const REAL* Si = S + i * N;                                                        \
            for (int64_t j = 0; j < N; ++j) acc += Si[j] * (REAL)a[base + j];                  \
            sa[i] = acc;                                                                       \
        }                                                                                      \
        for (int64_t i = 0; i < N; ++i) {                                                      \
            REAL* Si = S + i * N;                                                              \
            const REAL vi = (REAL)v[base + i], sai = sa[i];                                    \
            REAL acc = 0;                                                                      \
            for (int64_t j = 0; j < N; ++j) {                                                  \
                const REAL s = Si[j] * wv[j] + (sai * (REAL)bb[base + j] + (REAL)k[base + j] * vi); \
                Si[j] = s;                                                                     \
                acc += s * (REAL)r[base + j];                                                  \
            }                                                                                  \
            if (y) y[base + i] = (float)acc;                                                   \
            if (sa_out) sa_out[base + i] = (float)sai;                                         \
        }                                                                                      \
    }                                                                                          \
    if (sT) for (int64_t e = 0; e < N * N; ++e) sT[e] = (float)S[e];                           \
}                                                                                              \
                                                                                               \
/* one forward step S <- S diag(w) + sa b^T + v k^T, returning sa = S a */                     \
static void step_##SUF(int64_t N, const REAL* wv, const float* k, const float* v,             \
        const float* a, const float* bb, const REAL* Sin, REAL* Sout, REAL* sa)                \
{                                                                                              \
    for (int64_t i = 0; i < N; ++i) {                                                          \
        REAL acc = 0;                                                                          \
        const REAL* Si = Sin + i * N;                                                          \
        for (int64_t j = 0; j < N; ++j) acc += Si[j] * (REAL)a[j];                             \
        sa[i] = acc;                                                                           \
    }                                                                                          \
    for (int64_t i = 0; i < N; ++i) {                                                          \
        const REAL* Si = Sin + i * N;                                                          \
        REAL* So = Sout + i * N;                                                               \
        const REAL vi = (REAL)v[i], sai = sa[i];                                               \
        for (int64_t j = 0; j < N; ++j)                                                        \
            So[j] = Si[j] * wv[j] + (sai * (REAL)bb[j] + (REAL)k[j] * vi);                     \
    }                                                                                          \
}                                                                                              \
                                                                                               \
static int chain_bwd_##SUF(int64_t T, int64_t H, int64_t N, int64_t ck, int64_t b, int64_t h, \
        const float* r, const float* wi, const float* k, const float* v, const float* a,      \
        const float* bb, const float* dy, const float* dsa_ext,                               \
        float* dr, float* dw, float* dk, float* dv, float* da, float* db, int decay,           \
        const float* s0, const float* dsT, float* ds0)                                         \
{                                                                                              \
    const int64_t nck = (T + ck - 1) / ck;                                                     \
    const int64_t NN = N * N;                                                                  \
    REAL* ckpt = (REAL*)malloc(sizeof(REAL) * (size_t)(nck > 0 ? nck : 1) * NN);               \
    REAL* Sbuf = (REAL*)malloc(sizeof(REAL) * (size_t)(ck + 1) * NN);                          \
    REAL* sabuf = (REAL*)malloc(sizeof(REAL) * (size_t)ck * N);                                \
    REAL* wbuf = (REAL*)malloc(sizeof(REAL) * (size_t)ck * N);                                 \
    REAL* dS = (REAL*)calloc((size_t)NN, sizeof(REAL));                                        \
    REAL* dsa = (REAL*)malloc(sizeof(REAL) * (size_t)N);                                       \
    REAL* wtmp = (REAL*)malloc(sizeof(REAL) * (size_t)N);                                      \
    REAL* satmp = (REAL*)malloc(sizeof(REAL) * (size_t)N);                                     \
    if (!ckpt || !Sbuf || !sabuf || !wbuf || !dS || !dsa || !wtmp || !satmp) {                 \
        free(ckpt); free(Sbuf); free(sabuf); free(wbuf); free(dS); free(dsa); free(wtmp);     \
        free(satmp); return ORACLE_ERR_NOMEM;                                                  \
    }                                                                                          \
    /* forward pass keeping the state at the start of every checkpoint interval */             \
    if (s0) for (int64_t e = 0; e < NN; ++e) Sbuf[e] = (REAL)s0[e];                            \
    else memset(Sbuf, 0, sizeof(REAL) * NN);                                                   \
    if (dsT) for (int64_t e = 0; e < NN; ++e) dS[e] = (REAL)dsT[e];                            \
    for (int64_t c = 0; c < nck; ++c) {                                                        \
        memcpy(ckpt + c * NN, Sbuf, sizeof(REAL) * NN);                                        \
        const int64_t t1 = (c + 1) * ck < T ? (c + 1) * ck : T;                                \
        for (int64_t t = c * ck; t < t1; ++t) {                                                \
            const int64_t base = ((b * T + t) * H + h) * N;                                    \
            for (int64_t j = 0; j < N; ++j)                                                    \
                wtmp[j] = EXPF(logdecay_##SUF((REAL)wi[base + j], decay));      \
            step_##SUF(N, wtmp, k + base, v + base, a + base, bb + base, Sbuf,                 \
                       Sbuf + NN, satmp);                                                      \
            memcpy(Sbuf, Sbuf + NN, sizeof(REAL) * NN);                                        \
        }                                                                                      \
    }                                                                                          \
    /* reverse pass, one checkpoint interval at a time */                                      \
    for (int64_t c = nck - 1; c >= 0; --c) {                                                   \
        const int64_t t0 = c * ck;                                                             \
        const int64_t len = ((c + 1) * ck < T ? (c + 1) * ck : T) - t0;                        \
        memcpy(Sbuf, ckpt + c * NN, sizeof(REAL) * NN);                                        \
        for (int64_t u = 0; u < len; ++u) {                                                    \
            const int64_t base = ((b * T + t0 + u) * H + h) * N;                               \
            for (int64_t j = 0; j < N; ++j)                                                    \
                wbuf[u * N + j] = EXPF(logdecay_##SUF((REAL)wi[base + j], decay)); \
            step_##SUF(N, wbuf + u * N, k + base, v + base, a + base, bb + base,               \
                       Sbuf + u * NN, Sbuf + (u + 1) * NN, sabuf + u * N);                     \
        }                                                                                      \
        for (int64_t u = len - 1; u >= 0; --u) {                                               \
            const int64_t base = ((b * T + t0 + u) * H + h) * N;                               \
            const REAL* Sp = Sbuf + u * NN;       /* S_{t-1} */                                \
            const REAL* Sc = Sbuf + (u + 1) * NN; /* S_t */                                    \
            const REAL* sat = sabuf + u * N;                                                   \
            const REAL* wt = wbuf + u * N;                                                     \
            /* dS += dy_t r_t^T ; dr_j = sum_i S_t[i][j] dy_i */                               \
            for (int64_t i = 0; i < N; ++i) {                                                  \
                const REAL dyi = (REAL)dy[base + i];                                           \
                REAL* dSi = dS + i * N;                                                        \
                for (int64_t j = 0; j < N; ++j) dSi[j] += dyi * (REAL)r[base + j];             \
            }                                                                                  \
            for (int64_t j = 0; j < N; ++j) {                                                  \
                REAL acc = 0;                                                                  \
                for (int64_t i = 0; i < N; ++i) acc += Sc[i * N + j] * (REAL)dy[base + i];     \
                dr[base + j] = (float)acc;                                                     \
            }                                                                                  \
            /* dsa_i = sum_j dS[i][j] b_j (+ external), dv_i = sum_j dS[i][j] k_j */           \
            for (int64_t i = 0; i < N; ++i) {                                                  \
                REAL accs = dsa_ext ? (REAL)dsa_ext[base + i] : (REAL)0, accv = 0;             \
                const REAL* dSi = dS + i * N;                                                  \
                for (int64_t j = 0; j < N; ++j) {                                              \
                    accs += dSi[j] * (REAL)bb[base + j];                                       \
                    accv += dSi[j] * (REAL)k[base + j];                                        \
                }                                                                              \
                dsa[i] = accs;                                                                 \
                dv[base + i] = (float)accv;                                                    \
            }                                                                                  \
            /* column sums over i: dw, dk, db, da */                                           \
            for (int64_t j = 0; j < N; ++j) {                                                  \
                REAL aw = 0, ak = 0, ab = 0, aa = 0;                                           \
                for (int64_t i = 0; i < N; ++i) {                                              \
                    const REAL g = dS[i * N + j];                                              \
                    aw += g * Sp[i * N + j];                                                   \
                    ak += g * (REAL)v[base + i];                                               \
                    ab += g * sat[i];                                                          \
                    aa += dsa[i] * Sp[i * N + j];                                              \
                }                                                                              \
                dw[base + j] = (float)(aw * wt[j] * dlogdecay_##SUF((REAL)wi[base + j], decay)); \
                dk[base + j] = (float)ak;                                                      \
                db[base + j] = (float)ab;                                                      \
                da[base + j] = (float)aa;                                                      \
            }                                                                                  \
            /* dS_{t-1} = dS diag(w_t) + dsa a_t^T */                                          \
            for (int64_t i = 0; i < N; ++i) {                                                  \
                REAL* dSi = dS + i * N;                                                        \
                for (int64_t j = 0; j < N; ++j)                                                \
                    dSi[j] = dSi[j] * wt[j] + dsa[i] * (REAL)a[base + j];                      \
            }                                                                                  \
        }                                                                                      \
    }                                                                                          \
    if (ds0) for (int64_t e = 0; e < NN; ++e) ds0[e] = (float)dS[e];                           \
    free(ckpt); free(Sbuf); free(sabuf); free(wbuf); free(dS); free(dsa); free(wtmp);         \
    free(satmp);                                                                               \
    return ORACLE_OK;                                                                          \
}                                                                                              \
                                                                                               \
int wkv7_oracle_fwd_##SUF(int64_t B, int64_t T, int64_t H, int64_t N,                         \
        const float* r, const float* w, const float* k, const float* v, const float* a,       \
        const float* b, float* y, float* sa, int decay, int nthreads)                          \
{                                                                                              \
    if (B < 0 || T < 0 || H < 0 || N <= 0) return ORACLE_ERR_ARG;                              \
    int err = ORACLE_OK;                                                                       \
    _Pragma("omp parallel for schedule(dynamic) num_threads(nthreads > 0 ? nthreads : 1)")     \
    for (int64_t c = 0; c < B * H; ++c) {                                                      \
        REAL* S = (REAL*)malloc(sizeof(REAL) * (size_t)N * N);                                 \
        REAL* sab = (REAL*)malloc(sizeof(REAL) * (size_t)N * 2);                               \
        if (!S || !sab) { free(S); free(sab); err = ORACLE_ERR_NOMEM; continue; }              \
        chain_fwd_##SUF(T, H, N, c / H, c % H, r, w, k, v, a, b, y, sa, S, sab, sab + N,       \
                        NULL, NULL, decay);                                                    \
        free(S); free(sab);                                                                    \
    }                                                                                          \
    return err;                                                                                \
}                                                                                              \
                                                                                               \
/* Forward from a given start state: s0 (NULL = zero) and the final state sT  \
 * (NULL = not returned) are [B, H, N, N] with element ((b*H + h)*N + i)*N + j \
 * = S[i][j].  The reference has no stateful call; this is the same         \
 * recurrence with S_{-1} = s0 instead of 0, which makes a forward over     \
 * [0, T1) followed by one over [T1, T) from its final state equal a single \
 * forward over [0, T). */                                                     \
int wkv7_oracle_fwd_state_##SUF(int64_t B, int64_t T, int64_t H, int64_t N,                   \
        const float* r, const float* w, const float* k, const float* v, const float* a,       \
        const float* b, const float* s0, float* y, float* sa, float* sT, int decay,            \
        int nthreads)                                                                          \
{                                                                                              \
    if (B < 0 || T < 0 || H < 0 || N <= 0) return ORACLE_ERR_ARG;                              \
    int err = ORACLE_OK;                                                                       \
    _Pragma("omp parallel for schedule(dynamic) num_threads(nthreads > 0 ? nthreads : 1)")     \
    for (int64_t c = 0; c < B * H; ++c) {                                                      \
        REAL* S = (REAL*)malloc(sizeof(REAL) * (size_t)N * N);                                 \
        REAL* sab = (REAL*)malloc(sizeof(REAL) * (size_t)N * 2);                               \
        if (!S || !sab) { free(S); free(sab); err = ORACLE_ERR_NOMEM; continue; }              \
        chain_fwd_##SUF(T, H, N, c / H, c % H, r, w, k, v, a, b, y, sa, S, sab, sab + N,       \
                        s0 ? s0 + c * N * N : NULL, sT ? sT + c * N * N : NULL, decay);        \
        free(S); free(sab);                                                                    \
    }                                                                                          \
    return err;                                                                                \
}                                                                                              \
                                                                                               \
int wkv7_oracle_bwd_##SUF(int64_t B, int64_t T, int64_t H, int64_t N, int64_t ckpt,           \
        const float* r, const float* w, const float* k, const float* v, const float* a,       \
        const float* b, const float* dy, const float* dsa,                                    \
        float* dr, float* dw, float* dk, float* dv, float* da, float* db, int decay,           \
        int nthreads)                                                                          \
{                                                                                              \
    if (B < 0 || T < 0 || H < 0 || N <= 0 || ckpt <= 0) return ORACLE_ERR_ARG;                 \
    int err = ORACLE_OK;                                                                       \
    _Pragma("omp parallel for schedule(dynamic) num_threads(nthreads > 0 ? nthreads : 1)")     \
    for (int64_t c = 0; c < B * H; ++c) {                                                      \
        int e = chain_bwd_##SUF(T, H, N, ckpt, c / H, c % H, r, w, k, v, a, b, dy, dsa,        \
                                dr, dw, dk, dv, da, db, decay, NULL, NULL, NULL);              \
        if (e) err = e;                                                                        \
    }                                                                                          \
    return err;                                                                                \
}                                                                                              \
                                                                                               \
/* Backward of a sequence carried across calls: s0 the start state of the    \
 * forward, dsT the gradient of its final state (NULL = zero), ds0 receives   \
 * the gradient of the start state (all [B, H, N, N], NULL allowed). */         \
int wkv7_oracle_bwd_state_##SUF(int64_t B, int64_t T, int64_t H, int64_t N, int64_t ckpt,     \
        const float* r, const float* w, const float* k, const float* v, const float* a,       \
        const float* b, const float* dy, const float* dsa, const float* s0, const float* dsT,  \
        float* ds0, float* dr, float* dw, float* dk, float* dv, float* da, float* db,          \
        int decay, int nthreads)                                                               \
{                                                                                              \
    if (B < 0 || T < 0 || H < 0 || N <= 0 || ckpt <= 0) return ORACLE_ERR_ARG;                 \
    int err = ORACLE_OK;                                                                       \
    _Pragma("omp parallel for schedule(dynamic) num_threads(nthreads > 0 ? nthreads : 1)")     \
    for (int64_t c = 0; c < B * H; ++c) {                                                      \
        int e = chain_bwd_##SUF(T, H, N, ckpt, c / H, c % H, r, w, k, v, a, b, dy, dsa,        \
                                dr, dw, dk, dv, da, db, decay, s0 ? s0 + c * N * N : NULL,     \
                                dsT ? dsT + c * N * N : NULL, ds0 ? ds0 + c * N * N : NULL);   \
        if (e) err = e;                                                                        \
    }                                                                                          \
    return err;                                                                                \
}

DEFINE_ORACLE(double, f64, exp)
DEFINE_ORACLE(float, f32, expf)

/* Transition decay as the reference computes it, exposed for tests. */
double wkv7_oracle_decay(double w_in) { return exp(W_SCALE_D / (1.0 + exp(-w_in))); }
