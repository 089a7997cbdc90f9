/*
 * k-mamba block and model API (reference include/kmamba.h:228-321) on the
 * B200: every arithmetic step of the block forward / backward, the LM head,
 * the softmax cross-entropy, the gradient norms and the optimizers runs on
 * the device (csrc/cuda/block.cu).
 *
 * Data flow of one call: the host arrays of the MambaBlock / KMamba structs
 * stay the source of truth (callers read and write them directly, as with
 * the reference).  A call stages the tensors it needs on the device
 * (kmb_stage_in / kmb_stage_out: pooled device buffers, or the caller's
 * own pointer when it is already device memory), runs the kernels on the
 * library stream and copies the updated tensors back in kmb_stage_finish.
 *
 * Token layout of a block call: rows = batch * seq_len, channel-last
 * [rows, dim].  The five input projections write one [rows, W] matrix
 * with W = R + 2 + 2*N*R columns: u (R) | dt (1) | lambda (1) | B (N*R) |
 * C (N*R), the order in which the reference evaluates them
 * (src/mamba_block.c:89-120, :483-491).
 *
 * Error behaviour follows the reference: void functions return silently on
 * invalid input, int functions return -1, float functions return NAN; the
 * reason is recorded for kmb_last_error().
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../kmb_internal.h"
#include "kmamba.h"
#include "kmamba_resident.h"

/* ------------------------------------------------------------------ */
/* block tensor tables                                                 */
/* ------------------------------------------------------------------ */

/* Parameter order used for staging, gradients and moments. */
enum {
    P_WIN,
    P_DP,
    P_LP,
    P_WB,
    P_WC,
    P_BB,
    P_BC,
    P_A,
    P_TH,
    P_WOUT,
    P_COUNT
};

static size_t blk_R(const MBConfig *c) { return c->mimo_rank > 1 ? c->mimo_rank : 1; }
static size_t blk_TS(const MBConfig *c) { return c->state_size / 2 > 0 ? c->state_size / 2 : 1; }

typedef struct {
    int D, N, R, NR, W, TS;
    int has_dp, has_lp;
    size_t n[P_COUNT];
} BlockDims;

static BlockDims block_dims(const MambaBlock *b) {
    BlockDims d;
    d.D = (int)b->config.dim;
    d.N = (int)b->config.state_size;
    d.R = (int)blk_R(&b->config);
    d.NR = d.N * d.R;
    d.W = d.R + 2 + 2 * d.NR;
    d.TS = (int)blk_TS(&b->config);
    d.has_dp = b->delta_proj.rows > 0 && b->delta_proj.data != NULL;
    d.has_lp = b->lambda_proj.rows > 0 && b->lambda_proj.data != NULL;
    d.n[P_WIN] = (size_t)d.R * d.D;
    d.n[P_DP] = (size_t)d.D;
    d.n[P_LP] = (size_t)d.D;
    d.n[P_WB] = (size_t)d.NR * d.D;
    d.n[P_WC] = (size_t)d.NR * d.D;
    d.n[P_BB] = (size_t)d.NR;
    d.n[P_BC] = (size_t)d.NR;
    d.n[P_A] = (size_t)d.N;
    d.n[P_TH] = (size_t)d.TS;
    d.n[P_WOUT] = (size_t)d.D * d.R;
    return d;
}

static void block_param_ptrs(const MambaBlock *b, float **p) {
    p[P_WIN] = b->W_in.data;
    p[P_DP] = b->delta_proj.data;
    p[P_LP] = b->lambda_proj.data;
    p[P_WB] = b->W_B.data;
    p[P_WC] = b->W_C.data;
    p[P_BB] = b->b_B;
    p[P_BC] = b->b_C;
    p[P_A] = b->A_log.data;
    p[P_TH] = b->theta;
    p[P_WOUT] = b->W_out.data;
}

static void optstate_grad_ptrs(const MBOptimState *s, float **g) {
    g[P_WIN] = s->g_W_in;
    g[P_DP] = s->g_delta_proj;
    g[P_LP] = s->g_lambda_proj;
    g[P_WB] = s->g_W_B;
    g[P_WC] = s->g_W_C;
    g[P_BB] = s->g_b_B;
    g[P_BC] = s->g_b_C;
    g[P_A] = s->g_A_log;
    g[P_TH] = s->g_theta;
    g[P_WOUT] = s->g_W_out;
}

static void optstate_moment_ptrs(const MBOptimState *s, float **m, float **v) {
    m[P_WIN] = s->m_W_in;
    m[P_DP] = s->m_delta_proj;
    m[P_LP] = s->m_lambda_proj;
    m[P_WB] = s->m_W_B;
    m[P_WC] = s->m_W_C;
    m[P_BB] = s->m_b_B;
    m[P_BC] = s->m_b_C;
    m[P_A] = s->m_A_log;
    m[P_TH] = s->m_theta;
    m[P_WOUT] = s->m_W_out;
    v[P_WIN] = s->v_W_in;
    v[P_DP] = s->v_delta_proj;
    v[P_LP] = s->v_lambda_proj;
    v[P_WB] = s->v_W_B;
    v[P_WC] = s->v_W_C;
    v[P_BB] = s->v_b_B;
    v[P_BC] = s->v_b_C;
    v[P_A] = s->v_A_log;
    v[P_TH] = s->v_theta;
    v[P_WOUT] = s->v_W_out;
}

/* Device view of one block for the duration of a call. */
typedef struct {
    BlockDims d;
    MBConfig cfg;
    float *p[P_COUNT]; /* parameters */
    float *g[P_COUNT]; /* gradients (NULL: parameter gradients not wanted) */
    float *m[P_COUNT]; /* first moments (NULL when no optimizer step) */
    float *v[P_COUNT]; /* second moments (AdamW) */
    float *ws;         /* split-K workspace of the call (KMB_GEMM_WS floats) */
} DevBlock;

/* Split-K workspace per call: the split count is at most ceil(296 / tiles)
 * for tiles < 148 64x64 output tiles, so S * M * N stays below
 * (296 + 148) * 4096 floats. */
#define KMB_GEMM_WS ((size_t)(296 + 148) * 4096)

static float *gemm_ws(KmbStage *st) {
    return (float *)kmb_scratch(st, KMB_GEMM_WS * sizeof(float));
}

static int block_check(const MambaBlock *b) {
    BlockDims d;
    if (!b) return kmb_fail(KMB_EINVAL, "block: NULL block");
    d = block_dims(b);
    if (d.D <= 0 || d.N <= 0 || b->config.seq_len == 0)
        return kmb_fail(KMB_EINVAL, "block: dim, state_size and seq_len must be > 0");
    if (!b->W_in.data || !b->W_out.data || !b->A_log.data || !b->W_B.data || !b->W_C.data ||
        !b->b_B || !b->b_C || !b->theta)
        return kmb_fail(KMB_EINVAL, "block: parameters not allocated");
    if (d.R > 8) return kmb_fail(KMB_EUNSUPPORTED, "block: mimo_rank %d exceeds 8", d.R);
    if (d.N > 2048) return kmb_fail(KMB_EUNSUPPORTED, "block: state_size %d exceeds 2048", d.N);
    return KMB_OK;
}

/* Stages the parameters (updated in place when `writeback`), the gradient
 * buffers `g` (host arrays, accumulated when `g_accumulate`, else zeroed on
 * the device) and, when `mv` is set, the optimizer moments.  `ws` is the
 * call's split-K workspace (NULL when the call runs no block GEMM). */
static int dev_block_stage(KmbStage *st, const MambaBlock *b, DevBlock *db, int writeback,
                           float **g, int g_accumulate, int mv, float *ws) {
    float *hp[P_COUNT];
    memset(db, 0, sizeof *db);
    db->d = block_dims(b);
    db->cfg = b->config;
    db->ws = ws;
    block_param_ptrs(b, hp);
    for (int i = 0; i < P_COUNT; ++i) {
        const size_t bytes = db->d.n[i] * sizeof(float);
        if (!hp[i]) { /* absent projection (rows == 0): a zero row keeps the GEMMs uniform */
            db->p[i] = (float *)kmb_scratch(st, bytes);
            if (db->p[i]) cudaMemsetAsync(db->p[i], 0, bytes, st->s);
        } else if (writeback) {
            db->p[i] = (float *)kmb_stage_out(st, hp[i], bytes, 1);
        } else {
            db->p[i] = (float *)kmb_stage_in(st, hp[i], bytes);
        }
        if (!db->p[i]) return st->status ? st->status : kmb_fail(KMB_ENOMEM, "block staging");
    }
    if (g) {
        for (int i = 0; i < P_COUNT; ++i) {
            const size_t bytes = db->d.n[i] * sizeof(float);
            if (!g[i]) return kmb_fail(KMB_EINVAL, "block: gradient buffer %d missing", i);
            db->g[i] = (float *)kmb_stage_out(st, g[i], bytes, g_accumulate);
            if (!db->g[i]) return st->status ? st->status : kmb_fail(KMB_ENOMEM, "block staging");
            if (!g_accumulate) {
                cudaError_t e = cudaMemsetAsync(db->g[i], 0, bytes, st->s);
                if (e != cudaSuccess) return kmb_cuda_fail(e, "gradient zeroing");
            }
        }
    }
    if (mv) {
        const MBOptimState *s = b->opt_state;
        float *hm[P_COUNT], *hv[P_COUNT];
        optstate_moment_ptrs(s, hm, hv);
        for (int i = 0; i < P_COUNT; ++i) {
            const size_t bytes = db->d.n[i] * sizeof(float);
            if (hm[i]) {
                db->m[i] = (float *)kmb_stage_out(st, hm[i], bytes, 1);
                if (!db->m[i]) return st->status;
            }
            if (hv[i]) {
                db->v[i] = (float *)kmb_stage_out(st, hv[i], bytes, 1);
                if (!db->v[i]) return st->status;
            }
        }
    }
    return KMB_OK;
}

/* Forward activations of one block kept for its backward. */
typedef struct {
    float *zraw; /* [rows, W] projections before activation */
    float *zact; /* [rows, W] after activation (+ bias) */
    float *hh;   /* [rows, N] state history, or NULL */
    float *y;    /* [rows, R] scan output */
    float *part; /* [rows, warps per sequence, R + 2] scan partial sums */
} BlockActs;

static int acts_alloc(KmbStage *st, const BlockDims *d, long rows, int hist, BlockActs *a) {
    a->zraw = (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * d->W);
    a->zact = (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * d->W);
    a->y = (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * d->R);
    a->hh = hist ? (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * d->N) : NULL;
    a->part = (float *)kmb_scratch(
        st, sizeof(float) * (size_t)rows * kmb_m3_scan_groups(d->N) * (d->R + 2));
    if (!a->zraw || !a->zact || !a->y || (hist && !a->hh) || !a->part)
        return st->status ? st->status : kmb_fail(KMB_ENOMEM, "block activations");
    return KMB_OK;
}

#define TRY(x)                       \
    do {                             \
        int rc_ = (x);               \
        if (rc_ != KMB_OK) return rc_; \
    } while (0)

/* out[rows, D] = x + W_out * scan(act(x * Wcat^T)).  x and out may not
 * alias.  h_last [batch, N] receives the final states when non-NULL. */
static int blk_forward(const DevBlock *db, const float *x, float *out, long batch, long L,
                       BlockActs *a, float *h_last, cudaStream_t s) {
    const BlockDims *d = &db->d;
    const long rows = batch * L;
    const int D = d->D, R = d->R, NR = d->NR, W = d->W;
    const int c_off[5] = {0, R, R + 1, R + 2, R + 2 + NR};
    const int c_n[5] = {R, 1, 1, NR, NR};
    const float *wp[5] = {db->p[P_WIN], db->p[P_DP], db->p[P_LP], db->p[P_WB], db->p[P_WC]};
    cudaError_t e;
    /* Z[:, c0:c0+n] = X Wpart^T  (Wpart [n, D] row-major) */
    for (int k = 0; k < 5; ++k)
        TRY(kmb_gemm((int)rows, c_n[k], D, x, D, 1, wp[k], 1, D, a->zraw + c_off[k], W, 0,
                     db->ws, KMB_GEMM_WS, s));
    TRY(kmb_block_act(a->zraw, a->zact, db->p[P_BB], db->p[P_BC], rows, W, R, NR,
                      db->cfg.dt_min, db->cfg.dt_max, d->has_dp, d->has_lp, db->cfg.dt_scale,
                      NULL, s));
    TRY(kmb_m3_scan((int)batch, (int)L, d->N, R, W, a->zact, db->p[P_A], db->p[P_TH], a->hh,
                    h_last, a->y, NULL, NULL, NULL, NULL, a->part, s));
    /* out = x + y W_out^T  (W_out [D, R]) */
    e = cudaMemcpyAsync(out, x, sizeof(float) * (size_t)rows * D, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "block residual copy");
    return kmb_gemm((int)rows, D, R, a->y, R, 1, db->p[P_WOUT], 1, R, out, D, 1, db->ws,
                    KMB_GEMM_WS, s);
}

/* Adjoint of blk_forward: dx = dY + d(block)/dx^T dY; parameter gradients
 * are accumulated into db->g when set.  `a` must hold the activations of
 * the same x (with the state history).  dz [rows, W] and dyr [rows, R]
 * are scratch. */
static int blk_backward(const DevBlock *db, const float *x, const BlockActs *a, const float *dY,
                        float *dx, long batch, long L, float *dz, float *dyr, float *dA_tmp,
                        float *dth_tmp, cudaStream_t s) {
    const BlockDims *d = &db->d;
    const long rows = batch * L;
    const int D = d->D, R = d->R, NR = d->NR, W = d->W;
    const int c_off[5] = {0, R, R + 1, R + 2, R + 2 + NR};
    const int c_n[5] = {R, 1, 1, NR, NR};
    const int gi[5] = {P_WIN, P_DP, P_LP, P_WB, P_WC};
    float *dA = db->g[P_A] ? db->g[P_A] : dA_tmp;
    float *dth = db->g[P_TH] ? db->g[P_TH] : dth_tmp;
    cudaError_t e;

    /* dy_r[t, r] = sum_d dY[t, d] W_out[d, r] */
    TRY(kmb_gemm((int)rows, R, D, dY, D, 1, db->p[P_WOUT], R, 1, dyr, R, 0, db->ws,
                 KMB_GEMM_WS, s));
    /* g_W_out[d, r] += sum_t dY[t, d] y[t, r] */
    if (db->g[P_WOUT])
        TRY(kmb_gemm(D, R, (int)rows, dY, 1, D, a->y, R, 1, db->g[P_WOUT], R, 1, db->ws,
                     KMB_GEMM_WS, s));
    /* scan adjoint: dz (all W columns), dA, dtheta */
    TRY(kmb_m3_scan((int)batch, (int)L, d->N, R, W, a->zact, db->p[P_A], db->p[P_TH], a->hh,
                    NULL, (float *)a->y, dyr, dz, dA, dth, a->part, s));
    /* activations: dz becomes the gradient of the raw projections */
    TRY(kmb_block_act(a->zraw, a->zact, db->p[P_BB], db->p[P_BC], rows, W, R, NR,
                      db->cfg.dt_min, db->cfg.dt_max, d->has_dp, d->has_lp, db->cfg.dt_scale,
                      dz, s));
    if (db->g[P_BB]) {
        TRY(kmb_colsum_acc(dz, rows, W, R + 2, NR, db->g[P_BB], s));
        TRY(kmb_colsum_acc(dz, rows, W, R + 2 + NR, NR, db->g[P_BC], s));
    }
    /* g_Wpart[c, k] += sum_t dz[t, c0 + c] x[t, k] */
    if (db->g[P_WIN]) {
        for (int k = 0; k < 5; ++k) {
            if ((k == 1 && !d->has_dp) || (k == 2 && !d->has_lp)) continue;
            TRY(kmb_gemm(c_n[k], D, (int)rows, dz + c_off[k], 1, W, x, D, 1, db->g[gi[k]], D, 1,
                         db->ws, KMB_GEMM_WS, s));
        }
    }
    /* dx = dY + dz Wcat */
    if (dx) {
        const float *wp[5] = {db->p[P_WIN], db->p[P_DP], db->p[P_LP], db->p[P_WB], db->p[P_WC]};
        if (dx != dY) {
            e = cudaMemcpyAsync(dx, dY, sizeof(float) * (size_t)rows * D, cudaMemcpyDeviceToDevice,
                                s);
            if (e != cudaSuccess) return kmb_cuda_fail(e, "block residual gradient copy");
        }
        for (int k = 0; k < 5; ++k)
            TRY(kmb_gemm((int)rows, D, c_n[k], dz + c_off[k], W, 1, wp[k], D, 1, dx, D, 1,
                         db->ws, KMB_GEMM_WS, s));
    }
    return KMB_OK;
}

/* Scratch of one block backward. */
typedef struct {
    float *dz, *dyr, *dA, *dth;
} BwdScratch;

static int bwd_scratch(KmbStage *st, const BlockDims *d, long rows, BwdScratch *b) {
    b->dz = (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * d->W);
    b->dyr = (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * d->R);
    b->dA = (float *)kmb_scratch(st, sizeof(float) * (size_t)d->N);
    b->dth = (float *)kmb_scratch(st, sizeof(float) * (size_t)d->TS);
    if (!b->dz || !b->dyr || !b->dA || !b->dth)
        return st->status ? st->status : kmb_fail(KMB_ENOMEM, "block backward scratch");
    return KMB_OK;
}

/* Squared-norm slots: one double per parameter tensor, zeroed here. */
static int blk_sumsq(const DevBlock *db, double *slots, cudaStream_t s) {
    const float *x[P_COUNT];
    double *out[P_COUNT];
    long n[P_COUNT];
    cudaError_t e = cudaMemsetAsync(slots, 0, sizeof(double) * P_COUNT, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "sumsq zeroing");
    for (int i = 0; i < P_COUNT; ++i) {
        x[i] = db->g[i];
        n[i] = (long)db->d.n[i];
        out[i] = slots + i;
    }
    return kmb_sumsq_multi(P_COUNT, x, n, out, s);
}

/* Reference summation order of mamba_block_grad_sqnorm
 * (src/mamba_block.c:354-371): W_in, W_out, A_log, W_B, W_C, b_B, b_C,
 * delta_proj, lambda_proj, theta. */
static double blk_sqnorm_host(const double *slots) {
    static const int order[P_COUNT] = {P_WIN, P_WOUT, P_A, P_WB, P_WC, P_BB, P_BC, P_DP, P_LP, P_TH};
    double acc = 0.0;
    for (int i = 0; i < P_COUNT; ++i) {
        const float n = sqrtf((float)slots[order[i]]);
        acc += (double)n * n;
    }
    return acc;
}

/* MUON matrix update (kernels/optimizer_f32.c:130-161): m = mu m + g;
 * G = m orthogonalised by 5 Newton-Schulz steps G <- 1.5G - 0.5 G G^T G;
 * p -= lr * G * min(1, clip/||G||). */
static int muon_mat(KmbStage *st, float *p, const float *g, float *m, int rows, int cols,
                    const MBOptimConfig *c, double *slot, cudaStream_t s) {
    const long n = (long)rows * cols;
    float *G = (float *)kmb_scratch(st, sizeof(float) * (size_t)n);
    float *T = (float *)kmb_scratch(st, sizeof(float) * (size_t)n);
    float *GG = (float *)kmb_scratch(st, sizeof(float) * (size_t)rows * rows);
    cudaError_t e;
    if (!G || !T || !GG) return st->status;
    TRY(kmb_momentum(m, g, n, c->mu, s));
    e = cudaMemcpyAsync(G, m, sizeof(float) * (size_t)n, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "muon copy");
    for (int it = 0; it < 5; ++it) {
        /* GG[i, j] = sum_k G[i, k] G[j, k] */
        TRY(kmb_gemm(rows, rows, cols, G, cols, 1, G, 1, cols, GG, rows, 0, NULL, 0, s));
        /* T = GG G */
        TRY(kmb_gemm(rows, cols, rows, GG, rows, 1, G, cols, 1, T, cols, 0, NULL, 0, s));
        TRY(kmb_ns_combine(G, T, n, s));
    }
    e = cudaMemsetAsync(slot, 0, sizeof(double), s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "muon norm zeroing");
    TRY(kmb_sumsq(G, n, slot, s));
    return kmb_scaled_sub(p, G, n, c->lr, c->clip_norm, slot, s);
}

/* MUON vector update (kernels/optimizer_f32.c:110-127). */
static int muon_vec(float *p, const float *g, float *m, long n, const MBOptimConfig *c,
                    double *slot, cudaStream_t s) {
    cudaError_t e;
    TRY(kmb_momentum(m, g, n, c->mu, s));
    e = cudaMemsetAsync(slot, 0, sizeof(double), s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "muon norm zeroing");
    TRY(kmb_sumsq(m, n, slot, s));
    return kmb_scaled_sub(p, m, n, c->lr, c->clip_norm, slot, s);
}

/* One optimizer step of a staged block (src/mamba_block.c:373-408).  The
 * reference runs AdamW for every type but MUON (ADAM_CLIP is AdamW; it
 * does not clip).  SGD, whose moments the reference never allocates, is
 * plain p -= lr g here. */
static int blk_opt_step(KmbStage *st, const DevBlock *db, OptimizerType type, size_t step,
                        const MBOptimConfig *c, double *slots, cudaStream_t s) {
    const BlockDims *d = &db->d;
    if (type == OPTIMIZER_MUON) {
        const int mat_rows[P_COUNT] = {d->R, 0, 0, d->NR, d->NR, 0, 0, 0, 0, d->D};
        const int mat_cols[P_COUNT] = {d->D, 0, 0, d->D, d->D, 0, 0, 0, 0, d->R};
        for (int i = 0; i < P_COUNT; ++i) {
            if (!db->m[i]) return kmb_fail(KMB_EINVAL, "MUON: momentum buffers missing");
            if (mat_rows[i])
                TRY(muon_mat(st, db->p[i], db->g[i], db->m[i], mat_rows[i], mat_cols[i], c,
                             slots + i, s));
            else
                TRY(muon_vec(db->p[i], db->g[i], db->m[i], (long)d->n[i], c, slots + i, s));
        }
        return KMB_OK;
    }
    if (type == OPTIMIZER_SGD) {
        for (int i = 0; i < P_COUNT; ++i)
            TRY(kmb_scaled_sub(db->p[i], db->g[i], (long)d->n[i], c->lr, 0.f, NULL, s));
        return KMB_OK;
    }
    {
        const float bc1 = 1.0f - powf(0.9f, (float)step);
        const float bc2 = 1.0f - powf(0.999f, (float)step);
        long n[P_COUNT];
        for (int i = 0; i < P_COUNT; ++i) {
            if (!db->m[i] || !db->v[i]) return kmb_fail(KMB_EINVAL, "AdamW: moment buffers missing");
            n[i] = (long)d->n[i];
        }
        return kmb_adamw_multi(P_COUNT, db->p, (const float *const *)db->g, db->m, db->v, n,
                               c->lr, 0.9f, 0.999f, c->eps, c->weight_decay, bc1, bc2, s);
    }
}

/* ------------------------------------------------------------------ */
/* block lifecycle (host memory, reference layout)                     */
/* ------------------------------------------------------------------ */

/*
 * Tensors that every call copies to and from the device (parameters,
 * gradients, optimizer moments, embedding, head) live in page-locked host
 * memory when a GPU is present, so those copies run at the full PCIe rate.
 * Without a GPU (host-only use: create, init, save, load) they are ordinary
 * zeroed heap memory.  pinned_free tells the two apart.
 */
static int g_pinned = -1; /* -1 unknown, 0 no pinned allocation possible, 1 ok */

static void *pinned_calloc(size_t n, size_t sz) {
    const size_t bytes = (n ? n : 1) * sz;
    void *p = NULL;
    if (__atomic_load_n(&g_pinned, __ATOMIC_RELAXED) != 0) {
        if (cudaMallocHost(&p, bytes) == cudaSuccess) {
            __atomic_store_n(&g_pinned, 1, __ATOMIC_RELAXED);
            memset(p, 0, bytes);
            return p;
        }
        (void)cudaGetLastError();
        if (__atomic_load_n(&g_pinned, __ATOMIC_RELAXED) == -1)
            __atomic_store_n(&g_pinned, 0, __ATOMIC_RELAXED);
    }
    return calloc(1, bytes);
}

static void pinned_free(void *p) {
    struct cudaPointerAttributes at;
    if (!p) return;
    if (__atomic_load_n(&g_pinned, __ATOMIC_RELAXED) == 1 &&
        cudaPointerGetAttributes(&at, p) == cudaSuccess && at.type == cudaMemoryTypeHost) {
        cudaFreeHost(p);
        return;
    }
    (void)cudaGetLastError();
    free(p);
}

static int mat_alloc(MBMatrix *m, size_t rows, size_t cols) {
    m->rows = rows;
    m->cols = cols;
    m->data = (float *)pinned_calloc(rows * cols, sizeof(float));
    return m->data ? 0 : -1;
}

MambaBlock *mamba_block_create(const MBConfig *config) {
    MambaBlock *b;
    size_t R, N, D, L;
    if (!config) return NULL;
    b = (MambaBlock *)calloc(1, sizeof *b);
    if (!b) return NULL;
    b->config = *config;
    if (b->config.mimo_rank == 0) b->config.mimo_rank = 1;
    if (km_normalize_spatial_topology(&b->config.spatial_ndims, b->config.spatial_dims,
                                      (long)b->config.seq_len, b->config.use_convnd,
                                      &b->config.convnd_ndims, b->config.convnd_K) != 0) {
        free(b);
        return NULL;
    }
    R = blk_R(&b->config);
    N = b->config.state_size;
    D = b->config.dim;
    L = b->config.seq_len;
    if (mat_alloc(&b->W_in, R, D) || mat_alloc(&b->W_out, D, R) || mat_alloc(&b->A_log, N, 1) ||
        mat_alloc(&b->W_B, N * R, D) || mat_alloc(&b->W_C, N * R, D) ||
        mat_alloc(&b->delta_proj, 1, D) || mat_alloc(&b->lambda_proj, 1, D)) {
        mamba_block_free(b);
        return NULL;
    }
    b->b_B = (float *)pinned_calloc(N * R, sizeof(float));
    b->b_C = (float *)pinned_calloc(N * R, sizeof(float));
    b->theta = (float *)pinned_calloc(blk_TS(&b->config), sizeof(float));
    b->hidden = (float *)calloc(N + 1, sizeof(float));
    b->delta = (float *)calloc(L + 1, sizeof(float));
    b->scan_B = (float *)calloc(L * N * R + 1, sizeof(float));
    b->scan_C = (float *)calloc(L * N * R + 1, sizeof(float));
    b->scan_delta = (float *)calloc(L * N + 1, sizeof(float));
    b->scan_h = (float *)calloc(N + 1, sizeof(float));
    b->wavefront_plan = km_wavefront_plan_create(b->config.spatial_dims, b->config.spatial_ndims);
    if (!b->b_B || !b->b_C || !b->theta || !b->hidden || !b->delta || !b->scan_B || !b->scan_C ||
        !b->scan_delta || !b->scan_h || !b->wavefront_plan) {
        mamba_block_free(b);
        return NULL;
    }
    if (b->config.use_convnd && b->config.convnd_K > 0) {
        /* dense K^ndims x dim depthwise kernel (convnd.h layout); the
         * reference sizes this buffer in bytes and then overruns it
         * (src/mamba_block.c:223-234) */
        long vol = 1, nd = b->config.convnd_ndims > 0 ? b->config.convnd_ndims
                                                       : b->config.spatial_ndims;
        for (long i = 0; i < nd; ++i) vol *= b->config.convnd_K;
        b->convnd_kernel = (float *)calloc((size_t)vol * D, sizeof(float));
        b->convnd_bias = (float *)calloc(D, sizeof(float));
        if (!b->convnd_kernel || !b->convnd_bias) {
            mamba_block_free(b);
            return NULL;
        }
    }
    return b;
}

void mamba_block_free(MambaBlock *b) {
    if (!b) return;
    mamba_free_optimizer(b);
    pinned_free(b->W_in.data);
    pinned_free(b->W_out.data);
    pinned_free(b->A_log.data);
    pinned_free(b->W_B.data);
    pinned_free(b->W_C.data);
    pinned_free(b->delta_proj.data);
    pinned_free(b->lambda_proj.data);
    pinned_free(b->b_B);
    pinned_free(b->b_C);
    pinned_free(b->theta);
    free(b->hidden);
    free(b->delta);
    free(b->scan_B);
    free(b->scan_C);
    free(b->scan_delta);
    free(b->scan_h);
    if (b->wavefront_plan) km_wavefront_plan_free(b->wavefront_plan);
    free(b->convnd_kernel);
    free(b->convnd_bias);
    free(b);
}

/* Same rand() sequence as the reference initialiser
 * (src/mamba_block.c:269-293), so a seeded model has identical weights. */
void mamba_block_init(MambaBlock *b) {
    MBMatrix *mats[4];
    size_t R, N;
    float base;
    if (!b) return;
    for (size_t i = 0; i < b->config.state_size; ++i) b->A_log.data[i] = -1.0f;
    mats[0] = &b->W_in;
    mats[1] = &b->W_out;
    mats[2] = &b->W_B;
    mats[3] = &b->W_C;
    for (int k = 0; k < 4; ++k) {
        MBMatrix *M = mats[k];
        const float scale = sqrtf(6.0f / (float)(M->rows + M->cols));
        for (size_t i = 0; i < M->rows * M->cols; ++i)
            M->data[i] = ((float)rand() / RAND_MAX * 2.0f - 1.0f) * scale;
    }
    R = blk_R(&b->config);
    N = b->config.state_size;
    memset(b->b_B, 0, N * R * sizeof(float));
    memset(b->b_C, 0, N * R * sizeof(float));
    base = 2.0f * 3.14159f / (float)N;
    for (size_t i = 0; i < blk_TS(&b->config); ++i)
        b->theta[i] = ((float)rand() / RAND_MAX) * base;
    for (size_t i = 0; i < b->delta_proj.rows * b->delta_proj.cols; ++i)
        b->delta_proj.data[i] = ((float)rand() / RAND_MAX - 0.5f) * 0.02f;
    for (size_t i = 0; i < b->lambda_proj.rows * b->lambda_proj.cols; ++i)
        b->lambda_proj.data[i] = ((float)rand() / RAND_MAX - 0.5f) * 0.02f;
}

MambaBlockWorkspace *mamba_block_workspace_create(const MambaBlock *b) {
    MambaBlockWorkspace *ws;
    size_t N, L, R;
    if (!b) return NULL;
    ws = (MambaBlockWorkspace *)calloc(1, sizeof *ws);
    if (!ws) return NULL;
    N = b->config.state_size;
    L = b->config.seq_len;
    R = blk_R(&b->config);
    ws->hidden = (float *)calloc(N + 1, sizeof(float));
    ws->delta = (float *)calloc(L + 1, sizeof(float));
    ws->scan_B = (float *)calloc(L * N * R + 1, sizeof(float));
    ws->scan_C = (float *)calloc(L * N * R + 1, sizeof(float));
    ws->scan_delta = (float *)calloc(L * N + 1, sizeof(float));
    ws->scan_h = (float *)calloc(N + 1, sizeof(float));
    if (!ws->hidden || !ws->delta || !ws->scan_B || !ws->scan_C || !ws->scan_delta ||
        !ws->scan_h) {
        mamba_block_workspace_free(ws);
        return NULL;
    }
    return ws;
}

void mamba_block_workspace_free(MambaBlockWorkspace *ws) {
    if (!ws) return;
    free(ws->hidden);
    free(ws->delta);
    free(ws->scan_B);
    free(ws->scan_C);
    free(ws->scan_delta);
    free(ws->scan_h);
    free(ws);
}

/* ------------------------------------------------------------------ */
/* block forward                                                       */
/* ------------------------------------------------------------------ */

/* Copies column block [c0, c0+n) of `rows` rows of a [*, W] device matrix
 * to a dense host array. */
static int copy_cols_to_host(float *dst, const float *src, long rows, int W, int c0, int n,
                             cudaStream_t s) {
    cudaError_t e = cudaMemcpy2DAsync(dst, sizeof(float) * (size_t)n, src + c0,
                                      sizeof(float) * (size_t)W, sizeof(float) * (size_t)n,
                                      (size_t)rows, cudaMemcpyDeviceToHost, s);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "workspace copy");
}

static int block_forward_impl(MambaBlock *b, MambaBlockWorkspace *ws, float *output,
                              const float *input, size_t batch) {
    KmbStage st;
    DevBlock db;
    BlockActs a;
    const float *x;
    float *out, *hl = NULL;
    long L, rows;
    size_t io_bytes;
    int rc;
    if (!output || !input) return kmb_fail(KMB_EINVAL, "mamba_block_forward: NULL buffer");
    TRY(block_check(b));
    if (batch == 0) return KMB_OK;
    L = (long)b->config.seq_len;
    rows = (long)batch * L;
    io_bytes = sizeof(float) * (size_t)rows * b->config.dim;
    kmb_stage_begin(&st);
    rc = dev_block_stage(&st, b, &db, 0, NULL, 0, 0, gemm_ws(&st));
    if (rc == KMB_OK) {
        x = (const float *)kmb_stage_in(&st, input, io_bytes);
        out = (float *)kmb_stage_out(&st, output, io_bytes, 0);
        if (ws) hl = (float *)kmb_scratch(&st, sizeof(float) * (size_t)batch * db.d.N);
        rc = st.status;
        if (rc == KMB_OK && x == out) rc = kmb_fail(KMB_EINVAL, "block forward: output aliases input");
        if (rc == KMB_OK) rc = acts_alloc(&st, &db.d, rows, 0, &a);
        if (rc == KMB_OK) rc = blk_forward(&db, x, out, (long)batch, L, &a, hl, st.s);
        if (rc == KMB_OK && ws) {
            /* the reference leaves the last batch item's controls in ws */
            const long r0 = rows - L;
            const int R = db.d.R, NR = db.d.NR, W = db.d.W;
            rc = copy_cols_to_host(ws->delta, a.zact + r0 * W, L, W, R, 1, st.s);
            if (rc == KMB_OK)
                rc = copy_cols_to_host(ws->scan_B, a.zact + r0 * W, L, W, R + 2, NR, st.s);
            if (rc == KMB_OK)
                rc = copy_cols_to_host(ws->scan_C, a.zact + r0 * W, L, W, R + 2 + NR, NR, st.s);
            if (rc == KMB_OK) {
                cudaError_t e = cudaMemcpyAsync(ws->scan_h, hl + (long)(batch - 1) * db.d.N,
                                                sizeof(float) * db.d.N, cudaMemcpyDeviceToHost,
                                                st.s);
                if (e != cudaSuccess) rc = kmb_cuda_fail(e, "workspace state copy");
            }
        }
    }
    return kmb_stage_finish(&st, rc);
}

void mamba_block_forward(MambaBlock *b, float *output, const float *input, size_t batch) {
    (void)block_forward_impl(b, NULL, output, input, batch);
}

void mamba_block_forward_ws(MambaBlock *b, MambaBlockWorkspace *ws, float *output,
                            const float *input, size_t batch) {
    (void)block_forward_impl(b, ws, output, input, batch);
}

/* ------------------------------------------------------------------ */
/* block backward                                                      */
/* ------------------------------------------------------------------ */

/* One sequence [seq_len, dim]: recomputes the forward of `input`, then the
 * adjoint.  Gradients accumulate into `gsrc` (an MBOptimState whose g_*
 * arrays are set) when non-NULL; d_input is overwritten when non-NULL. */
static int block_backward_impl(MambaBlock *b, const float *dY, const float *input,
                               float *d_input, const MBOptimState *gsrc) {
    KmbStage st;
    DevBlock db;
    BlockActs a;
    BwdScratch bs;
    float *g[P_COUNT];
    const float *x, *dy;
    float *dx = NULL, *fwd_out;
    long L;
    size_t io_bytes;
    int rc;
    if (!dY || !input) return kmb_fail(KMB_EINVAL, "mamba_backward: NULL buffer");
    TRY(block_check(b));
    L = (long)b->config.seq_len;
    io_bytes = sizeof(float) * (size_t)L * b->config.dim;
    if (gsrc) optstate_grad_ptrs(gsrc, g);
    kmb_stage_begin(&st);
    rc = dev_block_stage(&st, b, &db, 0, gsrc ? g : NULL, 1, 0, gemm_ws(&st));
    if (rc == KMB_OK) {
        x = (const float *)kmb_stage_in(&st, input, io_bytes);
        dy = (const float *)kmb_stage_in(&st, dY, io_bytes);
        if (d_input) dx = (float *)kmb_stage_out(&st, d_input, io_bytes, 0);
        fwd_out = (float *)kmb_scratch(&st, io_bytes);
        rc = st.status;
        if (rc == KMB_OK && dx && (dx == x)) rc = kmb_fail(KMB_EINVAL, "mamba_backward: d_input aliases input");
        if (rc == KMB_OK) rc = acts_alloc(&st, &db.d, L, 1, &a);
        if (rc == KMB_OK) rc = bwd_scratch(&st, &db.d, L, &bs);
        if (rc == KMB_OK) rc = blk_forward(&db, x, fwd_out, 1, L, &a, NULL, st.s);
        if (rc == KMB_OK)
            rc = blk_backward(&db, x, &a, dy, dx, 1, L, bs.dz, bs.dyr, bs.dA, bs.dth, st.s);
    }
    return kmb_stage_finish(&st, rc);
}

void mamba_backward(MambaBlock *b, const float *dY, const float *input, float *d_input,
                    size_t batch_index) {
    (void)batch_index;
    if (!b) return;
    (void)block_backward_impl(b, dY, input, d_input, b->opt_state);
}

void mamba_backward_ws(MambaBlock *b, MambaBlockWorkspace *ws, const float *dY,
                       const float *input, float *d_input, size_t batch_index) {
    (void)ws;
    mamba_backward(b, dY, input, d_input, batch_index);
}

void mamba_backward_ws_local(MambaBlock *b, MambaBlockWorkspace *ws, const float *dY,
                             const float *input, float *d_input, size_t batch_index,
                             MBOptimState *local_grad) {
    (void)ws;
    (void)batch_index;
    if (!b) return;
    (void)block_backward_impl(b, dY, input, d_input, local_grad ? local_grad : b->opt_state);
}

/* ------------------------------------------------------------------ */
/* optimizer state (host arrays, reference layout)                      */
/* ------------------------------------------------------------------ */

static int grads_alloc(MBOptimState *s, const MambaBlock *b) {
    const BlockDims d = block_dims(b);
    float **g[P_COUNT] = {&s->g_W_in, &s->g_delta_proj, &s->g_lambda_proj, &s->g_W_B, &s->g_W_C,
                          &s->g_b_B,  &s->g_b_C,        &s->g_A_log,       &s->g_theta, &s->g_W_out};
    for (int i = 0; i < P_COUNT; ++i) {
        *g[i] = (float *)pinned_calloc(d.n[i], sizeof(float));
        if (!*g[i]) return -1;
    }
    return 0;
}

static void grads_free(MBOptimState *s) {
    float *g[P_COUNT];
    optstate_grad_ptrs(s, g);
    for (int i = 0; i < P_COUNT; ++i) pinned_free(g[i]);
}

static void moments_free(MBOptimState *s) {
    float *m[P_COUNT], *v[P_COUNT];
    optstate_moment_ptrs(s, m, v);
    for (int i = 0; i < P_COUNT; ++i) {
        pinned_free(m[i]);
        pinned_free(v[i]);
    }
}

void mamba_attach_optimizer(MambaBlock *b, OptimizerType type, const MBOptimConfig *optconf) {
    MBOptimState *s;
    (void)optconf;
    if (!b) return;
    mamba_free_optimizer(b);
    s = (MBOptimState *)calloc(1, sizeof *s);
    if (!s) return;
    s->type = type;
    if (grads_alloc(s, b)) goto fail;
    if (type != OPTIMIZER_SGD) {
        const BlockDims d = block_dims(b);
        float **m[P_COUNT] = {&s->m_W_in, &s->m_delta_proj, &s->m_lambda_proj, &s->m_W_B,
                              &s->m_W_C,  &s->m_b_B,        &s->m_b_C,         &s->m_A_log,
                              &s->m_theta, &s->m_W_out};
        float **v[P_COUNT] = {&s->v_W_in, &s->v_delta_proj, &s->v_lambda_proj, &s->v_W_B,
                              &s->v_W_C,  &s->v_b_B,        &s->v_b_C,         &s->v_A_log,
                              &s->v_theta, &s->v_W_out};
        for (int i = 0; i < P_COUNT; ++i) {
            *m[i] = (float *)pinned_calloc(d.n[i], sizeof(float));
            if (!*m[i]) goto fail;
            if (type == OPTIMIZER_ADAMW || type == OPTIMIZER_ADAM_CLIP) {
                *v[i] = (float *)pinned_calloc(d.n[i], sizeof(float));
                if (!*v[i]) goto fail;
            }
        }
    }
    b->opt_state = s;
    return;
fail:
    grads_free(s);
    moments_free(s);
    free(s);
}

void mamba_free_optimizer(MambaBlock *b) {
    if (!b || !b->opt_state) return;
    grads_free(b->opt_state);
    moments_free(b->opt_state);
    free(b->opt_state);
    b->opt_state = NULL;
}

void mamba_zero_grads(MambaBlock *b) {
    float *g[P_COUNT];
    BlockDims d;
    if (!b || !b->opt_state) return;
    d = block_dims(b);
    optstate_grad_ptrs(b->opt_state, g);
    for (int i = 0; i < P_COUNT; ++i) {
        memset(g[i], 0, d.n[i] * sizeof(float));
        (void)kmb_resident_update(g[i]);
    }
}

float mamba_block_grad_sqnorm(const MambaBlock *b) {
    KmbStage st;
    DevBlock db;
    float *g[P_COUNT];
    double *slots, host[P_COUNT];
    int rc;
    if (!b || !b->opt_state) return 0.0f;
    if (block_check(b) != KMB_OK) return 0.0f;
    optstate_grad_ptrs(b->opt_state, g);
    kmb_stage_begin(&st);
    rc = dev_block_stage(&st, b, &db, 0, g, 1, 0, NULL);
    slots = (double *)kmb_scratch(&st, sizeof(double) * P_COUNT);
    if (rc == KMB_OK) rc = st.status;
    if (rc == KMB_OK) rc = blk_sumsq(&db, slots, st.s);
    if (rc == KMB_OK) {
        cudaError_t e = cudaMemcpyAsync(host, slots, sizeof host, cudaMemcpyDeviceToHost, st.s);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "sqnorm copy");
    }
    /* gradients are read only: do not copy them back */
    for (int i = 0; i < st.n; ++i) st.b[i].out = 0;
    rc = kmb_stage_finish(&st, rc);
    return rc == KMB_OK ? (float)blk_sqnorm_host(host) : 0.0f;
}

void mamba_optimizer_step(MambaBlock *b, const MBOptimConfig *conf) {
    KmbStage st;
    DevBlock db;
    float *g[P_COUNT];
    double *slots;
    MBOptimState *s;
    int rc;
    if (!b || !b->opt_state || !conf) return;
    if (block_check(b) != KMB_OK) return;
    s = b->opt_state;
    s->step++;
    optstate_grad_ptrs(s, g);
    kmb_stage_begin(&st);
    rc = dev_block_stage(&st, b, &db, 1, g, 1, 1, NULL);
    slots = (double *)kmb_scratch(&st, sizeof(double) * P_COUNT);
    if (rc == KMB_OK) rc = st.status;
    if (rc == KMB_OK) rc = blk_opt_step(&st, &db, s->type, s->step, conf, slots, st.s);
    (void)kmb_stage_finish(&st, rc);
}

MBOptimState *mamba_local_grad_alloc(const MambaBlock *b) {
    MBOptimState *s;
    if (!b) return NULL;
    s = (MBOptimState *)calloc(1, sizeof *s);
    if (!s) return NULL;
    if (grads_alloc(s, b)) {
        grads_free(s);
        free(s);
        return NULL;
    }
    return s;
}

void mamba_local_grad_reduce(MambaBlock *b, const MBOptimState *local) {
    KmbStage st;
    BlockDims d;
    float *gd[P_COUNT], *gl[P_COUNT];
    int rc = KMB_OK;
    if (!b || !b->opt_state || !local) return;
    d = block_dims(b);
    optstate_grad_ptrs(b->opt_state, gd);
    optstate_grad_ptrs(local, gl);
    kmb_stage_begin(&st);
    for (int i = 0; i < P_COUNT && rc == KMB_OK; ++i) {
        float *y = (float *)kmb_stage_out(&st, gd[i], d.n[i] * sizeof(float), 1);
        const float *x = (const float *)kmb_stage_in(&st, gl[i], d.n[i] * sizeof(float));
        rc = st.status;
        if (rc == KMB_OK) rc = kmb_axpby(y, x, (long)d.n[i], 1.0f, 1.0f, st.s);
    }
    (void)kmb_stage_finish(&st, rc);
}

void mamba_local_grad_free(MBOptimState *local) {
    if (!local) return;
    grads_free(local);
    free(local);
}

/* ------------------------------------------------------------------ */
/* matrix helpers (declared by the reference header, defined here)     */
/* ------------------------------------------------------------------ */

MBMatrix *mb_matrix_create(size_t rows, size_t cols) {
    MBMatrix *m = (MBMatrix *)malloc(sizeof *m);
    if (!m) return NULL;
    if (mat_alloc(m, rows, cols)) {
        free(m);
        return NULL;
    }
    return m;
}

void mb_matrix_free(MBMatrix *m) {
    if (!m) return;
    pinned_free(m->data);
    free(m);
}

void mb_matrix_zero(MBMatrix *m) {
    if (!m || !m->data) return;
    memset(m->data, 0, m->rows * m->cols * sizeof(float));
}

void mb_matrix_copy(MBMatrix *dst, const MBMatrix *src) {
    if (!dst || !src || !dst->data || !src->data) return;
    if (dst->rows != src->rows || dst->cols != src->cols) return;
    memcpy(dst->data, src->data, src->rows * src->cols * sizeof(float));
}

void mb_matrix_print(const MBMatrix *m) {
    if (!m || !m->data) return;
    printf("MBMatrix %zu x %zu\n", m->rows, m->cols);
    for (size_t i = 0; i < m->rows; ++i) {
        for (size_t j = 0; j < m->cols; ++j) printf(" %9.5f", m->data[i * m->cols + j]);
        printf("\n");
    }
}

/* out[rows] = m v */
void mb_matrix_vec_mult(float *out, const MBMatrix *m, const float *v) {
    KmbStage st;
    const float *dm, *dv;
    float *dout;
    int rc;
    if (!out || !m || !m->data || !v || !m->rows) return;
    kmb_stage_begin(&st);
    dm = (const float *)kmb_stage_in(&st, m->data, sizeof(float) * m->rows * m->cols);
    dv = (const float *)kmb_stage_in(&st, v, sizeof(float) * (m->cols ? m->cols : 1));
    dout = (float *)kmb_stage_out(&st, out, sizeof(float) * m->rows, 0);
    rc = st.status;
    if (rc == KMB_OK)
        rc = kmb_gemm((int)m->rows, 1, (int)m->cols, dm, (long)m->cols, 1, dv, 1, 1, dout, 1, 0,
                      NULL, 0, st.s);
    (void)kmb_stage_finish(&st, rc);
}

static void vec_axpby(float *y, const float *x, size_t n, float a, float b) {
    KmbStage st;
    float *dy;
    const float *dx = NULL;
    int rc;
    if (!y || !n) return;
    kmb_stage_begin(&st);
    dy = (float *)kmb_stage_out(&st, y, sizeof(float) * n, 1);
    if (x) dx = (const float *)kmb_stage_in(&st, x, sizeof(float) * n);
    rc = st.status;
    if (rc == KMB_OK) rc = kmb_axpby(dy, dx, (long)n, a, b, st.s);
    (void)kmb_stage_finish(&st, rc);
}

void mb_vec_add(float *y, const float *x, size_t n) {
    if (!x) return;
    vec_axpby(y, x, n, 1.0f, 1.0f);
}

void mb_vec_scale(float *v, float alpha, size_t n) { vec_axpby(v, NULL, n, alpha, 0.0f); }

/* delta_out[t] = clamp(softplus(delta_proj . delta_in[t, :]), dt_min,
 * dt_max) for t < seq_len (dt_scale without a delta projection), the
 * controller rule of src/mamba_block.c:122-134. */
void mb_compute_delta(float *delta_out, const MambaBlock *b, const float *delta_in,
                      size_t seq_len) {
    KmbStage st;
    const float *dx, *dw;
    float *dout, *z;
    const size_t D = b ? b->config.dim : 0;
    int rc;
    if (!delta_out || !b || !delta_in || !seq_len) return;
    if (b->delta_proj.rows == 0 || !b->delta_proj.data) {
        for (size_t t = 0; t < seq_len; ++t) delta_out[t] = b->config.dt_scale;
        return;
    }
    kmb_stage_begin(&st);
    dx = (const float *)kmb_stage_in(&st, delta_in, sizeof(float) * seq_len * D);
    dw = (const float *)kmb_stage_in(&st, b->delta_proj.data, sizeof(float) * D);
    dout = (float *)kmb_stage_out(&st, delta_out, sizeof(float) * seq_len, 0);
    z = (float *)kmb_scratch(&st, sizeof(float) * seq_len);
    rc = st.status;
    if (rc == KMB_OK)
        rc = kmb_gemm((int)seq_len, 1, (int)D, dx, (long)D, 1, dw, 1, 1, z, 1, 0, NULL, 0, st.s);
    if (rc == KMB_OK)
        rc = kmb_dt_act(z, dout, (long)seq_len, b->config.dt_min, b->config.dt_max, st.s);
    (void)kmb_stage_finish(&st, rc);
}

/* ------------------------------------------------------------------ */
/* model                                                               */
/* ------------------------------------------------------------------ */

/* ------------------------------------------------------------------ */
/* device-resident models                                              */
/* ------------------------------------------------------------------ */

typedef struct {
    float *p;
    size_t bytes;
} HostArr;

/* Every host array of m the calls stage (weights, gradients, moments),
 * each once; returns the count (<= cap) or -1 when cap is too small. */
static int model_host_arrays(const KMamba *m, HostArr *out, int cap) {
    int n = 0;
    const size_t VD = sizeof(float) * m->cfg.vocab_size * m->cfg.dim;
#define KMB_ADD(ptr, nbytes) do { float *q_ = (ptr); int dup_ = 0; \
        if (q_) { for (int k_ = 0; k_ < n; ++k_) dup_ |= out[k_].p == q_; \
                  if (!dup_) { if (n >= cap) return -1; out[n].p = q_; out[n].bytes = (nbytes); ++n; } } \
    } while (0)
    KMB_ADD(m->embedding, VD);
    KMB_ADD(m->head, VD);
    KMB_ADD(m->m_embedding, VD);
    KMB_ADD(m->v_embedding, VD);
    KMB_ADD(m->m_head, VD);
    KMB_ADD(m->v_head, VD);
    for (size_t l = 0; l < m->cfg.n_layers; ++l) {
        const MambaBlock *b = m->layers[l];
        if (!b) continue;
        const BlockDims d = block_dims(b);
        float *hp[P_COUNT];
        block_param_ptrs(b, hp);
        for (int i = 0; i < P_COUNT; ++i) KMB_ADD(hp[i], d.n[i] * sizeof(float));
        if (b->opt_state) {
            float *g[P_COUNT], *hm[P_COUNT], *hv[P_COUNT];
            optstate_grad_ptrs(b->opt_state, g);
            optstate_moment_ptrs(b->opt_state, hm, hv);
            for (int i = 0; i < P_COUNT; ++i) {
                KMB_ADD(g[i], d.n[i] * sizeof(float));
                KMB_ADD(hm[i], d.n[i] * sizeof(float));
                KMB_ADD(hv[i], d.n[i] * sizeof(float));
            }
        }
    }
#undef KMB_ADD
    return n;
}

/* Applies op (0 add, 1 sync, 2 remove with copy back, 3 remove, 4 update)
 * to every host array of m. */
static int model_resident_op(KMamba *m, int op) {
    if (!m || !m->layers) return kmb_fail(KMB_EINVAL, "resident: NULL model");
    const int cap = 6 + (int)m->cfg.n_layers * 4 * P_COUNT;
    HostArr *a = (HostArr *)malloc(sizeof *a * (size_t)cap);
    if (!a) return kmb_fail(KMB_ENOMEM, "resident: host allocation failed");
    const int n = model_host_arrays(m, a, cap);
    int rc = n < 0 ? kmb_fail(KMB_EINVAL, "resident: array table overflow") : KMB_OK;
    for (int i = 0; i < n && rc == KMB_OK; ++i) {
        if (op == 0) rc = kmb_resident_add(a[i].p, a[i].bytes);
        else if (op == 1) rc = kmb_resident_sync(a[i].p);
        else if (op == 4) rc = kmb_resident_update(a[i].p);
        else rc = kmb_resident_remove(a[i].p, op == 2);
    }
    free(a);
    return rc;
}

int kmamba_set_device_resident(KMamba *m, int on) {
    kmb_clear_error();
    return model_resident_op(m, on ? 0 : 2);
}

int kmamba_sync_to_host(KMamba *m) {
    kmb_clear_error();
    if (!kmb_resident_count()) return m ? KMB_OK : kmb_fail(KMB_EINVAL, "resident: NULL model");
    return model_resident_op(m, 1);
}

KMamba *kmamba_create(const KMambaConfig *cfg) {
    KMamba *m;
    if (!cfg || !cfg->vocab_size || !cfg->dim || !cfg->seq_len || !cfg->n_layers) return NULL;
    m = (KMamba *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->cfg = *cfg;
    if (km_normalize_spatial_topology(&m->cfg.spatial_ndims, m->cfg.spatial_dims,
                                      (long)m->cfg.seq_len, m->cfg.use_convnd,
                                      &m->cfg.convnd_ndims, m->cfg.convnd_K) != 0) {
        free(m);
        return NULL;
    }
    m->embedding = (float *)pinned_calloc(m->cfg.vocab_size * m->cfg.dim, sizeof(float));
    m->head = m->cfg.weight_tying
                  ? m->embedding
                  : (float *)pinned_calloc(m->cfg.dim * m->cfg.vocab_size, sizeof(float));
    m->layers = (MambaBlock **)calloc(m->cfg.n_layers, sizeof(MambaBlock *));
    if (!m->embedding || !m->head || !m->layers) {
        kmamba_free(m);
        return NULL;
    }
    for (size_t i = 0; i < m->cfg.n_layers; ++i) {
        MBConfig bc;
        memset(&bc, 0, sizeof bc);
        bc.dim = m->cfg.dim;
        bc.state_size = m->cfg.state_size;
        bc.seq_len = m->cfg.seq_len;
        bc.mimo_rank = m->cfg.mimo_rank > 0 ? m->cfg.mimo_rank : 1;
        bc.dt_scale = m->cfg.dt_scale;
        bc.dt_min = m->cfg.dt_min;
        bc.dt_max = m->cfg.dt_max;
        bc.spatial_ndims = m->cfg.spatial_ndims;
        memcpy(bc.spatial_dims, m->cfg.spatial_dims, sizeof bc.spatial_dims);
        bc.use_convnd = m->cfg.use_convnd;
        bc.convnd_K = m->cfg.convnd_K;
        bc.convnd_ndims = m->cfg.convnd_ndims;
        m->layers[i] = mamba_block_create(&bc);
        if (!m->layers[i]) {
            kmamba_free(m);
            return NULL;
        }
    }
    return m;
}

void kmamba_free(KMamba *m) {
    if (!m) return;
    /* release device-resident copies first: a later host allocation at the
     * same address must not find them */
    if (m->layers && kmb_resident_count()) (void)model_resident_op(m, 3);
    if (m->layers) {
        for (size_t i = 0; i < m->cfg.n_layers; ++i) mamba_block_free(m->layers[i]);
        free(m->layers);
    }
    if (m->head != m->embedding) pinned_free(m->head);
    pinned_free(m->embedding);
    pinned_free(m->m_embedding);
    pinned_free(m->v_embedding);
    pinned_free(m->m_head);
    pinned_free(m->v_head);
    free(m);
}

static void xavier(float *w, size_t fan_in, size_t fan_out, size_t n) {
    const float scale = sqrtf(6.0f / ((float)fan_in + (float)fan_out));
    for (size_t i = 0; i < n; ++i) w[i] = ((float)rand() / (float)RAND_MAX * 2.0f - 1.0f) * scale;
}

/* srand(seed) then the reference's rand() order (src/kmamba.c:177-188). */
int kmamba_init(KMamba *m, uint32_t seed) {
    if (!m) return -1;
    srand((unsigned)seed);
    xavier(m->embedding, m->cfg.vocab_size, m->cfg.dim, m->cfg.vocab_size * m->cfg.dim);
    if (!m->cfg.weight_tying)
        xavier(m->head, m->cfg.dim, m->cfg.vocab_size, m->cfg.dim * m->cfg.vocab_size);
    for (size_t i = 0; i < m->cfg.n_layers; ++i) mamba_block_init(m->layers[i]);
    /* a device-resident model takes the new values */
    if (kmb_resident_count() && model_resident_op(m, 4) != KMB_OK) return -1;
    return 0;
}

int kmamba_enable_training(KMamba *m, const MBOptimConfig *opt_blocks, float lr_embed_head,
                           float weight_decay) {
    return kmamba_enable_training_with_optimizer(m, OPTIMIZER_ADAM_CLIP, opt_blocks, lr_embed_head,
                                                 weight_decay);
}

int kmamba_enable_training_with_optimizer(KMamba *m, OptimizerType type,
                                          const MBOptimConfig *opt_blocks, float lr_embed_head,
                                          float weight_decay) {
    size_t VD;
    if (!m || !opt_blocks) return -1;
    m->for_training = 1;
    m->opt_blocks = *opt_blocks;
    m->lr_embed_head = lr_embed_head;
    m->weight_decay = weight_decay;
    for (size_t i = 0; i < m->cfg.n_layers; ++i) {
        mamba_attach_optimizer(m->layers[i], type, opt_blocks);
        if (!m->layers[i]->opt_state) return -1;
    }
    VD = m->cfg.vocab_size * m->cfg.dim;
    pinned_free(m->m_embedding);
    pinned_free(m->v_embedding);
    pinned_free(m->m_head);
    pinned_free(m->v_head);
    m->m_embedding = (float *)pinned_calloc(VD, sizeof(float));
    m->v_embedding = (float *)pinned_calloc(VD, sizeof(float));
    m->m_head = (float *)pinned_calloc(VD, sizeof(float));
    m->v_head = (float *)pinned_calloc(VD, sizeof(float));
    m->step_embed_head = 0;
    if (!m->m_embedding || !m->v_embedding || !m->m_head || !m->v_head) return -1;
    return 0;
}

/* Checkpoint header of the reference's KMAMBA v4 format
 * (src/kmamba.c:218-231); the field order and padding must match for
 * files to be exchanged with the reference. */
typedef struct {
    char magic[8];
    uint32_t version;
    uint32_t reserved;
    uint64_t vocab_size;
    uint64_t dim;
    uint64_t state_size;
    uint64_t seq_len;
    uint64_t n_layers;
    uint64_t mimo_rank;
    float dt_scale;
    float dt_min;
    float dt_max;
} KmbCkptHeader;

static int io_floats(FILE *f, float *p, size_t n, int wr) {
    return (wr ? fwrite(p, sizeof(float), n, f) : fread(p, sizeof(float), n, f)) == n ? 0 : -1;
}

static int model_tensors_io(FILE *f, KMamba *m, int wr) {
    if (io_floats(f, m->embedding, m->cfg.vocab_size * m->cfg.dim, wr) ||
        io_floats(f, m->head, m->cfg.dim * m->cfg.vocab_size, wr))
        return -1;
    for (size_t i = 0; i < m->cfg.n_layers; ++i) {
        MambaBlock *b = m->layers[i];
        if (io_floats(f, b->W_in.data, b->W_in.rows * b->W_in.cols, wr) ||
            io_floats(f, b->W_out.data, b->W_out.rows * b->W_out.cols, wr) ||
            io_floats(f, b->A_log.data, b->A_log.rows * b->A_log.cols, wr) ||
            io_floats(f, b->W_B.data, b->W_B.rows * b->W_B.cols, wr) ||
            io_floats(f, b->W_C.data, b->W_C.rows * b->W_C.cols, wr) ||
            io_floats(f, b->b_B, b->W_B.rows, wr) || io_floats(f, b->b_C, b->W_C.rows, wr) ||
            io_floats(f, b->delta_proj.data, b->delta_proj.rows * b->delta_proj.cols, wr) ||
            io_floats(f, b->lambda_proj.data, b->lambda_proj.rows * b->lambda_proj.cols, wr) ||
            io_floats(f, b->theta, blk_TS(&b->config), wr))
            return -1;
    }
    return 0;
}

int kmamba_save(const KMamba *m, const char *path) {
    KmbCkptHeader h;
    FILE *f;
    int rc;
    if (!m || !path) return -1;
    /* a device-resident model's current values are on the device */
    if (kmb_resident_count() && model_resident_op((KMamba *)m, 1) != KMB_OK) return -1;
    f = fopen(path, "wb");
    if (!f) return -1;
    memset(&h, 0, sizeof h);
    memcpy(h.magic, "KMAMBA", 6);
    h.version = 4;
    h.vocab_size = m->cfg.vocab_size;
    h.dim = m->cfg.dim;
    h.state_size = m->cfg.state_size;
    h.seq_len = m->cfg.seq_len;
    h.n_layers = m->cfg.n_layers;
    h.mimo_rank = m->cfg.mimo_rank > 0 ? m->cfg.mimo_rank : 1;
    h.dt_scale = m->cfg.dt_scale;
    h.dt_min = m->cfg.dt_min;
    h.dt_max = m->cfg.dt_max;
    rc = fwrite(&h, sizeof h, 1, f) == 1 ? model_tensors_io(f, (KMamba *)m, 1) : -1;
    if (fclose(f) != 0) rc = -1;
    return rc;
}

KMamba *kmamba_load(const char *path, int for_training, const MBOptimConfig *opt_blocks,
                    float lr_embed_head, float weight_decay) {
    KmbCkptHeader h;
    KMambaConfig cfg;
    KMamba *m;
    FILE *f;
    if (!path) return NULL;
    f = fopen(path, "rb");
    if (!f) return NULL;
    if (fread(&h, sizeof h, 1, f) != 1 || memcmp(h.magic, "KMAMBA", 6) != 0 || h.version > 4) {
        fclose(f);
        return NULL;
    }
    memset(&cfg, 0, sizeof cfg);
    cfg.vocab_size = (size_t)h.vocab_size;
    cfg.dim = (size_t)h.dim;
    cfg.state_size = (size_t)h.state_size;
    cfg.seq_len = (size_t)h.seq_len;
    cfg.n_layers = (size_t)h.n_layers;
    cfg.mimo_rank = (h.version >= 4 && h.mimo_rank > 0) ? (size_t)h.mimo_rank : 1;
    cfg.dt_scale = h.dt_scale;
    cfg.dt_min = h.dt_min;
    cfg.dt_max = h.dt_max;
    m = kmamba_create(&cfg);
    if (!m) {
        fclose(f);
        return NULL;
    }
    if (for_training &&
        (!opt_blocks || kmamba_enable_training(m, opt_blocks, lr_embed_head, weight_decay))) {
        kmamba_free(m);
        fclose(f);
        return NULL;
    }
    if (model_tensors_io(f, m, 0)) {
        kmamba_free(m);
        fclose(f);
        return NULL;
    }
    fclose(f);
    return m;
}

/* ------------------------------------------------------------------ */
/* model forward / training on the device                               */
/* ------------------------------------------------------------------ */

static int model_check(const KMamba *m) {
    if (!m || !m->layers || !m->embedding || !m->head)
        return kmb_fail(KMB_EINVAL, "kmamba: model not created");
    for (size_t i = 0; i < m->cfg.n_layers; ++i) TRY(block_check(m->layers[i]));
    return KMB_OK;
}

/* Everything one model call keeps on the device. */
typedef struct {
    DevBlock *blk;      /* [n_layers] */
    BlockActs *acts;    /* [n_layers] */
    float *emb, *head;  /* parameters */
    float *hs;          /* [(n_layers + 1), rows, D] activations */
    const unsigned *tok; /* [batch, L + 1] or [L] */
    unsigned *tok_in, *tok_tgt; /* compacted [rows] */
} ModelDev;

static void model_free_dev(ModelDev *md) {
    free(md->blk);
    free(md->acts);
}

/* Splits [batch, L+1] token rows into input and target columns on the
 * device (a strided copy). */
static int split_tokens(const unsigned *tok, unsigned *in, unsigned *tgt, long batch, long L,
                        cudaStream_t s) {
    cudaError_t e = cudaMemcpy2DAsync(in, sizeof(unsigned) * (size_t)L, tok,
                                      sizeof(unsigned) * (size_t)(L + 1),
                                      sizeof(unsigned) * (size_t)L, (size_t)batch,
                                      cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(tgt, sizeof(unsigned) * (size_t)L, tok + 1,
                              sizeof(unsigned) * (size_t)(L + 1), sizeof(unsigned) * (size_t)L,
                              (size_t)batch, cudaMemcpyDeviceToDevice, s);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "token split");
}

/* Embedding, every block and the logits of `batch` sequences.  hidden
 * states stay in md->hs; activations of every block are kept when
 * `train`. */
static int model_forward_dev(KmbStage *st, KMamba *m, ModelDev *md, long batch, int train,
                             float *logits) {
    const long L = (long)m->cfg.seq_len, D = (long)m->cfg.dim, V = (long)m->cfg.vocab_size;
    const long rows = batch * L;
    const size_t nl = m->cfg.n_layers;
    TRY(kmb_embed(md->emb, md->tok_in, rows, D, V, md->hs, NULL, NULL, st->s));
    for (size_t i = 0; i < nl; ++i) {
        TRY(acts_alloc(st, &md->blk[i].d, rows, train, &md->acts[i]));
        TRY(blk_forward(&md->blk[i], md->hs + (long)i * rows * D, md->hs + (long)(i + 1) * rows * D,
                        batch, L, &md->acts[i], NULL, st->s));
    }
    /* logits = hidden [rows, D] @ head [D, V] */
    return kmb_gemm((int)rows, (int)V, (int)D, md->hs + (long)nl * rows * D, D, 1, md->head, V, 1,
                    logits, V, 0, md->blk[0].ws, KMB_GEMM_WS, st->s);
}

int kmamba_forward(KMamba *m, const uint32_t *tokens, float *logits_out) {
    KmbStage st;
    ModelDev md;
    float *logits, *ws;
    long L, D, V;
    int rc;
    if (!m || !tokens || !logits_out) return -1;
    if (model_check(m) != KMB_OK) return -1;
    L = (long)m->cfg.seq_len;
    D = (long)m->cfg.dim;
    V = (long)m->cfg.vocab_size;
    for (size_t i = 0; i < m->cfg.n_layers; ++i) {
        memset(m->layers[i]->hidden, 0, m->cfg.state_size * sizeof(float));
        memset(m->layers[i]->scan_h, 0, m->cfg.state_size * sizeof(float));
    }
    memset(&md, 0, sizeof md);
    md.blk = (DevBlock *)calloc(m->cfg.n_layers, sizeof(DevBlock));
    md.acts = (BlockActs *)calloc(m->cfg.n_layers, sizeof(BlockActs));
    if (!md.blk || !md.acts) {
        model_free_dev(&md);
        return -1;
    }
    kmb_stage_begin(&st);
    rc = kmb_stage_reserve(&st, 16 + 24 * (int)m->cfg.n_layers);
    ws = gemm_ws(&st);
    for (size_t i = 0; i < m->cfg.n_layers && rc == KMB_OK; ++i)
        rc = dev_block_stage(&st, m->layers[i], &md.blk[i], 0, NULL, 0, 0, ws);
    if (rc == KMB_OK) {
        md.emb = (float *)kmb_stage_in(&st, m->embedding, sizeof(float) * (size_t)(V * D));
        md.head = (float *)kmb_stage_in(&st, m->head, sizeof(float) * (size_t)(D * V));
        md.tok_in = (unsigned *)kmb_stage_in(&st, tokens, sizeof(uint32_t) * (size_t)L);
        md.hs = (float *)kmb_scratch(&st, sizeof(float) * (size_t)((m->cfg.n_layers + 1) * L * D));
        logits = (float *)kmb_stage_out(&st, logits_out, sizeof(float) * (size_t)(L * V), 0);
        rc = st.status;
        if (rc == KMB_OK) rc = model_forward_dev(&st, m, &md, 1, 0, logits);
    }
    rc = kmb_stage_finish(&st, rc);
    model_free_dev(&md);
    return rc == KMB_OK ? 0 : -1;
}

/* Forward + backward + optimizer step over `batch` sequences of
 * [L + 1] tokens (src/kmamba.c:377-466 for one sequence, :468-630 for a
 * batch): dlogits are scaled by 1/(batch*L), gradients are summed over the
 * batch, the grad norm is recorded (not clipped), then every block and the
 * embedding / head take one step. */
static float model_train(KMamba *m, const uint32_t *tokens, size_t batch) {
    KmbStage st;
    ModelDev md;
    const long L = (long)m->cfg.seq_len, D = (long)m->cfg.dim, V = (long)m->cfg.vocab_size;
    const long rows = (long)batch * L;
    const size_t nl = m->cfg.n_layers;
    float *logits = NULL, *dlogits = NULL, *row_loss = NULL, *g_head = NULL, *g_emb = NULL;
    float *dcur = NULL, *dnext = NULL, *ws;
    double *slots = NULL;
    float *loss_host = NULL;
    double *slots_host = NULL;
    BwdScratch bs;
    float loss = NAN;
    int rc;

    if (model_check(m) != KMB_OK) return NAN;
    if (!kmb_is_device_ptr(tokens)) {
        for (size_t b = 0; b < batch; ++b)
            for (long t = 1; t <= L; ++t)
                if (tokens[b * (size_t)(L + 1) + t] >= (uint32_t)V) {
                    kmb_fail(KMB_EINVAL, "kmamba train: target token %u >= vocab_size %ld",
                             tokens[b * (size_t)(L + 1) + t], V);
                    return NAN;
                }
    }
    for (size_t i = 0; i < nl; ++i)
        if (!m->layers[i]->opt_state) {
            kmb_fail(KMB_EINVAL, "kmamba train: layer %zu has no optimizer state", i);
            return NAN;
        }
    if (!m->m_embedding || !m->v_embedding || !m->m_head || !m->v_head) {
        kmb_fail(KMB_EINVAL, "kmamba train: training not enabled");
        return NAN;
    }
    memset(&md, 0, sizeof md);
    md.blk = (DevBlock *)calloc(nl, sizeof(DevBlock));
    md.acts = (BlockActs *)calloc(nl, sizeof(BlockActs));
    loss_host = (float *)malloc(sizeof(float) * (size_t)rows);
    slots_host = (double *)malloc(sizeof(double) * (P_COUNT * nl + 2));
    if (!md.blk || !md.acts || !loss_host || !slots_host) {
        model_free_dev(&md);
        free(loss_host);
        free(slots_host);
        kmb_fail(KMB_ENOMEM, "kmamba train: host allocation failed");
        return NAN;
    }

    kmb_stage_begin(&st);
    rc = kmb_stage_reserve(&st, 64 + 64 * (int)nl);
    ws = gemm_ws(&st);
    for (size_t i = 0; i < nl && rc == KMB_OK; ++i) {
        float *g[P_COUNT];
        optstate_grad_ptrs(m->layers[i]->opt_state, g);
        rc = dev_block_stage(&st, m->layers[i], &md.blk[i], 1, g, 0, 1, ws);
    }
    if (rc == KMB_OK) {
        const size_t VD = (size_t)(V * D);
        unsigned *tok;
        md.emb = (float *)kmb_stage_out(&st, m->embedding, sizeof(float) * VD, 1);
        md.head = (float *)kmb_stage_out(&st, m->head, sizeof(float) * VD, 1);
        tok = (unsigned *)kmb_stage_in(&st, tokens, sizeof(uint32_t) * batch * (size_t)(L + 1));
        md.tok_in = (unsigned *)kmb_scratch(&st, sizeof(unsigned) * (size_t)rows);
        md.tok_tgt = (unsigned *)kmb_scratch(&st, sizeof(unsigned) * (size_t)rows);
        md.hs = (float *)kmb_scratch(&st, sizeof(float) * (nl + 1) * (size_t)rows * D);
        logits = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows * V);
        dlogits = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows * V);
        row_loss = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows);
        g_head = (float *)kmb_scratch(&st, sizeof(float) * VD);
        g_emb = (float *)kmb_scratch(&st, sizeof(float) * VD);
        dcur = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows * D);
        dnext = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows * D);
        slots = (double *)kmb_scratch(&st, sizeof(double) * (P_COUNT * nl + 2));
        rc = st.status;
        if (rc == KMB_OK) rc = split_tokens(tok, md.tok_in, md.tok_tgt, (long)batch, L, st.s);
        if (rc == KMB_OK) {
            int W = 0;
            for (size_t i = 0; i < nl; ++i)
                if (md.blk[i].d.W > W) W = md.blk[i].d.W;
            bs.dz = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows * W);
            bs.dyr = (float *)kmb_scratch(&st, sizeof(float) * (size_t)rows * 8);
            bs.dA = NULL; /* blocks always carry gradients here */
            bs.dth = NULL;
            rc = st.status;
        }
    }
    if (rc == KMB_OK) rc = model_forward_dev(&st, m, &md, (long)batch, 1, logits);
    if (rc == KMB_OK)
        rc = kmb_softmax_ce(logits, md.tok_tgt, rows, V, dlogits, row_loss, st.s);
    if (rc == KMB_OK) {
        const float *hidden = md.hs + (long)nl * rows * D;
        /* the CE kernel scales by 1/rows = 1/(batch*L) (invBL of the batch
         * path; 1/L for one sequence) */
        /* d_hidden = dlogits [rows, V] @ head^T */
        rc = kmb_gemm((int)rows, (int)D, (int)V, dlogits, V, 1, md.head, 1, V, dcur, D, 0,
                      md.blk[0].ws, KMB_GEMM_WS, st.s);
        /* g_head = hidden^T @ dlogits */
        if (rc == KMB_OK)
            rc = kmb_gemm((int)D, (int)V, (int)rows, hidden, 1, D, dlogits, V, 1, g_head, V, 0,
                          md.blk[0].ws, KMB_GEMM_WS, st.s);
    }
    for (size_t li = nl; li-- > 0 && rc == KMB_OK;) {
        float *t;
        rc = blk_backward(&md.blk[li], md.hs + (long)li * rows * D, &md.acts[li], dcur, dnext,
                          (long)batch, L, bs.dz, bs.dyr, bs.dA, bs.dth, st.s);
        t = dcur;
        dcur = dnext;
        dnext = t;
    }
    if (rc == KMB_OK) {
        cudaError_t e = cudaMemsetAsync(g_emb, 0, sizeof(float) * (size_t)(V * D), st.s);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "embedding gradient zeroing");
        if (rc == KMB_OK) rc = kmb_embed(NULL, md.tok_in, rows, D, V, NULL, dcur, g_emb, st.s);
    }
    /* squared norms: [P_COUNT] per layer, then head, embedding */
    for (size_t i = 0; i < nl && rc == KMB_OK; ++i)
        rc = blk_sumsq(&md.blk[i], slots + i * P_COUNT, st.s);
    if (rc == KMB_OK) {
        cudaError_t e = cudaMemsetAsync(slots + nl * P_COUNT, 0, 2 * sizeof(double), st.s);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "norm zeroing");
        if (rc == KMB_OK) {
            const float *x[2] = {g_head, g_emb};
            const long n[2] = {V * D, V * D};
            double *out[2] = {slots + nl * P_COUNT, slots + nl * P_COUNT + 1};
            rc = kmb_sumsq_multi(2, x, n, out, st.s);
        }
    }
    if (rc == KMB_OK) {
        cudaError_t e = cudaMemcpyAsync(slots_host, slots, sizeof(double) * (P_COUNT * nl + 2),
                                        cudaMemcpyDeviceToHost, st.s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(loss_host, row_loss, sizeof(float) * (size_t)rows,
                                cudaMemcpyDeviceToHost, st.s);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "loss copy");
    }
    /* optimizer steps: blocks with their own counters, then embedding and
     * head with the block config (src/kmamba.c:455-460) */
    for (size_t i = 0; i < nl && rc == KMB_OK; ++i) {
        MBOptimState *s = m->layers[i]->opt_state;
        s->step++;
        rc = blk_opt_step(&st, &md.blk[i], s->type, s->step, &m->opt_blocks, slots + i * P_COUNT,
                          st.s);
    }
    if (rc == KMB_OK) {
        const MBOptimConfig *c = &m->opt_blocks;
        float bc1, bc2;
        float *mem, *vem, *mh, *vh;
        m->step_embed_head++;
        bc1 = 1.0f - powf(0.9f, (float)m->step_embed_head);
        bc2 = 1.0f - powf(0.999f, (float)m->step_embed_head);
        mem = (float *)kmb_stage_out(&st, m->m_embedding, sizeof(float) * (size_t)(V * D), 1);
        vem = (float *)kmb_stage_out(&st, m->v_embedding, sizeof(float) * (size_t)(V * D), 1);
        mh = (float *)kmb_stage_out(&st, m->m_head, sizeof(float) * (size_t)(V * D), 1);
        vh = (float *)kmb_stage_out(&st, m->v_head, sizeof(float) * (size_t)(V * D), 1);
        rc = st.status;
        /* embedding then head (one buffer twice when tied, as in the
         * reference): separate launches keep that order */
        if (rc == KMB_OK)
            rc = kmb_adamw(md.emb, g_emb, mem, vem, V * D, c->lr, 0.9f, 0.999f, c->eps,
                           c->weight_decay, bc1, bc2, st.s);
        if (rc == KMB_OK)
            rc = kmb_adamw(md.head, g_head, mh, vh, V * D, c->lr, 0.9f, 0.999f, c->eps,
                           c->weight_decay, bc1, bc2, st.s);
    }
    rc = kmb_stage_finish(&st, rc);
    if (rc == KMB_OK) {
        /* loss and norms in the reference's order and precision */
        const float invL = 1.0f / (float)L, invB = 1.0f / (float)batch;
        float total = 0.0f;
        double gsq;
        for (size_t b = 0; b < batch; ++b) {
            float sl = 0.0f;
            for (long t = 0; t < L; ++t) sl += loss_host[b * (size_t)L + t];
            total += batch == 1 ? sl : sl * invL;
        }
        loss = batch == 1 ? total * invL : total * invB;
        {
            const float gn_h = sqrtf((float)slots_host[nl * P_COUNT]);
            const float gn_e = sqrtf((float)slots_host[nl * P_COUNT + 1]);
            gsq = (double)gn_h * gn_h + (double)gn_e * gn_e;
        }
        for (size_t i = 0; i < nl; ++i) gsq += (double)(float)blk_sqnorm_host(slots_host + i * P_COUNT);
        m->last_grad_norm = sqrtf((float)gsq);
        m->last_grad_over_clip =
            m->opt_blocks.clip_norm > 0.0f ? m->last_grad_norm / m->opt_blocks.clip_norm : 0.0f;
        m->last_grad_would_clip =
            m->opt_blocks.clip_norm > 0.0f && m->last_grad_norm > m->opt_blocks.clip_norm;
    }
    model_free_dev(&md);
    free(loss_host);
    free(slots_host);
    return loss;
}

float kmamba_train_step(KMamba *m, const uint32_t *tokens_plus1) {
    if (!m || !tokens_plus1 || !m->for_training) return NAN;
    return model_train(m, tokens_plus1, 1);
}

float kmamba_train_batch(KMamba *m, const uint32_t *batch_tokens, size_t batch_size) {
    if (!m || !batch_tokens || !m->for_training || batch_size == 0) return NAN;
    return model_train(m, batch_tokens, batch_size);
}

/* The reference splits this step between host (embedding, head) and GPU
 * (blocks); here every part already runs on the device, so it is the same
 * step as kmamba_train_batch. */
float kmamba_train_batch_hybrid(KMamba *m, const uint32_t *batch_tokens, size_t batch_size) {
    return kmamba_train_batch(m, batch_tokens, batch_size);
}

float kmamba_last_grad_norm(const KMamba *m) { return m ? m->last_grad_norm : 0.0f; }
float kmamba_last_grad_over_clip(const KMamba *m) { return m ? m->last_grad_over_clip : 0.0f; }
int kmamba_last_grad_would_clip(const KMamba *m) { return m ? m->last_grad_would_clip : 0; }
size_t kmamba_step_count(const KMamba *m) { return m ? m->step_embed_head : 0; }

void kmamba_update_lr(KMamba *m, float lr_blocks, float lr_embed) {
    if (!m) return;
    m->opt_blocks.lr = lr_blocks;
    m->lr_embed_head = lr_embed;
}
