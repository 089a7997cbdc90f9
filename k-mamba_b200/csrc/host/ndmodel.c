/*
 * Mamba-ND model of kmamba_ndmodel.h: host orchestration of the block's
 * kernels (tensor-core projections, ConvND, ND scan, ndblock.cu pieces),
 * the LM head, AdamW and the data-parallel gradient exchange.
 *
 * Memory plan for one training step of T = batch * points tokens:
 *   - the residual stream x_l (fp32 [T, d]) of every layer l = 0..L is kept
 *     for the backward: (L + 1) T d floats;
 *   - one layer's activations live at a time: the backward recomputes
 *     layer l's forward from x_l, then runs its adjoint;
 *   - the ND scan keeps its state history [T, d, 16] for the layer being
 *     differentiated only.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "kmamba_ndmodel.h"
#include "../kmb_internal.h"

#define NDM_K 3
#define NDM_STATE 16
#define NDM_QC 35  /* q columns: 3 dt inputs, 16 B, 16 C */
#define NDM_QLD 40 /* row stride of the bf16 dq operand (a multiple of 8) */

typedef struct {
    float *W_a, *W_z, *W_out, *W_p, *dt_bias, *A_log, *conv_kernel, *conv_bias;
} LayerPtrs;

typedef struct {
    long batch;
    float *x_store;           /* [(L + 1), T, d] residual stream */
    uint16_t *x16, *g16, *d16a, *d16b, *c16; /* bf16 [T, d] GEMM operands */
    float *a, *z, *v, *c, *y, *tmp1, *tmp2, *tmp3; /* fp32 [T, d] */
    float *q;                 /* [T, 35] */
    uint16_t *dq16;           /* bf16 [T, NDM_QLD] */
    float *delta, *ddelta;    /* [batch, 3, P, d] */
    float *Bs, *Cs, *dBs, *dCs; /* [T, 16] */
    float *h;                 /* [T, d, 16] scan history */
    float *A, *dA_tmp;        /* [3, d, 16] */
    float *ck_tmp, *cb_tmp;   /* conv kernel / bias gradients of one pass */
    float *logits, *dlogits;  /* [T, vocab] */
    uint16_t *l16;            /* bf16 dlogits [T, vocab] */
    float *row_loss;          /* [T] */
    unsigned *tok, *tgt;      /* [T] */
    float *loss_dev;          /* [1] */
} Work;

struct KmbNDModel {
    KmbNDModelConfig cfg;
    long P, d, L, V, per_layer, n;
    float *params, *grads, *m, *v; /* device, flat */
    uint16_t *w16;                 /* bf16 copies: [L][(3 d + 35) d] then head [V d] */
    long step;
    KMambaDistributedContext *dist;
    Work w;
};

/* ------------------------------------------------------------------ */
/* layout                                                               */
/* ------------------------------------------------------------------ */

static long layer_size(long d) { return 3 * d * d + NDM_QC * d + 3 * d + 3 * d * NDM_STATE + 27 * d + d; }

static LayerPtrs layer_ptrs(float *base, const KmbNDModel *m, long l) {
    const long d = m->d;
    float *p = base + 2 * m->V * d + l * m->per_layer;
    LayerPtrs r;
    r.W_a = p;
    r.W_z = r.W_a + d * d;
    r.W_out = r.W_z + d * d;
    r.W_p = r.W_out + d * d;
    r.dt_bias = r.W_p + NDM_QC * d;
    r.A_log = r.dt_bias + 3 * d;
    r.conv_kernel = r.A_log + 3 * d * NDM_STATE;
    r.conv_bias = r.conv_kernel + 27 * d;
    return r;
}

/* bf16 copies of a layer's W_a, W_z, W_out, W_p (contiguous, as in the
 * fp32 layout), then the head */
static long w16_layer_elems(const KmbNDModel *m) { return (3 * m->d + NDM_QC) * m->d; }
static uint16_t *w16_layer(const KmbNDModel *m, long l) { return m->w16 + l * w16_layer_elems(m); }
static uint16_t *w16_head(const KmbNDModel *m) { return m->w16 + m->L * w16_layer_elems(m); }

/* ------------------------------------------------------------------ */
/* initialisation (host, counter-based normals)                         */
/* ------------------------------------------------------------------ */

static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
static double unif(uint64_t k) { return ((mix64(k) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
static float gauss(uint64_t k) {
    return (float)(sqrt(-2.0 * log(unif(2 * k))) * cos(6.283185307179586 * unif(2 * k + 1)));
}

static void init_host(const KmbNDModel *m, float *h) {
    const long d = m->d, V = m->V;
    uint64_t k = m->cfg.seed * 0x9e3779b97f4a7c15ull;
    const float sd = (float)(1.0 / sqrt((double)d));
    for (long i = 0; i < V * d; ++i) h[i] = gauss(k++);            /* embedding */
    for (long i = 0; i < V * d; ++i) h[V * d + i] = sd * gauss(k++); /* head */
    for (long l = 0; l < m->L; ++l) {
        LayerPtrs p = layer_ptrs(h, m, l);
        const float so = sd / (float)sqrt(2.0 * (double)m->L);
        for (long i = 0; i < d * d; ++i) p.W_a[i] = sd * gauss(k++);
        for (long i = 0; i < d * d; ++i) p.W_z[i] = sd * gauss(k++);
        for (long i = 0; i < d * d; ++i) p.W_out[i] = so * gauss(k++);
        for (long i = 0; i < NDM_QC * d; ++i) p.W_p[i] = sd * gauss(k++);
        /* dt_bias: softplus(dt_bias) log-uniform in [1e-3, 1e-1] */
        for (long i = 0; i < 3 * d; ++i) {
            const double dt0 = exp(log(1e-3) + unif(k++) * (log(1e-1) - log(1e-3)));
            p.dt_bias[i] = (float)log(expm1(dt0));
        }
        /* A = -1 - exp(A_log) uniform in [-16, -1.5] */
        for (long i = 0; i < 3 * d * NDM_STATE; ++i)
            p.A_log[i] = (float)log(0.5 + 14.5 * unif(k++));
        for (long i = 0; i < 27 * d; ++i) p.conv_kernel[i] = (float)(1.0 / sqrt(27.0)) * gauss(k++);
        for (long i = 0; i < d; ++i) p.conv_bias[i] = 0.f;
    }
}

/* ------------------------------------------------------------------ */
/* helpers                                                              */
/* ------------------------------------------------------------------ */

static int gemm16(const void *A, const void *B, void *C, long M, long N, long K, long lda,
                  long ldb, long ldc, int amn, int bmn, int c16, const float *residual,
                  int accumulate, cudaStream_t s) {
    KmbGemm g;
    memset(&g, 0, sizeof g);
    g.A = A;
    g.B = B;
    g.C = C;
    g.residual = residual;
    g.M = M;
    g.N = N;
    g.K = K;
    g.lda = lda;
    g.ldb = ldb;
    g.ldc = ldc;
    g.ldr = ldc;
    g.a_mn_major = amn;
    g.b_mn_major = bmn;
    g.c_bf16 = c16;
    g.accumulate = accumulate;
    return kmb_launch_gemm_bf16(&g, s);
}

static void *dalloc(size_t bytes, int *rc) {
    void *p = NULL;
    if (*rc) return NULL;
    const cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        *rc = kmb_cuda_fail(e, "ndmodel: cudaMalloc");
        return NULL;
    }
    return p;
}

static void work_free(Work *w) {
    void *all[] = {w->x_store, w->x16, w->g16, w->d16a, w->d16b, w->c16, w->dq16, w->a, w->z,
                   w->v, w->c, w->y, w->tmp1, w->tmp2, w->tmp3, w->q, w->delta, w->ddelta, w->Bs,
                   w->Cs,
                   w->dBs, w->dCs, w->h, w->A, w->dA_tmp, w->ck_tmp, w->cb_tmp, w->logits,
                   w->dlogits, w->l16, w->row_loss,
                   w->tok, w->tgt, w->loss_dev};
    for (size_t i = 0; i < sizeof all / sizeof *all; ++i)
        if (all[i]) cudaFree(all[i]);
    memset(w, 0, sizeof *w);
}

static int work_ensure(KmbNDModel *m, long batch) {
    Work *w = &m->w;
    if (w->batch == batch) return KMB_OK;
    work_free(w);
    const long d = m->d, T = batch * m->P, V = m->V;
    const size_t td = (size_t)T * d;
    int rc = KMB_OK;
    w->x_store = dalloc(sizeof(float) * td * (size_t)(m->L + 1), &rc);
    w->x16 = dalloc(2 * td, &rc);
    w->g16 = dalloc(2 * td, &rc);
    w->d16a = dalloc(2 * td, &rc);
    w->d16b = dalloc(2 * td, &rc);
    w->c16 = dalloc(2 * td, &rc);
    w->dq16 = dalloc(2 * (size_t)T * NDM_QLD, &rc);
    w->a = dalloc(4 * td, &rc);
    w->z = dalloc(4 * td, &rc);
    w->v = dalloc(4 * td, &rc);
    w->c = dalloc(4 * td, &rc);
    w->y = dalloc(4 * td, &rc);
    w->tmp1 = dalloc(4 * td, &rc);
    w->tmp2 = dalloc(4 * td, &rc);
    w->tmp3 = dalloc(4 * td, &rc);
    w->q = dalloc(sizeof(float) * (size_t)T * NDM_QC, &rc);
    w->delta = dalloc(4 * 3 * td, &rc);
    w->ddelta = dalloc(4 * 3 * td, &rc);
    w->Bs = dalloc(sizeof(float) * (size_t)T * NDM_STATE, &rc);
    w->Cs = dalloc(sizeof(float) * (size_t)T * NDM_STATE, &rc);
    w->dBs = dalloc(sizeof(float) * (size_t)T * NDM_STATE, &rc);
    w->dCs = dalloc(sizeof(float) * (size_t)T * NDM_STATE, &rc);
    w->h = dalloc(4 * td * NDM_STATE, &rc);
    w->A = dalloc(sizeof(float) * 3 * (size_t)d * NDM_STATE, &rc);
    w->dA_tmp = dalloc(sizeof(float) * 3 * (size_t)d * NDM_STATE, &rc);
    w->ck_tmp = dalloc(sizeof(float) * 27 * (size_t)d, &rc);
    w->cb_tmp = dalloc(sizeof(float) * (size_t)d, &rc);
    w->logits = dalloc(sizeof(float) * (size_t)T * V, &rc);
    w->dlogits = dalloc(sizeof(float) * (size_t)T * V, &rc);
    w->l16 = dalloc(2 * (size_t)T * V, &rc);
    w->row_loss = dalloc(sizeof(float) * (size_t)T, &rc);
    w->tok = dalloc(sizeof(unsigned) * (size_t)T, &rc);
    w->tgt = dalloc(sizeof(unsigned) * (size_t)T, &rc);
    w->loss_dev = dalloc(sizeof(float), &rc);
    if (rc) {
        work_free(w);
        return rc;
    }
    w->batch = batch;
    return KMB_OK;
}

/* ------------------------------------------------------------------ */
/* one block                                                            */
/* ------------------------------------------------------------------ */

/* Forward of layer l from x_in: leaves a, z, v, c, q, delta, B, C, A, h,
 * y and g16 in the workspace; writes x_out = x_in + g W_out^T when x_out. */
static int block_forward(KmbNDModel *m, long l, long batch, const float *x_in, float *x_out,
                         cudaStream_t s) {
    Work *w = &m->w;
    const long d = m->d, P = m->P, T = batch * P;
    LayerPtrs p = layer_ptrs(m->params, m, l);
    const uint16_t *w16 = w16_layer(m, l);
    int rc = kmb_nd_to_bf16(x_in, d, w->x16, d, T, d, s);
    if (!rc) rc = gemm16(w->x16, w16, w->a, T, d, d, d, d, d, 0, 0, 0, NULL, 0, s);
    if (!rc) rc = gemm16(w->x16, w16 + d * d, w->z, T, d, d, d, d, d, 0, 0, 0, NULL, 0, s);
    if (rc) return rc;
    KmbConvND cv;
    memset(&cv, 0, sizeof cv);
    cv.input = w->a;
    cv.kernel = p.conv_kernel;
    cv.bias = p.conv_bias;
    cv.output = w->v;
    for (int i = 0; i < 3; ++i) cv.dims[i] = m->cfg.dims[i];
    cv.ndims = 3;
    cv.batch = batch;
    cv.D = d;
    cv.K = NDM_K;
    if ((rc = kmb_launch_convnd_fwd(&cv, s))) return rc;
    if ((rc = kmb_nd_silu(w->v, w->c, w->c16, NULL, NULL, T * d, s))) return rc;
    if ((rc = gemm16(w->c16, w16 + 3 * d * d, w->q, T, NDM_QC, d, d, d, NDM_QC, 0, 0, 0, NULL, 0,
                     s)))
        return rc;
    if ((rc = kmb_nd_dt_bc(w->q, NDM_QC, p.dt_bias, w->delta, w->Bs, w->Cs, batch, P, d, s)))
        return rc;
    if ((rc = kmb_nd_neg_exp(p.A_log, w->A, NULL, 3 * d * NDM_STATE, s))) return rc;
    KmbScanND sn;
    memset(&sn, 0, sizeof sn);
    sn.x = w->c;
    sn.delta = w->delta;
    sn.A = w->A;
    sn.B = w->Bs;
    sn.C = w->Cs;
    sn.h = w->h;
    sn.y = w->y;
    for (int i = 0; i < 3; ++i) sn.dims[i] = m->cfg.dims[i];
    sn.ndims = 3;
    sn.batch = batch;
    sn.D = d;
    sn.M = NDM_STATE;
    sn.bc_shared = 1;
    if ((rc = kmb_scannd_fwd(&sn))) return rc;
    if ((rc = kmb_nd_gate(w->y, w->z, w->g16, NULL, NULL, NULL, T * d, s))) return rc;
    if (x_out)
        rc = gemm16(w->g16, w16 + 2 * d * d, x_out, T, d, d, d, d, d, 0, 0, 0, x_in, 0, s);
    return rc;
}

/* Backward of layer l: dx_out (fp32 [T, d], the gradient of x_out) in,
 * dx_in out (may not alias dx_out); parameter gradients into m->grads. */
static int block_backward(KmbNDModel *m, long l, long batch, const float *x_in,
                          const float *dx_out, float *dx_in, int acc, cudaStream_t s) {
    Work *w = &m->w;
    const long d = m->d, P = m->P, T = batch * P;
    LayerPtrs p = layer_ptrs(m->params, m, l);
    LayerPtrs gp = layer_ptrs(m->grads, m, l);
    const uint16_t *w16 = w16_layer(m, l);
    int rc = block_forward(m, l, batch, x_in, NULL, s); /* recompute */
    if (rc) return rc;
    uint16_t *dxo16 = w->d16a;
    float *dg = w->tmp1, *dys = w->tmp2, *dc = w->tmp3;
    if ((rc = kmb_nd_to_bf16(dx_out, d, dxo16, d, T, d, s))) return rc;
    /* out_proj: dg = dx_out W_out, dW_out = dx_out^T g */
    if ((rc = gemm16(dxo16, w16 + 2 * d * d, dg, T, d, d, d, d, d, 0, 1, 0, NULL, 0, s))) return rc;
    if ((rc = gemm16(dxo16, w->g16, gp.W_out, d, d, T, d, d, d, 1, 1, 0, NULL, acc, s))) return rc;
    /* gate */
    uint16_t *dz16 = w->d16b;
    if ((rc = kmb_nd_gate(w->y, w->z, NULL, dg, dys, dz16, T * d, s))) return rc;
    /* scan backward: dc (input gradient), ddelta, dA (into the A_log
     * gradient slot), dB, dC */
    KmbScanND sn;
    memset(&sn, 0, sizeof sn);
    sn.x = w->c;
    sn.delta = w->delta;
    sn.A = w->A;
    sn.B = w->Bs;
    sn.C = w->Cs;
    sn.h = w->h;
    sn.dy = dys;
    sn.dx = dc;
    sn.ddelta = w->ddelta;
    sn.dA = w->dA_tmp;
    sn.dB = w->dBs;
    sn.dC = w->dCs;
    for (int i = 0; i < 3; ++i) sn.dims[i] = m->cfg.dims[i];
    sn.ndims = 3;
    sn.batch = batch;
    sn.D = d;
    sn.M = NDM_STATE;
    sn.bc_shared = 1;
    if ((rc = kmb_scannd_bwd(&sn))) return rc;
    if ((rc = kmb_nd_dalog(p.A_log, w->dA_tmp, gp.A_log, acc, 3 * d * NDM_STATE, s))) return rc;
    /* dt / B / C projection */
    if ((rc = kmb_nd_dt_bwd(w->ddelta, w->q, NDM_QC, p.dt_bias, w->dBs, w->dCs, w->dq16, NDM_QLD,
                            gp.dt_bias, acc, batch, P, d, s)))
        return rc;
    /* dc += dq W_p, dW_p = dq^T c (bf16 operands, K of 35 zero-padded to the tile) */
    if ((rc = gemm16(w->dq16, w16 + 3 * d * d, dc, T, d, NDM_QC, NDM_QLD, d, d, 0, 1, 0, NULL, 1,
                     s)))
        return rc;
    if ((rc = gemm16(w->dq16, w->c16, gp.W_p, NDM_QC, d, T, NDM_QLD, d, d, 1, 1, 0, NULL, acc, s)))
        return rc;
    /* silu, then ConvND backward: da in tmp1 (dg is dead) */
    float *dv = dys, *da = dg;
    if ((rc = kmb_nd_silu(w->v, NULL, NULL, dc, dv, T * d, s))) return rc;
    KmbConvND cv;
    memset(&cv, 0, sizeof cv);
    cv.input = w->a;
    cv.kernel = p.conv_kernel;
    cv.dy = dv;
    cv.dinput = da;
    cv.dkernel = acc ? w->ck_tmp : gp.conv_kernel;
    cv.dbias = acc ? w->cb_tmp : gp.conv_bias;
    for (int i = 0; i < 3; ++i) cv.dims[i] = m->cfg.dims[i];
    cv.ndims = 3;
    cv.batch = batch;
    cv.D = d;
    cv.K = NDM_K;
    if ((rc = kmb_launch_convnd_bwd(&cv, s))) return rc;
    if (acc && ((rc = kmb_axpby(gp.conv_kernel, w->ck_tmp, 27 * d, 1.f, 1.f, s)) ||
                (rc = kmb_axpby(gp.conv_bias, w->cb_tmp, d, 1.f, 1.f, s))))
        return rc;
    /* in_proj: dx_in = dx_out + da W_a + dz W_z; dW_a = da^T x, dW_z = dz^T x */
    uint16_t *da16 = w->d16a;
    if ((rc = kmb_nd_to_bf16(da, d, da16, d, T, d, s))) return rc;
    if ((rc = gemm16(da16, w16, dx_in, T, d, d, d, d, d, 0, 1, 0, dx_out, 0, s))) return rc;
    if ((rc = gemm16(dz16, w16 + d * d, dx_in, T, d, d, d, d, d, 0, 1, 0, NULL, 1, s))) return rc;
    if ((rc = gemm16(da16, w->x16, gp.W_a, d, d, T, d, d, d, 1, 1, 0, NULL, acc, s))) return rc;
    return gemm16(dz16, w->x16, gp.W_z, d, d, T, d, d, d, 1, 1, 0, NULL, acc, s);
}

/* ------------------------------------------------------------------ */
/* model                                                                */
/* ------------------------------------------------------------------ */

static int refresh_w16(KmbNDModel *m, cudaStream_t s) {
    const long d = m->d;
    for (long l = 0; l < m->L; ++l) {
        LayerPtrs p = layer_ptrs(m->params, m, l);
        int rc = kmb_nd_to_bf16(p.W_a, d, w16_layer(m, l), d, 3 * d + NDM_QC, d, s);
        if (rc) return rc;
    }
    return kmb_nd_to_bf16(m->params + m->V * d, d, w16_head(m), d, m->V, d, s);
}

KmbNDModel *kmb_ndmodel_create(const KmbNDModelConfig *cfg) {
    if (!cfg || cfg->dim <= 0 || cfg->dim % 32 || cfg->n_layers <= 0 || cfg->vocab <= 0 ||
        cfg->vocab % 8) {
        kmb_fail(KMB_EINVAL, "ndmodel: dim must be a positive multiple of 32, n_layers > 0, "
                             "vocab a positive multiple of 8");
        return NULL;
    }
    long P = 1;
    for (int i = 0; i < 3; ++i) {
        if (cfg->dims[i] <= 0) {
            kmb_fail(KMB_EINVAL, "ndmodel: dims must be positive");
            return NULL;
        }
        P *= cfg->dims[i];
    }
    KmbNDModel *m = (KmbNDModel *)calloc(1, sizeof *m);
    if (!m) {
        kmb_fail(KMB_ENOMEM, "ndmodel: host allocation failed");
        return NULL;
    }
    m->cfg = *cfg;
    m->P = P;
    m->d = cfg->dim;
    m->L = cfg->n_layers;
    m->V = cfg->vocab;
    m->per_layer = layer_size(m->d);
    m->n = 2 * m->V * m->d + m->L * m->per_layer;
    int rc = KMB_OK;
    const size_t nb = sizeof(float) * (size_t)m->n;
    m->params = dalloc(nb, &rc);
    m->grads = dalloc(nb, &rc);
    m->m = dalloc(nb, &rc);
    m->v = dalloc(nb, &rc);
    m->w16 = dalloc(2 * ((size_t)m->L * w16_layer_elems(m) + (size_t)m->V * m->d), &rc);
    float *host = rc ? NULL : (float *)malloc(nb);
    if (!rc && !host) rc = kmb_fail(KMB_ENOMEM, "ndmodel: host allocation failed");
    if (!rc) {
        init_host(m, host);
        cudaError_t e = cudaMemcpy(m->params, host, nb, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(m->m, 0, nb);
        if (e == cudaSuccess) e = cudaMemset(m->v, 0, nb);
        if (e == cudaSuccess) e = cudaMemset(m->grads, 0, nb);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "ndmodel: initial copy");
    }
    free(host);
    if (!rc) rc = refresh_w16(m, kmb_stream());
    if (!rc) {
        const cudaError_t e = cudaStreamSynchronize(kmb_stream());
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "ndmodel: synchronize");
    }
    if (rc) {
        kmb_ndmodel_free(m);
        return NULL;
    }
    return m;
}

void kmb_ndmodel_free(KmbNDModel *m) {
    if (!m) return;
    cudaStreamSynchronize(kmb_stream());
    work_free(&m->w);
    void *all[] = {m->params, m->grads, m->m, m->v, m->w16};
    for (size_t i = 0; i < sizeof all / sizeof *all; ++i)
        if (all[i]) cudaFree(all[i]);
    free(m);
}

long kmb_ndmodel_param_count(const KmbNDModel *m) { return m ? m->n : 0; }
float *kmb_ndmodel_params(KmbNDModel *m) { return m ? m->params : NULL; }
float *kmb_ndmodel_grads(KmbNDModel *m) { return m ? m->grads : NULL; }

static int finish(int rc) {
    if (rc || !kmb_sync_enabled()) return rc;
    const cudaError_t e = cudaStreamSynchronize(kmb_stream());
    if (e != cudaSuccess) return kmb_cuda_fail(e, "ndmodel: synchronize");
    return kmb_gemm_check_error();
}

int kmb_ndmodel_sync_weights(KmbNDModel *m) {
    if (!m) return kmb_fail(KMB_EINVAL, "ndmodel: NULL model");
    return finish(refresh_w16(m, kmb_stream()));
}

int kmb_ndmodel_set_dist(KmbNDModel *m, KMambaDistributedContext *ctx) {
    if (!m) return kmb_fail(KMB_EINVAL, "ndmodel: NULL model");
    m->dist = ctx;
    return KMB_OK;
}

/* Tokens to the workspace, forward through every layer and the head;
 * leaves logits, dlogits (of the mean loss) and the loss on the device. */
static int forward_all(KmbNDModel *m, const unsigned *tokens, long batch, float weight,
                       cudaStream_t s) {
    Work *w = &m->w;
    const long d = m->d, T = batch * m->P;
    int rc = KMB_OK;
    const cudaError_t e = cudaMemcpyAsync(w->tok, tokens, sizeof(unsigned) * (size_t)T,
                                          cudaMemcpyDefault, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "ndmodel: tokens");
    if ((rc = kmb_embed(m->params, w->tok, T, d, m->V, w->x_store, NULL, NULL, s))) return rc;
    for (long l = 0; l < m->L; ++l) {
        float *xi = w->x_store + (size_t)l * T * d;
        if ((rc = block_forward(m, l, batch, xi, xi + (size_t)T * d, s))) return rc;
    }
    const float *xL = w->x_store + (size_t)m->L * T * d;
    if ((rc = kmb_nd_to_bf16(xL, d, w->x16, d, T, d, s))) return rc;
    if ((rc = gemm16(w->x16, w16_head(m), w->logits, T, m->V, d, d, d, m->V, 0, 0, 0, NULL, 0, s)))
        return rc;
    if ((rc = kmb_nd_roll_targets(w->tok, w->tgt, batch, m->P, s))) return rc;
    if ((rc = kmb_softmax_ce(w->logits, w->tgt, T, m->V, w->dlogits, w->row_loss, s))) return rc;
    /* this pass's share of the batch mean */
    if (weight != 1.f && (rc = kmb_axpby(w->dlogits, NULL, T * m->V, weight, 0.f, s))) return rc;
    return kmb_nd_mean(w->row_loss, T, w->loss_dev, s);
}

/* Volumes per pass: the configured micro-batch, or as many as fit in
 * 85 % of the free device memory (at least one). */
static long micro_batch(KmbNDModel *m, long batch) {
    if (m->cfg.micro_batch > 0) return m->cfg.micro_batch < batch ? m->cfg.micro_batch : batch;
    if (m->w.batch > 0 && m->w.batch <= batch) return m->w.batch;
    size_t freeb = 0, total = 0;
    if (cudaMemGetInfo(&freeb, &total) != cudaSuccess) {
        (void)cudaGetLastError();
        return 1;
    }
    /* per volume: residual stream of every layer, ~14 [P, d] fp32
     * activations, 6 for the two delta tensors, the scan history and the
     * scan's adjoint buffer (16 each), and the head's [P, vocab] buffers */
    const double per = 4.0 * m->P * m->d * (m->L + 1 + 14 + 6 + 32) + 12.0 * m->P * m->V;
    long mb = (long)(0.85 * (double)freeb / per);
    if (mb < 1) mb = 1;
    return mb < batch ? mb : batch;
}

static int read_loss(KmbNDModel *m, float *loss, cudaStream_t s) {
    if (!loss) return KMB_OK;
    cudaError_t e = cudaMemcpyAsync(loss, m->w.loss_dev, sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "ndmodel: loss");
}

static int check_call(KmbNDModel *m, const unsigned *tokens, long batch) {
    if (!m || !tokens) return kmb_fail(KMB_EINVAL, "ndmodel: NULL model or tokens");
    if (batch <= 0) return kmb_fail(KMB_EINVAL, "ndmodel: batch must be positive");
    kmb_clear_error();
    return KMB_OK;
}

int kmb_ndmodel_forward(KmbNDModel *m, const unsigned *tokens, long batch, float *loss) {
    int rc = check_call(m, tokens, batch);
    if (rc) return rc;
    const cudaStream_t s = kmb_stream();
    const long mb = micro_batch(m, batch);
    if ((rc = work_ensure(m, mb))) return rc;
    double total = 0.0;
    for (long i0 = 0; i0 < batch && !rc; i0 += mb) {
        const long bi = batch - i0 < mb ? batch - i0 : mb;
        float li = 0.f;
        rc = forward_all(m, tokens + i0 * m->P, bi, 1.f, s);
        if (!rc) rc = read_loss(m, &li, s);
        total += (double)li * (double)bi;
    }
    if (!rc && loss) *loss = (float)(total / (double)batch);
    return finish(rc);
}

/* One pass of forward + backward over `batch` volumes; gradients are
 * written (acc == 0) or added (acc == 1); the NCCL buckets are fed when
 * `last`. */
static int pass_backward(KmbNDModel *m, const unsigned *tokens, long batch, float weight,
                         int acc, int last, float *loss, cudaStream_t s) {
    int rc = forward_all(m, tokens, batch, weight, s);
    if (rc) return rc;
    Work *w = &m->w;
    const long d = m->d, T = batch * m->P, V = m->V;
    const size_t td = (size_t)T * d;
    void *sp = (void *)s;
    const int feed = last && m->dist;
    float *g_emb = m->grads, *g_head = m->grads + V * d;
    /* Gradient slots: the residual stream x_l sits in x_store slot l.  Once
     * layer l's backward has read x_l (its recompute converts it to bf16
     * first), slot l is free and receives d x_l; the gradient of x_{l+1}
     * is in slot l + 1 at that point.  x_L's slot takes d x_L after the
     * head's backward, whose weight gradient reads the bf16 copy of x_L. */
    if ((rc = kmb_nd_to_bf16(w->dlogits, V, w->l16, V, T, V, s))) return rc;
    if ((rc = gemm16(w->l16, w->x16, g_head, V, d, T, V, d, d, 1, 1, 0, NULL, acc, s))) return rc;
    if ((rc = gemm16(w->l16, w16_head(m), w->x_store + (size_t)m->L * td, T, d, V, V, d, d, 0,
                     1, 0, NULL, 0, s)))
        return rc;
    if (feed && (rc = kmb_dist_bucket_add(m->dist, g_head, (size_t)V * d, 1, sp))) return rc;
    for (long l = m->L - 1; l >= 0; --l) {
        float *slot = w->x_store + (size_t)l * td;
        if ((rc = block_backward(m, l, batch, slot, slot + td, slot, acc, s))) return rc;
        LayerPtrs gp = layer_ptrs(m->grads, m, l);
        if (feed && (rc = kmb_dist_bucket_add(m->dist, gp.W_a, (size_t)m->per_layer, 1, sp)))
            return rc;
    }
    /* embedding: scatter-add d x_0 */
    if (!acc) {
        const cudaError_t e = cudaMemsetAsync(g_emb, 0, sizeof(float) * (size_t)V * d, s);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "ndmodel: embedding gradient memset");
    }
    if ((rc = kmb_embed(NULL, w->tok, T, d, V, NULL, w->x_store, g_emb, s))) return rc;
    if (feed) {
        if ((rc = kmb_dist_bucket_add(m->dist, g_emb, (size_t)V * d, 1, sp))) return rc;
        if ((rc = kmb_dist_bucket_flush(m->dist, sp))) return rc;
        if ((rc = kmb_dist_wait(m->dist, sp))) return rc;
    }
    return read_loss(m, loss, s);
}

int kmb_ndmodel_backward(KmbNDModel *m, const unsigned *tokens, long batch, float *loss) {
    int rc = check_call(m, tokens, batch);
    if (rc) return rc;
    const cudaStream_t s = kmb_stream();
    const long mb = micro_batch(m, batch);
    if ((rc = work_ensure(m, mb))) return rc;
    double total = 0.0;
    for (long i0 = 0; i0 < batch && !rc; i0 += mb) {
        const long bi = batch - i0 < mb ? batch - i0 : mb;
        float li = 0.f;
        rc = pass_backward(m, tokens + i0 * m->P, bi, (float)bi / (float)batch, i0 > 0,
                           i0 + bi >= batch, &li, s);
        total += (double)li * (double)bi;
    }
    if (!rc && loss) *loss = (float)(total / (double)batch);
    return finish(rc);
}

int kmb_ndmodel_step(KmbNDModel *m, float lr, float weight_decay) {
    if (!m) return kmb_fail(KMB_EINVAL, "ndmodel: NULL model");
    const cudaStream_t s = kmb_stream();
    m->step++;
    const float b1 = 0.9f, b2 = 0.999f;
    const float bc1 = 1.f - powf(b1, (float)m->step), bc2 = 1.f - powf(b2, (float)m->step);
    int rc = kmb_adamw(m->params, m->grads, m->m, m->v, m->n, lr, b1, b2, 1e-8f, weight_decay,
                       bc1, bc2, s);
    if (!rc) rc = refresh_w16(m, s);
    return finish(rc);
}

int kmb_ndmodel_train_step(KmbNDModel *m, const unsigned *tokens, long batch, float lr,
                           float weight_decay, float *loss) {
    int rc = kmb_ndmodel_backward(m, tokens, batch, loss);
    if (rc) return rc;
    return kmb_ndmodel_step(m, lr, weight_decay);
}
