/*
 * Internal ABI between the C host layer (csrc/host) and the CUDA
 * launchers (csrc/cuda).  Plain C types only; every launcher takes
 * device pointers and a cudaStream_t and returns a KMB_* status.
 */
#ifndef KMB_INTERNAL_H
#define KMB_INTERNAL_H

#include <stddef.h>
#include <cuda_runtime_api.h>
#include "kmamba_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Records a status and a message for kmb_last_error(); returns status. */
int kmb_fail(int status, const char *fmt, ...);
int kmb_cuda_fail(cudaError_t e, const char *where);

/* 1D selective scan launchers (csrc/cuda/scan1d.cu).  The host layer sets
 * KMB_SCAN1D_DA_ACCUM in KmbScan1D.flags (after validating the caller's
 * zero) when it launches a call's batch in slices: the backward then
 * accumulates into dA instead of zeroing it first. */
#define KMB_SCAN1D_DA_ACCUM 0x10000
int kmb_launch_scan1d_fwd(const KmbScan1D *a, cudaStream_t s);
int kmb_launch_scan1d_bwd(const KmbScan1D *a, const float *ckpt_in,
                          cudaStream_t s);
/* Sequence-split kernels for the channel-shared layout (csrc/cuda/
 * scan1d_seg.cu).  bf16: x, dt, B, C, y, dy, dx, ddt (and dB / dC after the
 * fp32 accumulation in dB32 / dC32) are bf16.  seg_state holds batch * S *
 * D * 16 floats, flag batch * (D / 32) * S ints. */
int kmb_scan1d_seg_supported(const KmbScan1D *a, int elem_bytes);
int kmb_scan1d_seg_plan(long batch, long L, long D, int *S, int *seg_len);
/* Diagnostic (exported for the tests): out[i] = kmb_exp2_fma2(w[i]), the
 * FMA-pipe 2^w of csrc/cuda/kmb_common.cuh, on device pointers. */
int kmb_exp2_fma_eval(const float *w, float *out, long n);
int kmb_launch_scan1d_fwd_seg(const KmbScan1D *a, int bf16, int S, int seg_len,
                              float *seg_state, int *flag, cudaStream_t s);
int kmb_launch_scan1d_bwd_seg(const KmbScan1D *a, const float *ckpt_in, int bf16, int S,
                              int seg_len, float *seg_state, int *flag, float *dB32,
                              float *dC32, cudaStream_t s);
int kmb_launch_scan1d_bwd_m1_shared(const float *x, const float *A,
                                    const float *A_diag, const float *B,
                                    const float *C, const float *delta,
                                    const float *h0, const float *h,
                                    const float *dy, float *dx, float *dA,
                                    float *dB, float *dC, float *ddelta,
                                    long L, long D, cudaStream_t s);

/* ConvND launchers (csrc/cuda/convnd.cu). */
int kmb_launch_convnd_fwd(const KmbConvND *a, cudaStream_t s);
int kmb_launch_convnd_bwd(const KmbConvND *a, cudaStream_t s);
/* bf16 activations: shapes kmb_convnd_bf16_supported accepts */
int kmb_convnd_bf16_supported(const KmbConvND *a, int bwd);
int kmb_launch_convnd_fwd_bf16(const KmbConvND *a, cudaStream_t s);
int kmb_launch_convnd_bwd_bf16(const KmbConvND *a, cudaStream_t s);

/* ND scan launchers (csrc/cuda/scannd.cu).  Per-axis pointers so that
 * both the contiguous [ndims, P, D] delta of scan_nd.h and the separate
 * delta1 / delta2 of scan2d map onto the same kernels. */
#define KMB_MAX_AXES 8
typedef struct {
    const float *x, *B, *C, *dy;
    float *h, *y, *G, *dx, *dB, *dC;
    const float *delta[KMB_MAX_AXES];
    const float *A[KMB_MAX_AXES];
    float *dA[KMB_MAX_AXES];
    float *ddelta[KMB_MAX_AXES];
    const int *lvl_start, *lvl_off, *prev, *next;
    const int *sprev, *snext; /* prev / next in level-slot order */
    long P, D, M, batch;
    long delta_bstride; /* floats between batch items of each delta axis */
    long dims[KMB_MAX_AXES];
    float *scratch;       /* device scratch of the 2D kernels */
    size_t scratch_elems;
    int nd, nlevels, bc_shared;
} KmbNDLaunch;
int kmb_launch_scannd_fwd(const KmbNDLaunch *a, cudaStream_t s);
int kmb_launch_scannd_bwd(const KmbNDLaunch *a, cudaStream_t s);
/* 2D wavefront kernels (csrc/cuda/scan2d.cu) for nd == 2 with channel-shared
 * B/C, M a multiple of 4 up to 16 and D a multiple of 8; KMB_EUNSUPPORTED
 * for other shapes (the generic ND kernels take those). */
int kmb_launch_scan2d_fwd(const KmbNDLaunch *a, cudaStream_t s);
int kmb_launch_scan2d_bwd(const KmbNDLaunch *a, cudaStream_t s);
int kmb_scan2d_supported(const KmbNDLaunch *a);
/* bf16 tensors in the 2D kernels (M 8 or 16); the backward accumulates the
 * channel sums dB / dC in the fp32 buffers dB32 / dC32, then rounds them
 * into the bf16 outputs. */
int kmb_scan2d_bf16_supported(const KmbNDLaunch *a);
int kmb_launch_scan2d_fwd_bf16(const KmbNDLaunch *a, cudaStream_t s);
int kmb_launch_scan2d_bwd_bf16(const KmbNDLaunch *a, float *dB32, float *dC32, cudaStream_t s);
/* Elementwise conversions (round to nearest even to bf16). */
int kmb_launch_bf16_to_f32(const void *src, float *dst, long n, cudaStream_t s);
int kmb_launch_f32_to_bf16(const float *src, void *dst, long n, cudaStream_t s);
size_t kmb_scan2d_scratch_elems(const KmbNDLaunch *a);
/* KMB_ETIMEOUT once after a strip-split wait of the 2D kernels expired. */
int kmb_scan2d_check_error(void);

/* tcgen05 bf16 GEMM (csrc/cuda/gemm_tc.cu); operands already validated. */
int kmb_launch_gemm_bf16(const KmbGemm *g, cudaStream_t s);

/* Mamba-ND block pieces (csrc/cuda/ndblock.cu). */
int kmb_nd_to_bf16(const float *src, long lds, void *dst, long ldd, long rows, long cols,
                   cudaStream_t s);
int kmb_nd_silu(const float *v, float *c, void *c16, const float *dc, float *dv, long n,
                cudaStream_t s);
int kmb_nd_dt_bc(const float *q, long qld, const float *dtb, float *delta, float *B, float *C,
                 long batch, long P, long d, cudaStream_t s);
int kmb_nd_gate(const float *y, const float *z, void *g16, const float *dg, float *dy,
                void *dz16, long n, cudaStream_t s);
int kmb_nd_dt_bwd(const float *ddelta, const float *q, long qld, const float *dtb,
                  const float *dB, const float *dC, void *dq16, long dq_ld, float *ddtb, int acc,
                  long batch, long P, long d, cudaStream_t s);
int kmb_nd_dalog(const float *A_log, const float *dA, float *g, int acc, long n, cudaStream_t s);
int kmb_nd_neg_exp(const float *A_log, float *A, float *dA_inout, long n, cudaStream_t s);
int kmb_nd_roll_targets(const unsigned *tok, unsigned *tgt, long batch, long P, cudaStream_t s);
int kmb_nd_mean(const float *x, long n, float *out, cudaStream_t s);

/* Block / model kernels (csrc/cuda/block.cu). */
/* C[m*ldc + n] (+)= sum_k A[m*am + k*ak] * B[k*bk + n*bn], fp32.  ws
 * (ws_elems floats, may be NULL) lets small output grids split K across
 * CTAs; the partials are added in a fixed order. */
int kmb_gemm(int M, int N, int K, const float *A, long am, long ak, const float *B, long bk,
             long bn, float *C, long ldc, int accumulate, float *ws, size_t ws_elems,
             cudaStream_t s);
/* projection activations (dz_inplace == NULL) or their backward in place */
int kmb_block_act(const float *zraw, float *zact, const float *bB, const float *bC, long rows,
                  int W, int R, int NR, float dt_min, float dt_max, int has_dp, int has_lp,
                  float dt_scale, float *dz_inplace, cudaStream_t s);
int kmb_colsum_acc(const float *dz, long rows, int W, int c0, int ncols, float *out,
                   cudaStream_t s);
/* Mamba-3 scan forward (dy == NULL) or backward.  `part` holds
 * batch * kmb_m3_scan_groups(N) * L * (R + 2) floats of per-warp partial
 * sums. */
int kmb_m3_scan(int batch, int L, int N, int R, int W, const float *zact, const float *A,
                const float *theta, float *h_hist, float *h_last, float *y, const float *dy,
                float *dz, float *dA, float *dtheta, float *part, cudaStream_t s);
int kmb_m3_scan_groups(int N);
/* embedding gather (gemb == NULL) or gradient scatter-add */
int kmb_embed(const float *emb, const unsigned *tok, long L, long D, long V, float *out,
              const float *dx_for_grad, float *gemb, cudaStream_t s);
int kmb_softmax_ce(const float *logits, const unsigned *tgt, long L, long V, float *dlogits,
                   float *row_loss, cudaStream_t s);
int kmb_adamw(float *p, const float *g, float *m, float *v, long n, float lr, float b1,
              float b2, float eps, float wd, float bc1, float bc2, cudaStream_t s);
int kmb_sumsq(const float *x, long n, double *out, cudaStream_t s);
/* the same over up to 16 tensors in one launch */
int kmb_adamw_multi(int cnt, float *const *p, const float *const *g, float *const *m,
                    float *const *v, const long *n, float lr, float b1, float b2, float eps,
                    float wd, float bc1, float bc2, cudaStream_t s);
int kmb_sumsq_multi(int cnt, const float *const *x, const long *n, double *const *out,
                    cudaStream_t s);
/* y = a*y + b*x (x may be NULL: y = a*y) */
int kmb_axpby(float *y, const float *x, long n, float a, float b, cudaStream_t s);
/* out = clamp(softplus(z), dt_min, dt_max) */
int kmb_dt_act(const float *z, float *out, long n, float dt_min, float dt_max, cudaStream_t s);
/* MUON pieces: m = mu*m + g;  G = 1.5G - 0.5T;  p -= lr*x*clip_scale(sumsq) */
int kmb_momentum(float *m, const float *g, long n, float mu, cudaStream_t s);
int kmb_ns_combine(float *G, const float *T, long n, cudaStream_t s);
int kmb_scaled_sub(float *p, const float *x, long n, float lr, float clip, const double *sumsq,
                   cudaStream_t s);

/* Device copy of a grid's wavefront schedule (csrc/host/plan_cache.c):
 * level starts / offsets of km_wavefront_plan_create as int32 plus the
 * predecessor (p - e_axis) and successor (p + e_axis) offsets, -1 outside
 * the grid.  Cached per (device, dims); valid until kmb_plan_cache_clear. */
typedef struct {
    const int *lvl_start; /* [nlevels + 1] */
    const int *lvl_off;   /* [P] */
    const int *prev;      /* [P * nd] */
    const int *next;      /* [P * nd] */
    const int *sprev;     /* [P * nd]: prev of the point in level slot s at [s * nd] */
    const int *snext;     /* [P * nd]: next, in the same slot order */
    long P;
    int nlevels;
    int nd;
} KmbDevPlan;
int kmb_dev_plan(const long *dims, long ndims, KmbDevPlan *out);

/* ------------------------------------------------------------------ */
/* host runtime (csrc/host/runtime.c)                                   */
/* ------------------------------------------------------------------ */
cudaStream_t kmb_stream(void);
int kmb_sync_enabled(void);
/* 1 when p is device-accessible memory (device or managed). */
int kmb_is_device_ptr(const void *p);

/*
 * Staging of caller buffers.  kmb_stage_in/out return a device pointer:
 * the caller's own pointer when it is device memory, else a pooled device
 * buffer (inputs are copied host->device on the library stream; outputs
 * are copied back by kmb_stage_finish).  Passing the same host pointer
 * twice returns the same device buffer.
 */
#define KMB_STAGE_MAX 64
typedef struct {
    const void *user;
    void *dev;
    size_t bytes;
    int out;     /* copy back on finish */
    int owned;   /* dev is a pool block */
} KmbStageBuf;
typedef struct {
    KmbStageBuf inl[KMB_STAGE_MAX];
    KmbStageBuf *b;   /* inl, or a heap table from kmb_stage_reserve */
    int cap;
    int n;
    int status;
    cudaStream_t s;
} KmbStage;

/* Device-resident host arrays (kmamba_set_device_resident): staging returns
 * the registered device copy of such an array and copies nothing.  add
 * (re-)uploads the host value; update re-uploads only registered arrays;
 * sync copies the device value back; remove drops the registration (after
 * a copy back when asked). */
int kmb_resident_add(const void *host, size_t bytes);
int kmb_resident_update(const void *host); /* re-upload when registered */
int kmb_resident_sync(void *host);
int kmb_resident_remove(void *host, int copy_back);
int kmb_resident_count(void);
void kmb_stage_begin(KmbStage *st);
/* Grows the table to hold `cap` buffers (model calls that move every
 * parameter, gradient and moment of every layer).  Call right after
 * kmb_stage_begin. */
int kmb_stage_reserve(KmbStage *st, int cap);
void *kmb_stage_in(KmbStage *st, const void *p, size_t bytes);
void *kmb_stage_out(KmbStage *st, void *p, size_t bytes, int copy_in);
void *kmb_scratch(KmbStage *st, size_t bytes);
/* Copies outputs back (when status is OK), synchronizes when needed and
 * releases pooled buffers.  Returns the first error seen. */
int kmb_stage_finish(KmbStage *st, int status);

#ifdef __cplusplus
}
#endif

#endif
