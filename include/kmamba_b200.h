#ifndef KMAMBA_B200_H
#define KMAMBA_B200_H

/*
 * B200 extensions of the k-mamba C API: status-returning, batched entry
 * points for the hot path, and the runtime controls they share.  All
 * entry points run on the GPU; pointers may be device memory (used in
 * place) or host memory (staged through pooled device buffers inside the
 * call).  Nothing here falls back to the CPU.
 */

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every kmb_* entry point. */
#define KMB_OK            0
#define KMB_EINVAL       -1   /* bad pointer, size or layout */
#define KMB_ECUDA        -2   /* CUDA runtime / launch failure */
#define KMB_ENOMEM       -3   /* device or host allocation failed */
#define KMB_ETIMEOUT     -4   /* a bounded device-side wait gave up */
#define KMB_EUNSUPPORTED -5   /* shape outside what the kernels support */

/* Message and status of the last failure on the calling thread. */
const char *kmb_last_error(void);
int kmb_last_status(void);
void kmb_clear_error(void);

/* Stream used by every entry point of the library (a cudaStream_t; NULL
 * = legacy default stream).  Per calling thread. */
void kmb_set_stream(void *cuda_stream);
void *kmb_get_stream(void);

/* When on (default), entry points synchronize the stream before they
 * return, which the reference API requires.  With it off, kmb_* calls on
 * device pointers are asynchronous on the library stream. */
void kmb_set_sync(int on);
int kmb_get_sync(void);

/* Device buffer pool (replaces the reference's host km_memory_pool for
 * device scratch).  Blocks are cached per device and reused by size. */
void *kmb_pool_alloc(size_t bytes);
void kmb_pool_free(void *dptr);
/* Frees every cached, unused block; returns the bytes released. */
size_t kmb_pool_trim(void);
/* Bytes currently held from cudaMalloc (in use + cached). */
size_t kmb_pool_bytes_held(void);

/* Number of kernels the block / model path (kmamba.h) has launched in
 * this process, for measurement.  No reference counterpart. */
unsigned long long kmb_block_launch_count(void);

/* ------------------------------------------------------------------ */
/* Batched 1D selective scan                                           */
/* ------------------------------------------------------------------ */
/*
 * For every batch item b, channel d and state n:
 *   h_t = exp(dt_t*A[d,n]) * h_{t-1} + dt_t*B_t[n]*x_t      (h_{-1} = h0)
 *   y_t = sum_n C_t[n] * h_t
 * with x, dt, y [batch, L, D] and A [D, N].  B and C are [batch, L, N]
 * (shared by all channels) when bc_shared, else [batch, L, D, N].
 *
 * Forward outputs: y (may be NULL), h_last [batch, D, N], h_all
 * [batch, L, D, N] and ckpt (states every KMB_SCAN1D_CHUNK steps, size
 * kmb_scan1d_ckpt_elems()); each optional output may be NULL.
 *
 * Backward: reads dy and either h_all (stored states, the reference
 * contract) or ckpt (written by the forward); when both are NULL the
 * checkpoints are computed into pooled scratch.  Writes dx, ddt
 * [batch, L, D], dA [D, N] (summed over the batch) and dB, dC (same layout
 * as B, C; summed over D when bc_shared).  Every gradient is overwritten.
 * The backward treats the clamp as the identity, like the reference.
 */
/* Steps between two forward checkpoints (the backward's chunk length). */
#define KMB_SCAN1D_CHUNK 8

typedef struct {
    const float *x;
    const float *dt;
    const float *A;
    const float *B;
    const float *C;
    const float *h0;
    float *y;
    float *h_last;
    float *h_all;
    float *ckpt;
    const float *dy;
    float *dx;
    float *ddt;
    float *dA;
    float *dB;
    float *dC;
    long batch;
    long L;
    long D;
    long N;
    int bc_shared;
    int clamp;       /* 1: clamp states to [-1000, 1000] after every step */
    int flags;       /* reserved, must be 0 */
    int pad_;
} KmbScan1D;

long kmb_scan1d_ckpt_elems(long batch, long L, long D, long N);
int kmb_scan1d_fwd(const KmbScan1D *args);
int kmb_scan1d_bwd(const KmbScan1D *args);

/*
 * bf16-I/O variants of the same forward and backward (the reference has
 * only host-side bf16 conversions, include/kmamba_mixed_precision.h:
 * 106-112, which truncate).  x, dt, B, C, y, dy, dx, ddt, dB and dC point to
 * bf16 (rounded to nearest even on output); A, dA, h0, h_last and ckpt stay
 * fp32; arithmetic is fp32.  Device memory only, for the channel-shared
 * layout: bc_shared = 1, N = 16, D a multiple of 32, h_all = NULL, 16-byte
 * aligned tensors; other shapes return KMB_EUNSUPPORTED.
 */
int kmb_scan1d_fwd_bf16(const KmbScan1D *args);
int kmb_scan1d_bwd_bf16(const KmbScan1D *args);

/*
 * kmb_scan1d_bwd_noalloc -- no counterpart in the reference.
 *
 * The same backward as kmb_scan1d_bwd with h_all = ckpt = NULL, for
 * callers that cannot allocate device memory while it runs: a host whose
 * device memory is owned by another allocator (a framework's caching
 * allocator that has reserved it, so cudaMalloc would fail or fragment
 * its pool), a latency-bound loop that cannot absorb the device-wide
 * synchronisation cudaMalloc / cudaFree may impose, or a plugin host that
 * forbids allocations outside its own set-up phase.  It allocates nothing
 * and stages nothing: every pointer must be device memory, h_all and ckpt
 * must be NULL.  Every tensor must be memory of the current device.  The
 * forward checkpoints live in a static device array of
 * KMB_NOALLOC_CKPT_ELEMS floats (8 MiB, held by every GPU that has loaded
 * the library's device code, until exit); a call needing more -- batch *
 * ceil(L / KMB_SCAN1D_CHUNK) * D * N floats -- is rejected with
 * KMB_EUNSUPPORTED.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress); with lazy module loading, the
 * CUDA 12 default, that lookup is also what loads the module and its
 * 8 MiB onto the device, which allocates and can synchronise.  So make a
 * warm-up call during your own set-up phase, before any stream capture.
 * The address is cached per device and not refreshed after
 * cudaDeviceReset: do not use the entry point across a reset.  All calls
 * share the array: calls that overlap on the GPU race on it.
 */
#define KMB_NOALLOC_CKPT_ELEMS (2L * 1024 * 1024)
int kmb_scan1d_bwd_noalloc(const KmbScan1D *args);

/* ------------------------------------------------------------------ */
/* Batched causal depthwise ConvND                                     */
/* ------------------------------------------------------------------ */
/*
 * Per batch item the semantics of convnd() (convnd.h): input, output, dy,
 * dinput [batch, prod(dims), D]; kernel, dkernel [K^ndims, D]; bias,
 * dbias [D] (bias / dbias may be NULL).  The backward overwrites dinput
 * and writes dkernel / dbias summed over the batch.
 */
typedef struct {
    const float *input;
    const float *kernel;
    const float *bias;
    float *output;
    const float *dy;
    float *dinput;
    float *dkernel;
    float *dbias;
    long dims[8];
    long ndims;
    long batch;
    long D;
    long K;
} KmbConvND;

int kmb_convnd_fwd(const KmbConvND *args);
int kmb_convnd_bwd(const KmbConvND *args);

/*
 * The same with bf16 activations: input, output, dy and dinput point to
 * bf16 device memory (output and dinput rounded to nearest even); kernel,
 * bias, dkernel and dbias stay fp32, and every product and sum is fp32.
 * Shapes: 2D with D a multiple of 64, or 3D with D a multiple of 8; K <= 3;
 * 16-byte aligned device tensors (KMB_EUNSUPPORTED otherwise).
 */
int kmb_convnd_fwd_bf16(const KmbConvND *args);
int kmb_convnd_bwd_bf16(const KmbConvND *args);

/* ------------------------------------------------------------------ */
/* Batched ND selective scan with stored states                        */
/* ------------------------------------------------------------------ */
/*
 * Per batch item the recurrence of scannd() (scan_nd.h).  x, y, dx
 * [batch, P, D]; delta, ddelta [batch, ndims, P, D]; A, dA [ndims, D, M];
 * B, C, dB, dC [batch, P, D, M] or, when bc_shared, [batch, P, M] (shared
 * by all channels; dB / dC are then channel sums); h [batch, P, D, M] is
 * written by the forward and read by the backward.  dA is summed over the
 * batch.  The backward has no reference implementation: it is the adjoint
 * of the forward recurrence.
 */
typedef struct {
    const float *x;
    const float *delta;
    const float *A;
    const float *B;
    const float *C;
    float *h;
    float *y;
    const float *dy;
    float *dx;
    float *ddelta;
    float *dA;
    float *dB;
    float *dC;
    long dims[8];
    long ndims;
    long batch;
    long D;
    long M;
    int bc_shared;
    int flags;     /* reserved, must be 0 */
} KmbScanND;

int kmb_scannd_fwd(const KmbScanND *args);
int kmb_scannd_bwd(const KmbScanND *args);

/*
 * bf16-I/O variants (no reference counterpart beyond the truncating host
 * conversions of include/kmamba_mixed_precision.h:106-112): x, delta, B,
 * C, y, dy, dx, ddelta, dB and dC point to bf16 (rounded to nearest even
 * on output); A, dA and h stay fp32; arithmetic is fp32.  Device memory
 * only.  Two axes with channel-shared B/C, M = 8 or 16 and D a multiple of
 * 8 (the config-4 layout) run the 2D wavefront kernels on bf16 tensors
 * directly (16-byte aligned inputs); other shapes convert the bf16
 * tensors to pooled fp32 scratch around the fp32 kernels.
 */
int kmb_scannd_fwd_bf16(const KmbScanND *args);
int kmb_scannd_bwd_bf16(const KmbScanND *args);

/* ------------------------------------------------------------------ */
/* bf16 GEMM on the tensor cores (block projections)                   */
/* ------------------------------------------------------------------ */
/*
 * C[m, n] = act(sum_k A(m, k) B(n, k) + bias[n]) + residual[m, n]
 * (+ the previous C when accumulate), fp32 accumulation (tcgen05 / TMEM).
 * Replaces the reference's cuBLAS SGEMM projections (cuda/mamba_block.cu:
 * 54-72) on the bf16-compute path.
 *
 * A and B are bf16 device memory, 16-byte aligned, lda / ldb multiples of
 * 8 elements.  K-major storage: A[m * lda + k], B[n * ldb + k];
 * a_mn_major / b_mn_major select the transposed storage A[k * lda + m],
 * B[k * ldb + n] (the input- and weight-gradient GEMMs of a linear layer).
 * C is fp32 (c_bf16 = 0) or bf16 rounded to nearest even, row stride ldc;
 * bias [N] and residual [M, ldr] are fp32 and optional.  act: 0 identity,
 * 1 SiLU.  Runs on the library stream; synchronous when kmb_set_sync(1).
 */
typedef struct {
    const void *A;
    const void *B;
    void *C;
    const float *bias;
    const float *residual;
    long M;
    long N;
    long K;
    long lda;
    long ldb;
    long ldc;
    long ldr;
    int a_mn_major;
    int b_mn_major;
    int c_bf16;
    int act;
    int accumulate;
    int pad_;
} KmbGemm;

int kmb_gemm_bf16(const KmbGemm *args);
/* KMB_ETIMEOUT when a GEMM launch's bounded pipeline wait gave up since
 * the last check (synchronous calls check it themselves). */
int kmb_gemm_check_error(void);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_B200_H */
