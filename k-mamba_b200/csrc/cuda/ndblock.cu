/*
 * Elementwise and reduction kernels of the Mamba-ND block (the model of
 * BASELINE config 5, csrc/host/ndmodel.c).  The block's heavy operators
 * run elsewhere: projections on the tensor cores (gemm_tc.cu), the causal
 * ConvND (convnd.cu), the ND scan (scannd.cu).  Everything here is one
 * pass over [T, d] activations (T = batch * points), fp32 arithmetic:
 *
 *   silu          c = v sigmoid(v)
 *   dt / B / C    delta_k[b, k, p, j] = ln 3 + softplus(q[t, k] + dt_bias[k, j]),
 *                 B[t, :] = q[t, 3:19], C[t, :] = q[t, 19:35]
 *   gate          g = bf16(y * silu(z))
 * and their backward: the gate and silu derivatives, and the dt reduction
 *   dq[t, k]        = sum_j ddelta_k[t, j] sigmoid(q[t, k] + dt_bias[k, j])
 *   d dt_bias[k, j] = sum_t ddelta_k[t, j] sigmoid(q[t, k] + dt_bias[k, j]).
 */
#include <stdint.h>

#include <cuda_bf16.h>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kState = 16;

__device__ __forceinline__ float sigm(float v) { return 1.f / (1.f + __expf(-v)); }
__device__ __forceinline__ float softplus(float v) { return v > 20.f ? v : log1pf(__expf(v)); }

unsigned grid_for(long n, int threads = 256) {
    long g = (n + threads - 1) / threads;
    if (g > 148L * 16) g = 148L * 16;
    return (unsigned)(g < 1 ? 1 : g);
}

/* one row per CTA iteration (no per-element division) */
__global__ void k_to_bf16(const float *src, long lds, __nv_bfloat16 *dst, long ldd, long rows,
                          long cols) {
    for (long r = blockIdx.x; r < rows; r += gridDim.x) {
        const float *s = src + r * lds;
        __nv_bfloat16 *d = dst + r * ldd;
        for (long c = threadIdx.x; c < cols; c += blockDim.x) d[c] = __float2bfloat16_rn(s[c]);
    }
}

/* contiguous, 16-byte aligned, n a multiple of 4: four values per thread */
__global__ void k_to_bf16_flat(const float4 *src, uint2 *dst, long n4) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (long)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        dst[i] = make_uint2(*reinterpret_cast<unsigned *>(&a), *reinterpret_cast<unsigned *>(&b));
    }
}

__global__ void k_silu(const float *v, float *c, __nv_bfloat16 *c16, long n) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const float x = v[e], y = x * sigm(x);
        c[e] = y;
        if (c16) c16[e] = __float2bfloat16_rn(y);
    }
}

/* dv = dc * silu'(v), silu'(v) = s (1 + v (1 - s)) */
__global__ void k_silu_bwd(const float *dc, const float *v, float *dv, long n) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const float x = v[e], s = sigm(x);
        dv[e] = dc[e] * s * (1.f + x * (1.f - s));
    }
}

__global__ void k_dt_bc(const float *q, long qld, const float *dtb, float *delta, float *B,
                        float *C, long batch, long P, long d) {
    for (long b = 0; b < batch; ++b) {
        for (long p = blockIdx.x; p < P; p += gridDim.x) {
            const long t = b * P + p;
            const float *qr = q + t * qld;
            const float q0 = qr[0], q1 = qr[1], q2 = qr[2];
            float *d0 = delta + ((b * 3 + 0) * P + p) * d;
            float *d1 = delta + ((b * 3 + 1) * P + p) * d;
            float *d2 = delta + ((b * 3 + 2) * P + p) * d;
            for (long j = threadIdx.x; j < d; j += blockDim.x) {
                d0[j] = 1.0986122886681098f + softplus(q0 + dtb[j]);
                d1[j] = 1.0986122886681098f + softplus(q1 + dtb[d + j]);
                d2[j] = 1.0986122886681098f + softplus(q2 + dtb[2 * d + j]);
            }
            if (threadIdx.x < kState) {
                B[t * kState + threadIdx.x] = qr[3 + threadIdx.x];
                C[t * kState + threadIdx.x] = qr[3 + kState + threadIdx.x];
            }
        }
    }
}

__global__ void k_gate(const float *y, const float *z, __nv_bfloat16 *g, long n) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const float zz = z[e];
        g[e] = __float2bfloat16_rn(y[e] * zz * sigm(zz));
    }
}

/* dy = dg silu(z); dz = dg y silu'(z) (bf16, the GEMM operand) */
__global__ void k_gate_bwd(const float *dg, const float *y, const float *z, float *dy,
                           __nv_bfloat16 *dz, long n) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const float zz = z[e], s = sigm(zz), gg = dg[e];
        dy[e] = gg * zz * s;
        dz[e] = __float2bfloat16_rn(gg * y[e] * s * (1.f + zz * (1.f - s)));
    }
}

/* dq[t, k] for k < 3 (one warp per token), dq[t, 3 + n] = dB, dq[t, 19 + n]
 * = dC, written as bf16 rows of dq_ld values (the tensor-core GEMM operand;
 * the columns from 35 to dq_ld are zero) */
__global__ void k_dt_bwd_rows(const float *ddelta, const float *q, long qld, const float *dtb,
                              const float *dB, const float *dC, __nv_bfloat16 *dq, long dq_ld,
                              long batch, long P, long d) {
    const int lane = threadIdx.x & 31;
    const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
    for (long b = 0; b < batch; ++b) {
        for (long p = warp; p < P; p += nwarps) {
            const long t = b * P + p;
            const float *qr = q + t * qld;
            __nv_bfloat16 *out = dq + t * dq_ld;
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const float *dd = ddelta + ((b * 3 + k) * P + p) * d;
                const float qk = qr[k];
                float acc = 0.f;
                for (long j = lane; j < d; j += 32)
                    acc = fmaf(dd[j], sigm(qk + dtb[k * d + j]), acc);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane == 0) out[k] = __float2bfloat16_rn(acc);
            }
            if (lane < kState) {
                out[3 + lane] = __float2bfloat16_rn(dB[t * kState + lane]);
                out[3 + kState + lane] = __float2bfloat16_rn(dC[t * kState + lane]);
            }
            for (long c = 3 + 2 * kState + lane; c < dq_ld; c += 32) out[c] = __float2bfloat16_rn(0.f);
        }
    }
}

/* d dt_bias[k, j] += sum over a chunk of tokens (atomics per chunk) */
__global__ void k_dt_bwd_cols(const float *ddelta, const float *q, long qld, const float *dtb,
                              float *ddtb, long batch, long P, long d, long rows_per_cta) {
    /* rows [p0, p1) of every batch item */
    const long p0 = (long)blockIdx.y * rows_per_cta;
    const long p1 = min(P, p0 + rows_per_cta);
    const int k = blockIdx.z;
    for (long j = (long)blockIdx.x * blockDim.x + threadIdx.x; j < d; j += (long)gridDim.x * blockDim.x) {
        const float bias = dtb[k * d + j];
        float acc = 0.f;
        for (long b = 0; b < batch; ++b) {
            const float *dd = ddelta + ((b * 3 + k) * P) * d + j;
            const float *qc = q + (b * P) * qld + k;
            for (long p = p0; p < p1; ++p) acc = fmaf(dd[p * d], sigm(qc[p * qld] + bias), acc);
        }
        atomicAdd(ddtb + k * d + j, acc);
    }
}

/* A = -1 - exp(A_log) (dA_inout == NULL), or dA_log = dA * (-exp(A_log))
 * in place */
__global__ void k_neg_exp(const float *A_log, float *A, float *dA_inout, long n) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const float ex = __expf(A_log[e]);
        if (dA_inout) dA_inout[e] *= -ex;
        else A[e] = -1.f - ex;
    }
}

__global__ void k_roll_targets(const unsigned *tok, unsigned *tgt, long batch, long P) {
    const long n = batch * P;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const long b = e / P, p = e - b * P;
        tgt[e] = tok[b * P + (p + 1 == P ? 0 : p + 1)];
    }
}

/* out[0] = mean of x (one CTA, double accumulation) */
__global__ void __launch_bounds__(1024) k_mean(const float *x, long n, float *out) {
    __shared__ double red[32];
    double acc = 0.0;
    for (long i = threadIdx.x; i < n; i += blockDim.x) acc += x[i];
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        out[0] = (float)(t / (double)n);
    }
}

} // namespace

extern "C" int kmb_nd_mean(const float *x, long n, float *out, cudaStream_t s) {
    k_mean<<<1, 1024, 0, s>>>(x, n, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "nd: mean");
}

#define KMB_ND_RET(what)                                                       \
    do {                                                                       \
        const cudaError_t e_ = cudaGetLastError();                             \
        return e_ == cudaSuccess ? KMB_OK : kmb_cuda_fail(e_, what);           \
    } while (0)

extern "C" int kmb_nd_to_bf16(const float *src, long lds, void *dst, long ldd, long rows,
                              long cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return KMB_OK;
    const long n = rows * cols;
    if (lds == cols && ldd == cols && n % 4 == 0 && ((uintptr_t)src & 15u) == 0 &&
        ((uintptr_t)dst & 7u) == 0) {
        k_to_bf16_flat<<<grid_for(n / 4), 256, 0, s>>>(reinterpret_cast<const float4 *>(src),
                                                       static_cast<uint2 *>(dst), n / 4);
    } else {
        const unsigned g = (unsigned)(rows < 148L * 16 ? rows : 148L * 16);
        k_to_bf16<<<g, 256, 0, s>>>(src, lds, static_cast<__nv_bfloat16 *>(dst), ldd, rows, cols);
    }
    KMB_ND_RET("nd: bf16 conversion");
}

extern "C" int kmb_nd_silu(const float *v, float *c, void *c16, const float *dc, float *dv,
                           long n, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    if (dc) k_silu_bwd<<<grid_for(n), 256, 0, s>>>(dc, v, dv, n);
    else k_silu<<<grid_for(n), 256, 0, s>>>(v, c, static_cast<__nv_bfloat16 *>(c16), n);
    KMB_ND_RET("nd: silu");
}

extern "C" int kmb_nd_dt_bc(const float *q, long qld, const float *dtb, float *delta, float *B,
                            float *C, long batch, long P, long d, cudaStream_t s) {
    k_dt_bc<<<(unsigned)(P < 148L * 16 ? P : 148L * 16), 256, 0, s>>>(q, qld, dtb, delta, B, C,
                                                                        batch, P, d);
    KMB_ND_RET("nd: dt / B / C");
}

extern "C" int kmb_nd_gate(const float *y, const float *z, void *g16, const float *dg, float *dy,
                           void *dz16, long n, cudaStream_t s) {
    if (dg) k_gate_bwd<<<grid_for(n), 256, 0, s>>>(dg, y, z, dy, static_cast<__nv_bfloat16 *>(dz16), n);
    else k_gate<<<grid_for(n), 256, 0, s>>>(y, z, static_cast<__nv_bfloat16 *>(g16), n);
    KMB_ND_RET("nd: gate");
}

extern "C" int kmb_nd_dt_bwd(const float *ddelta, const float *q, long qld, const float *dtb,
                             const float *dB, const float *dC, void *dq16, long dq_ld,
                             float *ddtb, int acc, long batch, long P, long d, cudaStream_t s) {
    k_dt_bwd_rows<<<grid_for(P * 32), 256, 0, s>>>(ddelta, q, qld, dtb, dB, dC,
                                                   static_cast<__nv_bfloat16 *>(dq16), dq_ld,
                                                   batch, P, d);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return kmb_cuda_fail(e, "nd: dt backward rows");
    if (!acc) e = cudaMemsetAsync(ddtb, 0, sizeof(float) * 3 * d, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "nd: dt bias memset");
    const long rows = 256;
    dim3 grid((unsigned)((d + 255) / 256), (unsigned)((P + rows - 1) / rows), 3);
    k_dt_bwd_cols<<<grid, 256, 0, s>>>(ddelta, q, qld, dtb, ddtb, batch, P, d, rows);
    KMB_ND_RET("nd: dt backward columns");
}

/* g (+)= dA * (-exp(A_log)): the A_log gradient of a scan's dA */
__global__ void k_dalog(const float *A_log, const float *dA, float *g, int acc, long n) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (long)gridDim.x * blockDim.x) {
        const float v = -dA[e] * __expf(A_log[e]);
        g[e] = acc ? g[e] + v : v;
    }
}

extern "C" int kmb_nd_dalog(const float *A_log, const float *dA, float *g, int acc, long n,
                            cudaStream_t s) {
    k_dalog<<<grid_for(n), 256, 0, s>>>(A_log, dA, g, acc, n);
    KMB_ND_RET("nd: A_log gradient");
}

extern "C" int kmb_nd_neg_exp(const float *A_log, float *A, float *dA_inout, long n,
                              cudaStream_t s) {
    k_neg_exp<<<grid_for(n), 256, 0, s>>>(A_log, A, dA_inout, n);
    KMB_ND_RET("nd: -exp(A_log)");
}

extern "C" int kmb_nd_roll_targets(const unsigned *tok, unsigned *tgt, long batch, long P,
                                   cudaStream_t s) {
    k_roll_targets<<<grid_for(batch * P), 256, 0, s>>>(tok, tgt, batch, P);
    KMB_ND_RET("nd: targets");
}
