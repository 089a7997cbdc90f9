/*
 * bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by
 * TMA, with a fused epilogue.  Used by the projections of the Mamba block
 * (the reference runs them as cuBLAS SGEMM: cuda/mamba_block.cu:54-72,
 * call sites :404-436 and :781-833).
 *
 *   C[m, n] = act( sum_k A(m, k) B(n, k) + bias[n] ) + residual[m, n]  (+ C)
 *
 * A is [M, K] and B is [N, K], bf16.  Each operand is stored either
 * K-major (row-major with K contiguous: A[m * lda + k]) or MN-major (the
 * transposed storage: A[k * lda + m]), so the three GEMMs of a linear
 * layer -- forward, input gradient, weight gradient -- all run without a
 * transpose copy.  Accumulation is fp32 in tensor memory; C is fp32 or
 * bf16 (round to nearest even).
 *
 * CTA tile BM x BN x BK = 128 x BN x 64, STAGES shared-memory stages.
 * Split-K: when the M x N tiles do not fill the GPU and K is long (the
 * weight gradients: M x N = d x d, K = tokens), blockIdx.z takes a range of
 * the k-blocks; every split adds its fp32 tile to C with vector atomics
 * (split 0 also adds bias and residual; C is zeroed first unless the call
 * accumulates).  Only fp32 C without activation splits.
 * Warp roles inside a CTA of 128 threads:
 *   warp 0, one elected lane: TMA producer (two 2D tensor-map loads per
 *                             stage, 128-byte swizzle, no multicast);
 *   warp 1, one elected lane: MMA issuer (4 tcgen05.mma of K = 16 per
 *                             stage; tcgen05.commit frees the stage);
 *   warps 0-3:                epilogue, after the last commit: warp w
 *                             reads accumulator rows 32w..32w+31 from TMEM
 *                             (tcgen05.ld 32x32b) and writes C.
 * Every wait on an mbarrier is bounded (about 2^31 clock cycles); on
 * expiry the thread sets the CTA's abort flag and the launch's device
 * error word and leaves its loop, so the CTA still reaches the TMEM
 * release and exits.
 *
 * Tensor maps cover this GPU's own memory only (the caller's A and B).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <cuda.h>
#include <cuda_bf16.h>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;        /* bf16: 128 bytes, one swizzle row */
constexpr int kThreads = 128;
constexpr unsigned long long kWaitCycles = 1ull << 31;

__device__ int g_gemm_error; /* set by a launch whose wait expired */

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

/* Waits for the phase of the given parity; false (and the abort flag set)
 * when the wait gives up or another role already aborted. */
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
    const unsigned long long t0 = clock64();
    while (!mbar_test(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort = 1;
            atomicExch(&g_gemm_error, 1);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

/*
 * Shared-memory matrix descriptor of tcgen05.mma for a 128-byte swizzled
 * tile (start address >> 4 in bits 0-13, leading byte offset >> 4 in
 * 16-29, stride byte offset >> 4 in 32-45, descriptor version 1 in 46-47,
 * swizzle mode 2 = 128B in 61-63).
 *   K-major tile (rows of 64 K values, 128 B each): rows in groups of 8
 *     1024 B apart (stride offset); the leading offset is unused (1).
 *   MN-major tile (rows of 64 M or N values, one row per K): groups of 8
 *     K-rows 1024 B apart (stride offset); 64-wide M/N blocks `lbo` bytes
 *     apart (leading offset).
 */
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

/* tcgen05 instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 =
 * 1), bf16 A and B (bits 7-9, 10-12 = 1), A / B major (bits 15, 16: 0 =
 * K-major, 1 = MN-major), N >> 3 (bits 17-22), M >> 4 (bits 24-28). */
template <int BN, bool AMN, bool BMN>
__host__ __device__ constexpr uint32_t instr_desc() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((AMN ? 1u : 0u) << 15) | ((BMN ? 1u : 0u) << 16) |
           ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

struct GemmDev {
    void *C;
    const float *bias;
    const float *residual;
    long M, N, K, ldc, ldr;
    int c_bf16, act, accumulate;
    int kb_per_split; /* k-blocks of one split (gridDim.z splits) */
};

__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

/*
 * Epilogue of one tile for the calling warp: accumulator rows 32q..32q+31
 * (q = the warp's TMEM lane quarter) at TMEM column `col0`, written to C
 * rows m0 + 32q + lane, columns n0.. (bias, activation, residual; `split`:
 * fp32 atomics of a split-K share).  All 32 lanes must call it.
 */
template <int BN>
__device__ __forceinline__ void epilogue_rows(const GemmDev &p, uint32_t tmem, uint32_t col0,
                                              int q, int lane, long m0, long n0, bool ok,
                                              bool lead, bool split) {
    const long row = m0 + q * 32 + lane;
    const bool row_ok = ok && row < p.M;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + col0 + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, "
            "%10, %11, %12, %13, %14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
              "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
              "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (!row_ok) continue;
        const long n = n0 + c0;
        if (n >= p.N) continue;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            float t = __uint_as_float(r[j]);
            if (lead && p.bias && n + j < p.N) t += p.bias[n + j];
            if (p.act == 1) t = silu(t);
            if (lead && p.residual && n + j < p.N) t += p.residual[row * p.ldr + n + j];
            v[j] = t;
        }
        const bool full16 = n + 16 <= p.N;
        if (split) { /* fp32 C: this split's share, added atomically */
            float *c = reinterpret_cast<float *>(p.C) + row * p.ldc + n;
            if (full16 && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    atomicAdd(reinterpret_cast<float4 *>(c) + j,
                              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
            } else {
                for (int j = 0; j < 16 && n + j < p.N; ++j) atomicAdd(c + j, v[j]);
            }
            continue;
        }
        if (p.c_bf16) {
            __nv_bfloat16 *c = reinterpret_cast<__nv_bfloat16 *>(p.C) + row * p.ldc + n;
            if (full16 && !p.accumulate && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
                uint32_t w[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                    w[j] = *reinterpret_cast<const uint32_t *>(&h2);
                }
                reinterpret_cast<uint4 *>(c)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                reinterpret_cast<uint4 *>(c)[1] = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
                for (int j = 0; j < 16 && n + j < p.N; ++j) {
                    float t = v[j];
                    if (p.accumulate) t += __bfloat162float(c[j]);
                    c[j] = __float2bfloat16_rn(t);
                }
            }
        } else {
            float *c = reinterpret_cast<float *>(p.C) + row * p.ldc + n;
            if (full16 && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float4 t = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    if (p.accumulate) {
                        const float4 o = reinterpret_cast<const float4 *>(c)[j];
                        t.x += o.x; t.y += o.y; t.z += o.z; t.w += o.w;
                    }
                    reinterpret_cast<float4 *>(c)[j] = t;
                }
            } else {
                for (int j = 0; j < 16 && n + j < p.N; ++j) c[j] = p.accumulate ? c[j] + v[j] : v[j];
            }
        }
    }
}

template <int BN, int STAGES, bool AMN, bool BMN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
              GemmDev p) {
    constexpr int A_BYTES = kBM * kBK * 2;
    constexpr int B_BYTES = BN * kBK * 2;
    constexpr uint32_t TMEM_COLS = BN; /* fp32 accumulator: one column per n */
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    /* 1024-byte alignment of every tile (the swizzle pattern repeats
     * every 8 rows of 128 B) */
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(sB + STAGES * B_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
    const int nk_all = (int)((p.K + kBK - 1) / kBK);
    const int kb0 = (int)blockIdx.z * p.kb_per_split; /* this split's first k-block */
    const int nk = min(nk_all - kb0, p.kb_per_split);
    const bool split = gridDim.z > 1;
    const bool lead = blockIdx.z == 0; /* adds bias and residual */

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapA)));
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapB)));
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    int issued = 0; /* stages the producer has loaded */
    if (warp == 0 && lane == 0) {
        /* TMA producer */
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
            if (!mbar_wait(&empty[s], ph ^ 1u, abort)) break;
            issued = kb + 1;
            mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
            const int k0 = (kb0 + kb) * kBK;
            if (AMN) {
                tma_load_2d(sA + s * A_BYTES, &mapA, m0, k0, &full[s]);
                tma_load_2d(sA + s * A_BYTES + kBK * 128, &mapA, m0 + 64, k0, &full[s]);
            } else {
                tma_load_2d(sA + s * A_BYTES, &mapA, k0, m0, &full[s]);
            }
            if (BMN) {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j)
                    tma_load_2d(sB + s * B_BYTES + j * kBK * 128, &mapB, n0 + 64 * j, k0, &full[s]);
            } else {
                tma_load_2d(sB + s * B_BYTES, &mapB, k0, n0, &full[s]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        /* MMA issuer */
        constexpr uint32_t idesc = instr_desc<BN, AMN, BMN>();
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
            if (!mbar_wait(&full[s], ph, abort)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t a_addr = smem_u32(sA + s * A_BYTES);
            const uint32_t b_addr = smem_u32(sB + s * B_BYTES);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
                /* K step of 16: 32 bytes along a K-major row; 16 rows
                 * (2 swizzle groups of 1024 B) of an MN-major tile */
                const uint64_t da = AMN ? smem_desc(a_addr + k * 2048, kBK * 128)
                                        : smem_desc(a_addr + k * 32, 16);
                const uint64_t db = BMN ? smem_desc(b_addr + k * 2048, kBK * 128)
                                        : smem_desc(b_addr + k * 32, 16);
                const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(idesc), "r"(accum));
            }
            /* the stage is free once these MMAs have read it */
            asm volatile(
                "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                    smem_u32(&empty[s]))
                : "memory");
        }
        asm volatile(
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                smem_u32(acc_full))
            : "memory");
    }
    __syncwarp();

    /* epilogue: all four warps */
    const bool ok = nk > 0 && mbar_wait(acc_full, 0, abort);
    asm volatile("tcgen05.fence::after_thread_sync;");
    epilogue_rows<BN>(p, tmem, 0, warp, lane, m0, n0, ok, lead, split);

    if (warp == 0 && lane == 0 && *abort) {
        /* after an abort, let the copies still in flight land before the
         * CTA's shared memory goes away (each wait bounded again) */
        for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; ++kb) {
            const unsigned long long t0 = clock64();
            while (!mbar_test(&full[kb % STAGES], (uint32_t)(kb / STAGES) & 1u) &&
                   clock64() - t0 < kWaitCycles) {
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS));
    }
}

/* Row stride (floats) of an epilogue warp's staging tile [32 rows][64
 * columns]: 4 floats of padding put the 16-byte row segments of 8
 * consecutive lanes in disjoint banks. */
constexpr int kStgLd = 64 + 4;
constexpr int kStgBytes = 32 * kStgLd * 4;

/* Loads 4 consecutive floats of a row (16-byte aligned, or element-wise
 * when `vec` is false, up to `cnt` of them). */
__device__ __forceinline__ float4 load4(const float *src, bool vec, int cnt) {
    if (vec) return *reinterpret_cast<const float4 *>(src);
    float t[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < cnt && j < 4; ++j) t[j] = src[j];
    return make_float4(t[0], t[1], t[2], t[3]);
}

/*
 * Epilogue of one tile for the calling warp, staged through shared memory
 * so that C is written in whole row segments: for each group of 64
 * columns, the warp reads its 32 accumulator rows (TMEM lane quarter q)
 * with tcgen05.ld, applies bias and activation, and stores them to its
 * padded [32][64] staging tile (one row per lane); it then reads the tile
 * back row-wise (16 lanes x 16 B per fp32 row, 8 lanes x 16 B per bf16
 * row), adds the residual and, when accumulating, the old C, and writes
 * contiguous 256-byte (fp32) or 128-byte (bf16) row segments.
 */
template <int BN>
__device__ __forceinline__ void epilogue_staged(const GemmDev &p, uint32_t tmem, uint32_t col0,
                                                int q, int lane, long m0, long n0, float *stg,
                                                int cg0, int cg_step) {
#pragma unroll 1
    for (int cg = cg0; cg < BN; cg += cg_step) {
        const long nb = n0 + cg; /* first column of the group */
        /* the group's 64 accumulator columns in four loads, one wait */
        uint32_t r[64];
#pragma unroll
        for (int c16 = 0; c16 < 64; c16 += 16) {
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + col0 + (uint32_t)(cg + c16);
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, "
                "%10, %11, %12, %13, %14, %15}, [%16];"
                : "=r"(r[c16 + 0]), "=r"(r[c16 + 1]), "=r"(r[c16 + 2]), "=r"(r[c16 + 3]),
                  "=r"(r[c16 + 4]), "=r"(r[c16 + 5]), "=r"(r[c16 + 6]), "=r"(r[c16 + 7]),
                  "=r"(r[c16 + 8]), "=r"(r[c16 + 9]), "=r"(r[c16 + 10]), "=r"(r[c16 + 11]),
                  "=r"(r[c16 + 12]), "=r"(r[c16 + 13]), "=r"(r[c16 + 14]), "=r"(r[c16 + 15])
                : "r"(taddr));
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (!p.bias && p.act == 0) { /* the plain product: stored as loaded */
#pragma unroll
            for (int c4 = 0; c4 < 64; c4 += 4)
                *reinterpret_cast<uint4 *>(stg + lane * kStgLd + c4) =
                    make_uint4(r[c4], r[c4 + 1], r[c4 + 2], r[c4 + 3]);
        } else {
#pragma unroll
            for (int c4 = 0; c4 < 64; c4 += 4) {
                float v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float t = __uint_as_float(r[c4 + j]);
                    const long n = nb + c4 + j;
                    if (p.bias && n < p.N) t += p.bias[n];
                    if (p.act == 1) t = silu(t);
                    v[j] = t;
                }
                *reinterpret_cast<float4 *>(stg + lane * kStgLd + c4) =
                    make_float4(v[0], v[1], v[2], v[3]);
            }
        }
        __syncwarp();
        if (p.c_bf16) {
            const int rsub = lane >> 3, c8 = (lane & 7) * 8;
#pragma unroll 1
            for (int r0 = 0; r0 < 32; r0 += 4) {
                const int rr = r0 + rsub;
                const long row = m0 + q * 32 + rr, col = nb + c8;
                if (row >= p.M || col >= p.N) continue;
                const int cnt = (int)min((long)8, p.N - col);
                /* lanes 4-7 of each row read their second half first, so
                 * the 8 lanes of a row touch 8 distinct bank quads */
                const bool sw = (lane & 4) != 0;
                const float4 a0 = *reinterpret_cast<const float4 *>(stg + rr * kStgLd + c8 + (sw ? 4 : 0));
                const float4 b0 = *reinterpret_cast<const float4 *>(stg + rr * kStgLd + c8 + (sw ? 0 : 4));
                const float4 a = sw ? b0 : a0, b = sw ? a0 : b0;
                float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                if (p.residual) {
                    const float *rs = p.residual + row * p.ldr + col;
                    const bool rv = cnt == 8 && ((reinterpret_cast<uintptr_t>(rs) & 15) == 0);
                    const float4 x0 = load4(rs, rv, cnt), x1 = load4(rs + 4, rv, cnt - 4);
                    v[0] += x0.x; v[1] += x0.y; v[2] += x0.z; v[3] += x0.w;
                    v[4] += x1.x; v[5] += x1.y; v[6] += x1.z; v[7] += x1.w;
                }
                __nv_bfloat16 *c = reinterpret_cast<__nv_bfloat16 *>(p.C) + row * p.ldc + col;
                if (cnt == 8 && !p.accumulate && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
                    uint32_t w[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                        w[j] = *reinterpret_cast<const uint32_t *>(&h2);
                    }
                    *reinterpret_cast<uint4 *>(c) = make_uint4(w[0], w[1], w[2], w[3]);
                } else {
                    for (int j = 0; j < cnt; ++j) {
                        float t = v[j];
                        if (p.accumulate) t += __bfloat162float(c[j]);
                        c[j] = __float2bfloat16_rn(t);
                    }
                }
            }
        } else {
            const int rsub = lane >> 4, c4 = (lane & 15) * 4;
#pragma unroll 1
            for (int r0 = 0; r0 < 32; r0 += 2) {
                const int rr = r0 + rsub;
                const long row = m0 + q * 32 + rr, col = nb + c4;
                if (row >= p.M || col >= p.N) continue;
                const int cnt = (int)min((long)4, p.N - col);
                float4 t = *reinterpret_cast<const float4 *>(stg + rr * kStgLd + c4);
                if (p.residual) {
                    const float *rs = p.residual + row * p.ldr + col;
                    const float4 x = load4(rs, cnt == 4 && ((reinterpret_cast<uintptr_t>(rs) & 15) == 0), cnt);
                    t.x += x.x; t.y += x.y; t.z += x.z; t.w += x.w;
                }
                float *c = reinterpret_cast<float *>(p.C) + row * p.ldc + col;
                if (cnt == 4 && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
                    if (p.accumulate) {
                        const float4 o = *reinterpret_cast<const float4 *>(c);
                        t.x += o.x; t.y += o.y; t.z += o.z; t.w += o.w;
                    }
                    *reinterpret_cast<float4 *>(c) = t;
                } else {
                    const float tv[4] = {t.x, t.y, t.z, t.w};
                    for (int j = 0; j < cnt; ++j) c[j] = p.accumulate ? c[j] + tv[j] : tv[j];
                }
            }
        }
        __syncwarp();
    }
}

/*
 * Persistent variant for grids of many tiles (no split-K): one CTA per SM
 * walks the tiles blockIdx.x, blockIdx.x + gridDim.x, ... (n tile fastest,
 * so concurrent CTAs share the A row block in L2) with two accumulators in
 * TMEM (2 x BN columns), so that the epilogue of tile i overlaps the MMAs
 * of tile i + 1 and the TMA ring runs across tile boundaries.
 * Warps (192 threads):
 *   warp 0, one lane: TMA producer over every k-block of every tile;
 *   warp 1, one lane: MMA issuer; tile i accumulates into buffer i & 1
 *                     once the epilogue has drained it (acc_empty), and
 *                     commits acc_full[i & 1] after its last k-block;
 *   warps 2-9:        epilogue; warp w reads TMEM lane quarter w % 4 (rows
 *                     32 (w % 4) ..) of the finished buffer, warps 2-5 the
 *                     even and warps 6-9 the odd 64-column groups, writes
 *                     C in row segments through its shared staging tile
 *                     (epilogue_staged), and arrives on acc_empty (one
 *                     arrive per warp).
 * Without the epilogue the ring alone reaches 86 % of the measured bf16
 * peak at K = 1024; with one warp per lane quarter the epilogue of a
 * 128 x 256 bf16 tile outlasted the next tile's MMAs, hence two.
 * The staging tiles take 68 KB of shared memory, so the ring has 3 stages
 * at BN = 256 and 4 at BN = 128.
 * Every wait is bounded as in k_gemm_tc.
 */
constexpr int kPThreads = 320;
constexpr int kEpiWarps = 8;

template <int BN, int STAGES, bool AMN, bool BMN>
__global__ void __launch_bounds__(kPThreads, 1)
    k_gemm_tc_persist(const __grid_constant__ CUtensorMap mapA,
                      const __grid_constant__ CUtensorMap mapB, GemmDev p, int tiles_n,
                      int tiles) {
    constexpr int A_BYTES = kBM * kBK * 2;
    constexpr int B_BYTES = BN * kBK * 2;
    constexpr uint32_t TMEM_COLS = 2 * BN; /* two fp32 accumulators */
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    float *stg_all = reinterpret_cast<float *>(sB + STAGES * B_BYTES); /* [8][32][kStgLd] */
    uint64_t *full = reinterpret_cast<uint64_t *>(stg_all + kEpiWarps * 32 * kStgLd);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;    /* [2] */
    uint64_t *acc_empty = acc_full + 2;     /* [2] */
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = (int)((p.K + kBK - 1) / kBK);
    const int my_tiles = blockIdx.x < (unsigned)tiles
                             ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpiWarps);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapA)));
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapB)));
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    long issued = 0; /* k-blocks the producer has loaded, over all tiles */
    if (warp == 0 && lane == 0) {
        /* TMA producer */
        long g = 0;
        for (int i = 0; i < my_tiles && !*abort; ++i) {
            const int t = (int)blockIdx.x + i * (int)gridDim.x;
            const int n0 = (t % tiles_n) * BN, m0 = (t / tiles_n) * kBM;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = (int)(g % STAGES);
                const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort)) break;
                issued = g + 1;
                mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
                const int k0 = kb * kBK;
                if (AMN) {
                    tma_load_2d(sA + s * A_BYTES, &mapA, m0, k0, &full[s]);
                    tma_load_2d(sA + s * A_BYTES + kBK * 128, &mapA, m0 + 64, k0, &full[s]);
                } else {
                    tma_load_2d(sA + s * A_BYTES, &mapA, k0, m0, &full[s]);
                }
                if (BMN) {
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                        tma_load_2d(sB + s * B_BYTES + j * kBK * 128, &mapB, n0 + 64 * j, k0,
                                    &full[s]);
                } else {
                    tma_load_2d(sB + s * B_BYTES, &mapB, k0, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        /* MMA issuer */
        constexpr uint32_t idesc = instr_desc<BN, AMN, BMN>();
        long g = 0;
        for (int i = 0; i < my_tiles; ++i) {
            const int buf = i & 1;
            const uint32_t use = (uint32_t)(i >> 1) & 1u;
            /* the epilogue has drained this buffer (tile i - 2) */
            if (!mbar_wait(&acc_empty[buf], use ^ 1u, abort)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t acc = tmem + (uint32_t)(buf * BN);
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = (int)(g % STAGES);
                const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
                if (!mbar_wait(&full[s], ph, abort)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t a_addr = smem_u32(sA + s * A_BYTES);
                const uint32_t b_addr = smem_u32(sB + s * B_BYTES);
#pragma unroll
                for (int k = 0; k < kBK / 16; ++k) {
                    const uint64_t da = AMN ? smem_desc(a_addr + k * 2048, kBK * 128)
                                            : smem_desc(a_addr + k * 32, 16);
                    const uint64_t db = BMN ? smem_desc(b_addr + k * 2048, kBK * 128)
                                            : smem_desc(b_addr + k * 32, 16);
                    const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(acc),
                        "l"(da), "l"(db), "r"(idesc), "r"(accum));
                }
                asm volatile(
                    "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
                    "[%0];" ::"r"(smem_u32(&empty[s]))
                    : "memory");
            }
            if (!ok) break;
            asm volatile(
                "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                    smem_u32(&acc_full[buf]))
                : "memory");
        }
    } else if (warp >= 2) {
        /* epilogue warps */
        const int q = warp & 3;
        for (int i = 0; i < my_tiles; ++i) {
            const int buf = i & 1;
            const uint32_t ph = (uint32_t)(i >> 1) & 1u;
            const int t = (int)blockIdx.x + i * (int)gridDim.x;
            const long n0 = (long)(t % tiles_n) * BN, m0 = (long)(t / tiles_n) * kBM;
            const bool ok = mbar_wait(&acc_full[buf], ph, abort);
            asm volatile("tcgen05.fence::after_thread_sync;");
            if (!ok) break;
            epilogue_staged<BN>(p, tmem, (uint32_t)(buf * BN), q, lane, m0, n0,
                                stg_all + (warp - 2) * 32 * kStgLd, ((warp - 2) >> 2) * 64, 128);
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                                 smem_u32(&acc_empty[buf]))
                             : "memory");
        }
    }
    __syncwarp();

    if (warp == 0 && lane == 0 && *abort) {
        for (long g = issued > STAGES ? issued - STAGES : 0; g < issued; ++g) {
            const unsigned long long t0 = clock64();
            while (!mbar_test(&full[g % STAGES], (uint32_t)(g / STAGES) & 1u) &&
                   clock64() - t0 < kWaitCycles) {
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS));
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            (void)cudaGetLastError();
    }
    return fn;
}

/* 2D bf16 tensor map over a [rows, cols] row-major operand (cols
 * contiguous, ld elements between rows), box = box_cols x box_rows with a
 * 128-byte swizzle; reads past the edges return zeros. */
int make_map(CUtensorMap *m, const void *base, long rows, long cols, long ld, int box_cols,
             int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return kmb_fail(KMB_ECUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return kmb_fail(KMB_EINVAL, "gemm: tensor map rejected (CUresult %d)", (int)r);
    return KMB_OK;
}

/* Splits of K: enough CTAs for one wave of one per SM when the tiles alone
 * leave SMs idle, at least 8 k-blocks (512 of K) a split; only fp32 C
 * without activation (the splits are added atomically).  KMB_GEMM_SPLITK=0
 * disables it. */
int split_count(long tiles, long nk, const KmbGemm *g) {
    static int enabled = -1;
    if (enabled < 0) {
        const char *e = getenv("KMB_GEMM_SPLITK");
        enabled = !(e && e[0] == '0' && e[1] == 0);
    }
    if (!enabled || g->c_bf16 || g->act != 0 || tiles >= 148) return 1;
    long sp = 148 / tiles;
    if (sp > nk / 8) sp = nk / 8;
    return sp > 1 ? (int)sp : 1;
}

/* SMs of the current device (the persistent grid: one CTA per SM). */
int kmb_sm_count() {
    static int cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        (void)cudaGetLastError();
        return 148;
    }
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            (void)cudaGetLastError();
            n = 148;
        }
        cached[dev] = n;
    }
    return cached[dev];
}

/* The persistent kernel serves every call without split-K unless
 * KMB_GEMM_PERSIST=0 (one CTA per tile, k_gemm_tc). */
bool persist_enabled() {
    static int enabled = -1;
    if (enabled < 0) {
        const char *e = getenv("KMB_GEMM_PERSIST");
        enabled = !(e && e[0] == '0' && e[1] == 0);
    }
    return enabled != 0;
}

template <int BN, int STAGES, bool AMN, bool BMN>
int launch(const KmbGemm *g, cudaStream_t s) {
    CUtensorMap ma, mb;
    /* K-major operand: rows = M (or N), cols = K, box 64 x rows-of-tile;
     * MN-major operand: rows = K, cols = M (or N), box 64 x 64 (K rows) */
    int rc = AMN ? make_map(&ma, g->A, g->K, g->M, g->lda, 64, kBK)
                 : make_map(&ma, g->A, g->M, g->K, g->lda, kBK, kBM);
    if (rc) return rc;
    rc = BMN ? make_map(&mb, g->B, g->K, g->N, g->ldb, 64, kBK)
             : make_map(&mb, g->B, g->N, g->K, g->ldb, kBK, BN);
    if (rc) return rc;
    GemmDev p;
    p.C = g->C;
    p.bias = g->bias;
    p.residual = g->residual;
    p.M = g->M; p.N = g->N; p.K = g->K; p.ldc = g->ldc; p.ldr = g->ldr;
    p.c_bf16 = g->c_bf16; p.act = g->act; p.accumulate = g->accumulate;
    const size_t smem = 1024 + (size_t)STAGES * (kBM + BN) * kBK * 2 + (2 * STAGES + 1) * 8 + 16;
    auto kern = k_gemm_tc<BN, STAGES, AMN, BMN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm: smem attribute");
    const long tiles = ((g->N + BN - 1) / BN) * ((g->M + kBM - 1) / kBM);
    const long nk = (g->K + kBK - 1) / kBK;
    const int splits = split_count(tiles, nk, g);
    p.kb_per_split = (int)((nk + splits - 1) / splits);
    const unsigned gz = (unsigned)((nk + p.kb_per_split - 1) / p.kb_per_split); /* no empty split */
    if (gz == 1 && persist_enabled()) {
        constexpr int PST = BN == 256 ? 3 : 4;
        const int tiles_n = (int)((g->N + BN - 1) / BN);
        const int ntiles = (int)tiles;
        const size_t psmem = 1024 + (size_t)PST * (kBM + BN) * kBK * 2 + kEpiWarps * (size_t)kStgBytes +
                             (2 * PST + 4) * 8 + 16;
        auto pk = k_gemm_tc_persist<BN, PST, AMN, BMN>;
        e = cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm: smem attribute");
        const int grid_p = ntiles < kmb_sm_count() ? ntiles : kmb_sm_count();
        pk<<<(unsigned)grid_p, kPThreads, psmem, s>>>(ma, mb, p, tiles_n, ntiles);
        e = cudaGetLastError();
        return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "gemm: launch");
    }
    if (gz > 1 && !g->accumulate) {
        e = cudaMemset2DAsync(g->C, (size_t)g->ldc * 4, 0, (size_t)g->N * 4, (size_t)g->M, s);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm: split-K zero fill");
    }
    dim3 grid((unsigned)((g->N + BN - 1) / BN), (unsigned)((g->M + kBM - 1) / kBM), gz);
    kern<<<grid, kThreads, smem, s>>>(ma, mb, p);
    e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "gemm: launch");
}

template <int BN, int STAGES>
int dispatch(const KmbGemm *g, cudaStream_t s) {
    const bool amn = g->a_mn_major, bmn = g->b_mn_major;
    if (!amn && !bmn) return launch<BN, STAGES, false, false>(g, s);
    if (!amn && bmn) return launch<BN, STAGES, false, true>(g, s);
    if (amn && !bmn) return launch<BN, STAGES, true, false>(g, s);
    return launch<BN, STAGES, true, true>(g, s);
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

} // namespace

extern "C" int kmb_launch_gemm_bf16(const KmbGemm *g, cudaStream_t s) {
    if (g->N > 128) return dispatch<256, 4>(g, s);
    return dispatch<128, 6>(g, s);
}

extern "C" int kmb_gemm_bf16(const KmbGemm *g) {
    if (!g) return kmb_fail(KMB_EINVAL, "gemm: NULL arguments");
    if (g->M <= 0 || g->N <= 0 || g->K <= 0)
        return kmb_fail(KMB_EINVAL, "gemm: M, N and K must be positive");
    if (!g->A || !g->B || !g->C) return kmb_fail(KMB_EINVAL, "gemm: A, B and C are required");
    if (g->act < 0 || g->act > 1) return kmb_fail(KMB_EINVAL, "gemm: unknown activation %d", g->act);
    if (!aligned16(g->A) || !aligned16(g->B) || g->lda % 8 || g->ldb % 8)
        return kmb_fail(KMB_EUNSUPPORTED,
                        "gemm: A and B must be 16-byte aligned with lda, ldb multiples of 8");
    const long a_inner = g->a_mn_major ? g->M : g->K, b_inner = g->b_mn_major ? g->N : g->K;
    if (g->lda < a_inner || g->ldb < b_inner || g->ldc < g->N || (g->residual && g->ldr < g->N))
        return kmb_fail(KMB_EINVAL, "gemm: leading dimension smaller than the row");
    if (g->M >= (1L << 31) || g->N >= (1L << 31) || g->K >= (1L << 31))
        return kmb_fail(KMB_EUNSUPPORTED, "gemm: dimensions must be below 2^31");
    const void *ptrs[] = {g->A, g->B, g->C, g->bias, g->residual};
    for (const void *q : ptrs)
        if (q && !kmb_is_device_ptr(q))
            return kmb_fail(KMB_EINVAL, "gemm: operands must be device memory");
    kmb_clear_error();
    const cudaStream_t s = kmb_stream();
    int rc = kmb_launch_gemm_bf16(g, s);
    if (rc) return rc;
    if (kmb_sync_enabled()) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm: stream synchronize");
        return kmb_gemm_check_error();
    }
    return KMB_OK;
}

/* KMB_ETIMEOUT (and the flag cleared) when a launch's bounded wait gave up
 * since the last check. */
extern "C" int kmb_gemm_check_error(void) {
    int flag = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&flag, g_gemm_error, sizeof flag);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm: error word");
    if (flag) {
        const int zero = 0;
        (void)cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof zero);
        return kmb_fail(KMB_ETIMEOUT, "gemm: a pipeline wait expired (device error word set)");
    }
    return KMB_OK;
}
