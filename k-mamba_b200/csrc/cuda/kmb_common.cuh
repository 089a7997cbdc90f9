/*
 * Device helpers shared by the sm_100a kernels of this library.
 */
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

/* log2(e): exp(x) = 2^(x * log2(e)).  The scans pre-scale A by this
 * constant once per (channel, state) so that every discretisation step is
 * one multiply plus one MUFU ex2. */
#define KMB_LOG2E 1.4426950408889634f

/* 2^x on the MUFU unit (PTX ex2.approx, subnormal results flushed to 0). */
__device__ __forceinline__ float kmb_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

/* Asynchronous global->shared copies (cp.async, sm_80+).  A source size
 * below the copy size zero-fills the remainder of the destination. */
__device__ __forceinline__ void kmb_cp_async4(void *smem, const void *gmem,
                                              bool valid) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s),
                 "l"(gmem), "r"(n));
}

__device__ __forceinline__ void kmb_cp_async16(void *smem, const void *gmem,
                                               int src_bytes) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s),
                 "l"(gmem), "r"(src_bytes));
}

__device__ __forceinline__ void kmb_cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::);
}

template <int N>
__device__ __forceinline__ void kmb_cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

/*
 * Cooperative copy of a rows x cols float tile into shared memory with row
 * stride s_ld (a multiple of 4).  Rows >= rows_valid and columns >=
 * cols_valid are zero-filled.  vec selects 16-byte copies; it requires
 * g 16-byte aligned and g_ld a multiple of 4 floats.
 */
template <int NT>
__device__ __forceinline__ void kmb_load_tile(float *s, int s_ld,
                                              const float *g, long g_ld,
                                              int rows, int cols,
                                              int rows_valid, int cols_valid,
                                              bool vec, int tid) {
    if (vec) {
        const int c4 = (cols + 3) >> 2;
        const int total = rows * c4;
        for (int i = tid; i < total; i += NT) {
            const int r = i / c4;
            const int c = (i - r * c4) << 2;
            int bytes = 0;
            if (r < rows_valid) {
                int left = cols_valid - c;
                bytes = left >= 4 ? 16 : (left > 0 ? left * 4 : 0);
            }
            const float *src = bytes ? g + (long)r * g_ld + c : g;
            kmb_cp_async16(s + r * s_ld + c, src, bytes);
        }
    } else {
        const int total = rows * cols;
        for (int i = tid; i < total; i += NT) {
            const int r = i / cols;
            const int c = i - r * cols;
            const bool ok = (r < rows_valid) && (c < cols_valid);
            const float *src = ok ? g + (long)r * g_ld + c : g;
            kmb_cp_async4(s + r * s_ld + c, src, ok);
        }
    }
}
