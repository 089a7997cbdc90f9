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
#define KMB_LN2 0.6931471805599453f

/* 2^x on the MUFU unit (PTX ex2.approx, subnormal results flushed to 0). */
__device__ __forceinline__ float kmb_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

/*
 * Decay factor 2^w of the scans (w = dt * A * log2 e <= 0 in practice).
 *
 * A recurrence h_t = a_t h_{t-1} + ... with a_t close to 1 carries the
 * relative error of each a_t over ~1/|ln a_t| steps, so a per-step bias of
 * one ulp in a_t grows into a 1e-3 error on a weak-decay sequence.  Where
 * |w| < KMB_DECAY_POLY_MAX = 1/32 (memory longer than ~46 steps) 2^w is
 * therefore evaluated with a degree-3 polynomial fitted for minimax
 * relative error on [-1/32, 1/32] (iteratively reweighted least squares on
 * Chebyshev nodes: 1.1e-9 in real arithmetic, 0.55 ulp and a mean relative
 * error of 1e-9 in fp32 Horner form).  Elsewhere the memory is short and
 * MUFU ex2 (~2 ulp) is used.
 */
#define KMB_DECAY_POLY_MAX 0.03125f

__device__ __forceinline__ float kmb_decay_poly(float w) {
    float p = fmaf(0.05550280585885048f, w, 0.24023589491844177f);
    p = fmaf(p, w, 0.6931471824645996f);
    return fmaf(p, w, 1.0f);
}

/* Scalar decay: both evaluated and selected, so a warp never diverges. */
__device__ __forceinline__ float kmb_exp2_decay(float w) {
    const float m = kmb_ex2(w);
    const float p = kmb_decay_poly(w);
    return fabsf(w) < KMB_DECAY_POLY_MAX ? p : m;
}

/* Packed fp32 pairs (sm_100 FFMA2 / FMUL2 / FADD2): two single-precision
 * operations per instruction, each element rounded exactly as fmaf / * /
 * + round it, so pair code gives the scalar code's results bit for bit. */
__device__ __forceinline__ float2 kmb_f2(float x, float y) { return make_float2(x, y); }
__device__ __forceinline__ float2 kmb_f2s(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 kmb_fma2(float2 a, float2 b, float2 c) {
    return __ffma2_rn(a, b, c);
}
__device__ __forceinline__ float2 kmb_mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 kmb_add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

/* MUFU ex2 of both elements of a pair. */
__device__ __forceinline__ float2 kmb_ex2_2(float2 w) {
    return make_float2(kmb_ex2(w.x), kmb_ex2(w.y));
}

/* Given m = kmb_ex2_2(w), the pair kmb_exp2_decay would give: the
 * polynomial on FFMA2 pairs where |w| < KMB_DECAY_POLY_MAX, m elsewhere. */
__device__ __forceinline__ float2 kmb_decay_fix2(float2 w, float2 m) {
    float2 p = kmb_fma2(kmb_f2s(0.05550280585885048f), w, kmb_f2s(0.24023589491844177f));
    p = kmb_fma2(p, w, kmb_f2s(0.6931471824645996f));
    p = kmb_fma2(p, w, kmb_f2s(1.0f));
    return kmb_f2(fabsf(w.x) < KMB_DECAY_POLY_MAX ? p.x : m.x,
                  fabsf(w.y) < KMB_DECAY_POLY_MAX ? p.y : m.y);
}

/* kmb_exp2_decay of two values; each element equals kmb_exp2_decay. */
__device__ __forceinline__ float2 kmb_exp2_decay2(float2 w) {
    return kmb_decay_fix2(w, kmb_ex2_2(w));
}

/*
 * 2^w of both elements of a pair on the FMA pipe, without MUFU, so that a
 * kernel can move part of its exponentials off the 16-per-clock MUFU unit.
 *
 * Range reduction (exact, base 2 needs no split constant): t = w + 1.5 * 2^23
 * rounds w to the nearest integer n in t's low mantissa bits, n = t - 1.5 *
 * 2^23 and f = w - n in [-1/2, 1/2] are both exact.  2^f is a degree-6
 * polynomial with p(0) = 1 and p'(0) = ln 2 held fixed and the other
 * coefficients fitted for minimax relative error on [-1/2, 1/2]
 * (iteratively reweighted least squares on a dense grid): 3.0e-9 in real
 * arithmetic, 6.7e-8 maximum and 1.5e-10 mean relative error in fp32
 * Horner form, and a mean of -3e-11 on the weak-decay range |w| < 1/32,
 * so a long-memory recurrence accumulates no bias (MUFU ex2: ~1.4e-7 with
 * a negative mean).  2^n is then added to the exponent field: the low 9
 * bits of 1.5 * 2^23's pattern are zero, so (bits(t) << 23) is n << 23.
 *
 * Valid for |w| <= 125 (a normal result); callers check that bound and
 * redo the work with kmb_exp2_decay2 when it fails.  NaN inputs give a
 * finite or NaN pattern, so callers must also reject non-finite w.
 */
__device__ __forceinline__ float2 kmb_exp2_fma2(float2 w) {
    const float2 t = kmb_add2(w, kmb_f2s(12582912.0f));
    const float2 n = kmb_add2(t, kmb_f2s(-12582912.0f));
    const float2 f = kmb_fma2(n, kmb_f2s(-1.0f), w);
    float2 p = kmb_fma2(kmb_f2s(1.532424212200567e-4f), f, kmb_f2s(1.339093898423016e-3f));
    p = kmb_fma2(p, f, kmb_f2s(9.618517942726612e-3f));
    p = kmb_fma2(p, f, kmb_f2s(5.550359562039375e-2f));
    p = kmb_fma2(p, f, kmb_f2s(2.4022647738456726e-1f));
    p = kmb_fma2(p, f, kmb_f2s(6.931471824645996e-1f));
    p = kmb_fma2(p, f, kmb_f2s(1.0f));
    return kmb_f2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                  __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

/* Largest |w| for which kmb_exp2_fma2 is used (its valid range, with a
 * margin for the rounding of w = dt * A log2 e). */
#define KMB_EXP2_FMA_MAX 125.0f

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

/* The same with the destination as a shared-window address (the result
 * of __cvta_generic_to_shared), for loops that keep a base address. */
__device__ __forceinline__ void kmb_cp_async16_s(unsigned s, const void *gmem, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(src_bytes));
}

__device__ __forceinline__ void kmb_cp_async4_s(unsigned s, const void *gmem, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(src_bytes));
}

__device__ __forceinline__ void kmb_cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::);
}

template <int N>
__device__ __forceinline__ void kmb_cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

/*
 * kmb_load_tile with a compile-time tile shape (ROWS x COLS): the element
 * -> (row, column) split is a constant division, and the loop has a fixed
 * trip count.
 */
template <int NT, int ROWS, int COLS>
__device__ __forceinline__ void kmb_load_tile_c(float *s, int s_ld, const float *g, long g_ld,
                                                int rows_valid, int cols_valid, bool vec,
                                                int tid) {
    if (vec) {
        constexpr int C4 = (COLS + 3) >> 2;
        constexpr int TOTAL = ROWS * C4;
#pragma unroll
        for (int i0 = 0; i0 < TOTAL; i0 += NT) {
            const int i = i0 + tid;
            if (TOTAL % NT == 0 || i < TOTAL) {
                const int r = i / C4;
                const int c = (i - r * C4) << 2;
                int bytes = 0;
                if (r < rows_valid) {
                    const int left = cols_valid - c;
                    bytes = left >= 4 ? 16 : (left > 0 ? left * 4 : 0);
                }
                const float *src = bytes ? g + (long)r * g_ld + c : g;
                kmb_cp_async16(s + r * s_ld + c, src, bytes);
            }
        }
    } else {
        constexpr int TOTAL = ROWS * COLS;
#pragma unroll 4
        for (int i = tid; i < TOTAL; i += NT) {
            const int r = i / COLS;
            const int c = i - r * COLS;
            const bool ok = (r < rows_valid) && (c < cols_valid);
            const float *src = ok ? g + (long)r * g_ld + c : g;
            kmb_cp_async4(s + r * s_ld + c, src, ok);
        }
    }
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
