/*
 * Causal depthwise ND convolution (dense K^ndims kernel), forward and
 * backward, for sm_100a.  Semantics of the reference src/convnd.c:67-202:
 *
 *   out(p,d)  = bias[d] + sum_k in(p - (K-1-k_axis)_axis, d) * ker[k,d]
 *   din(s,d)  = sum_k dy(s + (K-1-k_axis)_axis, d) * ker[k,d]      (gather)
 *   dker[k,d] = sum_p dy(p,d) * in(p - (K-1-k_axis)_axis, d)
 *   dbias[d]  = sum_p dy(p,d)
 *
 * with k the row-major tap index (last axis fastest) and out-of-grid
 * neighbours counting as zero.  The convolution has no dependency between
 * outputs, so the reference's wavefront levels do not constrain the GPU:
 * every kernel is a single pass over the grid.
 *
 * 2D paths.  A thread owns one column j, a strip of rows and 4
 * consecutive channels (float4); a K x K window of float4 slides along the
 * strip in registers with the kernel taps, so each output row costs K*K
 * float4 FMAs.  The backward slides two windows (dy rows r..r+K-1 for the
 * gather-form dinput, input rows r-K+1..r for dkernel); dkernel/dbias
 * partials are folded in shared memory and added to global memory with
 * one atomic per CTA and (tap, channel).
 *
 *  - streamed rows (D a multiple of 64, K <= 3, 16-byte aligned tensors;
 *    the config-3 shape): a CTA covers 64 channels x 16 columns of a
 *    128-row (forward) or 256-row (backward) strip; whole rows with their column halo are copied by
 *    cp.async into a shared ring several rows ahead of the compute (deep
 *    enough to cover HBM latency at one CTA per SM), and each row reads
 *    only its new K values per tensor from shared memory;
 *  - direct (other 2D shapes): the windows load straight from global
 *    memory, column neighbours from L1.
 *
 * Any other rank uses the generic kernels (thread per point and channel).
 */
#include <string.h>

#include <type_traits>

#include <cuda_bf16.h>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kMaxNd = 8;

struct ConvDev {
    const float *in, *ker, *bias, *dy;
    float *out, *din, *dker, *dbias;
    long batch, P, D, K, KV;
    int nd;
    long dims[kMaxNd];
    long strides[kMaxNd];
};

/* ------------------------------------------------------------------ */
/* 2D fast path                                                        */
/* ------------------------------------------------------------------ */

constexpr int kThreads2d = 256;

template <int CW>
struct Vec;
template <>
struct Vec<4> {
    using T = float4;
    __device__ static T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
    __device__ static T load(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }
    __device__ static void store(float *p, T v) { *reinterpret_cast<float4 *>(p) = v; }
    __device__ static T fma(T a, T b, T c) {
        return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z),
                           fmaf(a.w, b.w, c.w));
    }
    __device__ static T add(T a, T b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
    __device__ static float get(T v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
};
/* float4 math on FFMA2 / FADD2 pairs (each element rounded as fmaf / +
 * round it), for the streamed backward whose issue rate it relieves */
struct Vec4p : Vec<4> {
    __device__ static T fma(T a, T b, T c) {
        const float2 lo = kmb_fma2(kmb_f2(a.x, a.y), kmb_f2(b.x, b.y), kmb_f2(c.x, c.y));
        const float2 hi = kmb_fma2(kmb_f2(a.z, a.w), kmb_f2(b.z, b.w), kmb_f2(c.z, c.w));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    __device__ static T add(T a, T b) {
        const float2 lo = kmb_add2(kmb_f2(a.x, a.y), kmb_f2(b.x, b.y));
        const float2 hi = kmb_add2(kmb_f2(a.z, a.w), kmb_f2(b.z, b.w));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    }
};
template <>
struct Vec<1> {
    using T = float;
    __device__ static T zero() { return 0.f; }
    __device__ static T load(const float *p) { return __ldg(p); }
    __device__ static void store(float *p, T v) { *p = v; }
    __device__ static T fma(T a, T b, T c) { return fmaf(a, b, c); }
    __device__ static T add(T a, T b) { return a + b; }
    __device__ static float get(T v, int) { return v; }
};

/* Activation element access of the streamed kernels.  The input, output,
 * dy and dinput tensors are E = float or bf16 in memory and fp32 in
 * registers; taps, bias, dkernel and dbias stay fp32.  bf16 results are
 * rounded to nearest even. */
template <typename E>
struct CIO;
template <>
struct CIO<float> {
    __device__ static float4 ld4(const float *s) { return *reinterpret_cast<const float4 *>(s); }
    __device__ static float2 ld2(const float *s) { return *reinterpret_cast<const float2 *>(s); }
    __device__ static float2 ldg2(const float *g) {
        return __ldg(reinterpret_cast<const float2 *>(g));
    }
    __device__ static void st4(float *g, float4 v) { *reinterpret_cast<float4 *>(g) = v; }
    __device__ static void st2(float *g, float2 v) { *reinterpret_cast<float2 *>(g) = v; }
};
template <>
struct CIO<__nv_bfloat16> {
    using E = __nv_bfloat16;
    __device__ static float2 cvt(unsigned u) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
    }
    __device__ static unsigned pack(float a, float b) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const unsigned *>(&h);
    }
    __device__ static float4 ld4(const E *s) {
        const uint2 u = *reinterpret_cast<const uint2 *>(s);
        const float2 a = cvt(u.x), b = cvt(u.y);
        return make_float4(a.x, a.y, b.x, b.y);
    }
    __device__ static float2 ld2(const E *s) { return cvt(*reinterpret_cast<const unsigned *>(s)); }
    __device__ static float2 ldg2(const E *g) {
        return cvt(__ldg(reinterpret_cast<const unsigned *>(g)));
    }
    __device__ static void st4(E *g, float4 v) {
        *reinterpret_cast<uint2 *>(g) = make_uint2(pack(v.x, v.y), pack(v.z, v.w));
    }
    __device__ static void st2(E *g, float2 v) { *reinterpret_cast<unsigned *>(g) = pack(v.x, v.y); }
};

/* Launch geometry of the 2D kernels: CGT channel groups x TJ columns per
 * CTA, TI rows per strip. */
struct Geo2d {
    int cgt, tj, ti;
    long ctiles, jtiles, strips;
};



template <int K, int CW>
__global__ void __launch_bounds__(kThreads2d) k_conv2d_fwd(ConvDev p, Geo2d g) {
    using V = Vec<CW>;
    using T = typename V::T;
    const int tid = threadIdx.x;
    const int cg = tid % g.cgt;
    const int jj = tid / g.cgt;
    const long H = p.dims[0], W = p.dims[1], D = p.D;
    const long ct = blockIdx.x % g.ctiles;
    const long jt = blockIdx.x / g.ctiles;
    const long j = jt * g.tj + jj;
    const long c = (ct * g.cgt + cg) * CW;
    const long b = blockIdx.z;
    const long r0 = (long)blockIdx.y * g.ti;
    if (j >= W || c >= D) return;

    T wk[K * K];
#pragma unroll
    for (int k = 0; k < K * K; ++k) wk[k] = V::load(p.ker + k * D + c);
    const T bias = p.bias ? V::load(p.bias + c) : V::zero();

    const float *base = p.in + b * H * W * D + c;
    float *obase = p.out + b * H * W * D + c;
    T win[K][K];
    /* rows r0-K+1 .. r0-1 */
#pragma unroll
    for (int a = 0; a < K - 1; ++a) {
        const long rr = r0 - (K - 1) + a;
#pragma unroll
        for (int q = 0; q < K; ++q) {
            const long cc = j - (K - 1) + q;
            win[a + 1][q] = (rr >= 0 && cc >= 0) ? V::load(base + (rr * W + cc) * D) : V::zero();
        }
    }
    const long rend = min(H, r0 + g.ti);
    for (long r = r0; r < rend; ++r) {
#pragma unroll
        for (int a = 0; a < K - 1; ++a)
#pragma unroll
            for (int q = 0; q < K; ++q) win[a][q] = win[a + 1][q];
#pragma unroll
        for (int q = 0; q < K; ++q) {
            const long cc = j - (K - 1) + q;
            win[K - 1][q] = cc >= 0 ? V::load(base + (r * W + cc) * D) : V::zero();
        }
        T s = bias;
#pragma unroll
        for (int a = 0; a < K; ++a)
#pragma unroll
            for (int q = 0; q < K; ++q) s = V::fma(win[a][q], wk[a * K + q], s);
        V::store(obase + (r * W + j) * D, s);
    }
}

template <int K, int CW>
__global__ void __launch_bounds__(kThreads2d) k_conv2d_bwd(ConvDev p, Geo2d g) {
    using V = Vec<CW>;
    using T = typename V::T;
    constexpr int NACC = K * K + 1; /* dkernel taps + dbias */
    extern __shared__ __align__(16) float red[]; /* [kThreads2d][NACC][CW] */
    const int tid = threadIdx.x;
    const int cg = tid % g.cgt;
    const int jj = tid / g.cgt;
    const long H = p.dims[0], W = p.dims[1], D = p.D;
    const long ct = blockIdx.x % g.ctiles;
    const long jt = blockIdx.x / g.ctiles;
    const long j = jt * g.tj + jj;
    const long c = (ct * g.cgt + cg) * CW;
    const long b = blockIdx.z;
    const long r0 = (long)blockIdx.y * g.ti;
    const bool act = j < W && c < D;

    T acc[NACC];
#pragma unroll
    for (int k = 0; k < NACC; ++k) acc[k] = V::zero();

    if (act) {
        T wk[K * K];
#pragma unroll
        for (int k = 0; k < K * K; ++k) wk[k] = V::load(p.ker + k * D + c);
        const float *ib = p.in + b * H * W * D + c;
        const float *gb = p.dy + b * H * W * D + c;
        float *db = p.din + b * H * W * D + c;
        const long rend = min(H, r0 + g.ti);
        /* walk rows downwards: r = rend-1 .. r0.
         * gwin[a][q] = dy(r + a, j + q)       a, q in [0, K)
         * iwin[a][q] = in(r - (K-1) + a, j - (K-1) + q) */
        T gwin[K][K], iwin[K][K];
        /* pre-shift state for r = rend-1: gwin[a] = dy(rend + a),
         * iwin[a] = in(rend - (K-1) + a), a in [0, K-1) */
#pragma unroll
        for (int a = 0; a < K - 1; ++a) {
            const long rg = rend + a;
            const long ri = rend - (K - 1) + a;
#pragma unroll
            for (int q = 0; q < K; ++q) {
                const long cg2 = j + q;
                const long ci = j - (K - 1) + q;
                gwin[a][q] = (rg < H && cg2 < W) ? V::load(gb + (rg * W + cg2) * D) : V::zero();
                iwin[a][q] = (ri >= 0 && ci >= 0) ? V::load(ib + (ri * W + ci) * D) : V::zero();
            }
        }
        for (long r = rend - 1; r >= r0; --r) {
            /* dy window: shift up (towards larger a), load row r at a = 0 */
#pragma unroll
            for (int a = K - 1; a > 0; --a)
#pragma unroll
                for (int q = 0; q < K; ++q) gwin[a][q] = gwin[a - 1][q];
#pragma unroll
            for (int q = 0; q < K; ++q) {
                const long cc = j + q;
                gwin[0][q] = cc < W ? V::load(gb + (r * W + cc) * D) : V::zero();
            }
            /* input window: rows r-(K-1) .. r; shift down, load row r-(K-1) */
#pragma unroll
            for (int a = K - 1; a > 0; --a)
#pragma unroll
                for (int q = 0; q < K; ++q) iwin[a][q] = iwin[a - 1][q];
            {
                const long rr = r - (K - 1);
#pragma unroll
                for (int q = 0; q < K; ++q) {
                    const long cc = j - (K - 1) + q;
                    iwin[0][q] = (rr >= 0 && cc >= 0) ? V::load(ib + (rr * W + cc) * D)
                                                      : V::zero();
                }
            }
            /* dinput(r, j): tap (k0, k1) reads dy(r + K-1-k0, j + K-1-k1) */
            T s = V::zero();
#pragma unroll
            for (int k0 = 0; k0 < K; ++k0)
#pragma unroll
                for (int k1 = 0; k1 < K; ++k1)
                    s = V::fma(gwin[K - 1 - k0][K - 1 - k1], wk[k0 * K + k1], s);
            V::store(db + (r * W + j) * D, s);
            /* dkernel / dbias at output (r, j) */
            const T gy = gwin[0][0];
#pragma unroll
            for (int k0 = 0; k0 < K; ++k0)
#pragma unroll
                for (int k1 = 0; k1 < K; ++k1)
                    acc[k0 * K + k1] = V::fma(gy, iwin[k0][k1], acc[k0 * K + k1]);
            acc[K * K] = V::add(acc[K * K], gy);
        }
    }

    /* fold the CTA's partials per (tap, channel) and add them to global */
#pragma unroll
    for (int k = 0; k < NACC; ++k)
#pragma unroll
        for (int i = 0; i < CW; ++i) red[(tid * NACC + k) * CW + i] = V::get(acc[k], i);
    __syncthreads();
    const int tj = g.tj;
    const int nout = g.cgt * NACC * CW;
    for (int o = tid; o < nout; o += kThreads2d) {
        const int i = o % CW;
        const int k = (o / CW) % NACC;
        const int cgo = o / (CW * NACC);
        const long cc = (ct * g.cgt + cgo) * CW + i;
        if (cc >= D) continue;
        float s = 0.f;
        for (int q = 0; q < tj; ++q) s += red[((q * g.cgt + cgo) * NACC + k) * CW + i];
        if (k < K * K) atomicAdd(p.dker + (long)k * D + cc, s);
        else if (p.dbias) atomicAdd(p.dbias + cc, s);
    }
}

/* ------------------------------------------------------------------ */
/* 2D backward, streamed rows                                          */
/* ------------------------------------------------------------------ */

/*
 * Backward for 64-channel tiles (D a multiple of 64: the config-3 shape),
 * bound by HBM: one read of dy and input and one write of dinput.  A CTA
 * of R2B_NT threads covers 64 channels as R2B_CG groups of R2B_CW channels
 * (a thread's float4) x R2B_TJ columns of a strip of R2B_TI rows and walks
 * the strip downwards.  "Stage" m carries dy row rend+K-2-m and input row
 * rend-1-m, each R2B_TJ + 2(K-1) columns wide (the column halo, zero-filled
 * outside the grid); row r = rend-1-n needs stages n .. n+K-1.  Stages are
 * copied by cp.async (16-byte units) into a ring of r2b_nr<K, E>() shared
 * rows, PD = r2b_pd<E>() stages ahead of the compute (R2B_PD for fp32
 * activations, twice that for bf16 ones, whose rows carry half the bytes).
 * A thread's K x K windows live
 * in registers indexed by stage % K (the row loop is unrolled by K, so no
 * window shifts) and only the new stage's K values per tensor come from
 * shared memory each row.  Rows n .. n+K-1 share one cp.async wait and one
 * barrier; a fast thread then issues stages n+PD .. n+PD+K-1 while a slow
 * one may still read stage n-1, so the ring holds PD + K + 1 rows.
 *
 * Tuning, config 3 on one B200 (backward, % of the measured copy
 * bandwidth): float4 channels, 256 threads, 6 stages, 256-row strips and
 * a register budget of one CTA per SM (196 registers) 76.7 %; the same
 * with 128-row strips 75.2 %, with 8 or 10 stages 76.1 / 76.6 %; float2
 * channel pairs (110 registers, 16 warps per SM) 72-74.7 %; the earlier
 * 182-register build 68.7 %.
 */
constexpr int R2_CG = 16;                 /* float4 channel groups per CTA (forward) */
constexpr int R2_TJ = kThreads2d / R2_CG; /* columns per CTA (forward) */
constexpr int R2_TI = 128;                /* rows per strip */
constexpr int R2_PD = 6;                  /* stages in flight */
constexpr int R2B_PD = 6;                  /* stages in flight */
constexpr int R2B_TI = 256;                /* rows per strip */
constexpr int R2B_CW = 4;                  /* channels per thread (a float4) */
constexpr int R2B_NT = 256;                /* threads per CTA */
constexpr int R2B_CG = 64 / R2B_CW;        /* channel groups per CTA */
constexpr int R2B_TJ = R2B_NT / R2B_CG;    /* columns per CTA */
using R2BVec = Vec4p;

/* ring rows: a fast thread issues stages n+PD .. n+PD+K-1 of its row group
 * while a slow one may still read stage n-1 of the previous group */
/* bf16 rows carry half the bytes: more stages keep the bytes in flight
 * per SM up */
#ifndef KMB_CONV_BF16_PD_MUL
#define KMB_CONV_BF16_PD_MUL 2
#endif
template <typename E>
__host__ __device__ constexpr int r2_pd() {
    return sizeof(E) == 2 ? KMB_CONV_BF16_PD_MUL * R2_PD : R2_PD;
}
template <typename E>
__host__ __device__ constexpr int r2b_pd() {
    return sizeof(E) == 2 ? KMB_CONV_BF16_PD_MUL * R2B_PD : R2B_PD;
}

template <int K, typename E>
__host__ __device__ constexpr int r2_nr() { return r2_pd<E>() + K + 1; }

template <int K>
__host__ __device__ constexpr int r2b_ws() { return R2B_TJ + 2 * (K - 1); }

template <int K, typename E>
__host__ __device__ constexpr int r2b_nr() { return r2b_pd<E>() + K + 1; }

template <int K, typename E>
__host__ __device__ constexpr size_t r2_smem_bytes() {
    /* two rings of r2b_nr rows of 64 channels; the final fold reuses them */
    const size_t ring = 2ull * r2b_nr<K, E>() * r2b_ws<K>() * 64 * sizeof(E);
    const size_t fold = (size_t)R2B_NT * (K * K + 1) * R2B_CW * 4;
    return ring > fold ? ring : fold;
}

template <int K, typename E>
__global__ void __launch_bounds__(R2B_NT, 1) k_conv2d_bwd_ring(ConvDev p, long ctiles,
                                                               long jtiles, long strips) {
    using V = R2BVec;
    using T = typename V::T;
    constexpr int CW = R2B_CW, CG = R2B_CG, TJ = R2B_TJ, NT = R2B_NT;
    constexpr int WS = r2b_ws<K>();
    constexpr int NR = r2b_nr<K, E>();
    constexpr int PD = r2b_pd<E>();
    constexpr int ROWF = WS * 64;                    /* elements per ring row */
    constexpr int NACC = K * K + 1;
    constexpr int EPU = 16 / (int)sizeof(E);         /* elements per 16-byte copy */
    constexpr int UPC = 64 / EPU;                    /* copies per column */
    constexpr int UNITS = WS * UPC;                  /* 16-byte copies per row */
    constexpr int CPT = (UNITS + NT - 1) / NT;       /* copies per thread */
    extern __shared__ __align__(16) float sm[];
    E *ring_g = reinterpret_cast<E *>(sm); /* dy rows   [NR][WS][64] */
    E *ring_i = ring_g + NR * ROWF;        /* input rows */

    const int tid = threadIdx.x;
    const int cg = tid % CG;
    const int jj = tid / CG;
    const long H = p.dims[0], W = p.dims[1], D = p.D;
    const long ct = blockIdx.x % ctiles;
    const long jt = blockIdx.x / ctiles;
    const long c0 = ct * 64;
    const long j0 = jt * TJ;
    const long j = j0 + jj;
    const long b = blockIdx.z;
    const long r0 = (long)blockIdx.y * R2B_TI;
    const long rend = min(H, r0 + R2B_TI);
    const int cnt = (int)(rend - r0);       /* rows of this strip */
    const int nstage = cnt + K - 1;
    const long jlo = j0 - (K - 1);
    const bool act = j < W;
    const E *gbase = reinterpret_cast<const E *>(p.dy) + b * H * W * D + c0;
    const E *ibase = reinterpret_cast<const E *>(p.in) + b * H * W * D + c0;

    /* this thread's copies of a stage: unit e = tid + c * NT of a row
     * (column jlo + e / UPC, channels EPU (e % UPC) ..); only the row moves */
    long coff[CPT];
    bool cok[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        const int e = tid + c * NT;
        const long col = jlo + e / UPC;
        cok[c] = e < UNITS && col >= 0 && col < W;
        coff[c] = col * D + (e % UPC) * EPU;
    }
    const long rowst = W * D;
    auto issue = [&](int m) {
        if (m < nstage) {
            const int slot = m % NR;
            const long rg = rend + K - 2 - m, ri = rend - 1 - m;
            E *dg = ring_g + slot * ROWF + tid * EPU, *di = ring_i + slot * ROWF + tid * EPU;
            const E *sg = gbase + rg * rowst, *si = ibase + ri * rowst;
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                if (UNITS % NT == 0 || tid + c * NT < UNITS) {
                    const bool gok = cok[c] && rg < H;
                    const bool iok = cok[c] && ri >= 0;
                    kmb_cp_async16(dg + c * NT * EPU, gok ? sg + coff[c] : gbase, gok ? 16 : 0);
                    kmb_cp_async16(di + c * NT * EPU, iok ? si + coff[c] : ibase, iok ? 16 : 0);
                }
            }
        }
        kmb_cp_async_commit();
    };

    T wk[K * K];
#pragma unroll
    for (int k = 0; k < K * K; ++k) wk[k] = V::load(p.ker + k * D + c0 + cg * CW);
    T acc[NACC];
#pragma unroll
    for (int k = 0; k < NACC; ++k) acc[k] = V::zero();
    T gw[K][K], iw[K][K]; /* [stage % K][column] */

    /* the new stage's K dy values (columns j .. j+K-1) and K input values
     * (columns j-K+1 .. j) of this thread */
    auto fetch = [&](int m, T (&g)[K], T (&iv)[K]) {
        const int slot = m % NR;
        const E *sg = ring_g + slot * ROWF + jj * 64 + cg * CW;
        const E *si = ring_i + slot * ROWF + jj * 64 + cg * CW;
#pragma unroll
        for (int q = 0; q < K; ++q) {
            g[q] = CIO<E>::ld4(sg + (K - 1 + q) * 64);
            iv[q] = CIO<E>::ld4(si + q * 64);
        }
    };

#pragma unroll 1
    for (int m = 0; m < PD; ++m) issue(m);
    /* stages 0 .. K-2 into the register windows */
    kmb_cp_async_wait<PD - (K - 1)>();
    __syncthreads();
#pragma unroll
    for (int m = 0; m < K - 1; ++m) fetch(m, gw[m % K], iw[m % K]);

    E *dbase = reinterpret_cast<E *>(p.din) + b * H * W * D + c0 + cg * CW;
    /* one row at compile-time phase PH = n % K (its stages are resident) */
    auto row = [&](int n, auto ph_tag) {
        constexpr int PH = decltype(ph_tag)::value;
        constexpr int NEW = (PH + K - 1) % K; /* slot of stage n+K-1 */
        fetch(n + K - 1, gw[NEW], iw[NEW]);
        if (act) {
            const long r = rend - 1 - n;
            /* dinput(r, j) = sum dy(r + K-1-k0, j + K-1-k1) w[k0][k1];
             * dy row r + K-1-k0 is stage n + k0 */
            T s = V::zero();
#pragma unroll
            for (int k0 = 0; k0 < K; ++k0)
#pragma unroll
                for (int k1 = 0; k1 < K; ++k1)
                    s = V::fma(gw[(PH + k0) % K][K - 1 - k1], wk[k0 * K + k1], s);
            CIO<E>::st4(dbase + (r * W + j) * D, s);
            /* dkernel: dy(r, j) (stage n+K-1, column 0) times input
             * (r - (K-1) + k0, j - (K-1) + k1) (stage n + K-1-k0) */
            const T gy = gw[NEW][0];
#pragma unroll
            for (int k0 = 0; k0 < K; ++k0)
#pragma unroll
                for (int k1 = 0; k1 < K; ++k1)
                    acc[k0 * K + k1] = V::fma(gy, iw[(PH + K - 1 - k0) % K][k1], acc[k0 * K + k1]);
            acc[K * K] = V::add(acc[K * K], gy);
        }
    };
    /* rows n .. n+K-1 share one wait and one barrier: they read stages
     * n+K-1 .. n+2K-2, and stages n+PD .. n+PD+K-1 go out first */
    for (int n = 0; n < cnt; n += K) {
#pragma unroll
        for (int i = 0; i < K; ++i) issue(n + PD + i);
        kmb_cp_async_wait<PD - K + 1>();
        __syncthreads();
        row(n, std::integral_constant<int, 0>{});
        if (K > 1 && n + 1 < cnt) row(n + 1, std::integral_constant<int, 1 % K>{});
        if (K > 2 && n + 2 < cnt) row(n + 2, std::integral_constant<int, 2 % K>{});
        if (K > 3 && n + 3 < cnt) row(n + 3, std::integral_constant<int, 3 % K>{});
        if (K > 4 && n + 4 < cnt) row(n + 4, std::integral_constant<int, 4 % K>{});
    }

    /* the ring is reused for the fold: no copy may still be in flight */
    kmb_cp_async_wait<0>();
    __syncthreads();
    float *red = sm; /* [NT][NACC][CW] */
#pragma unroll
    for (int k = 0; k < NACC; ++k)
        *reinterpret_cast<T *>(red + (tid * NACC + k) * CW) = act ? acc[k] : V::zero();
    __syncthreads();
    for (int o = tid; o < CG * NACC * CW; o += NT) {
        const int i = o % CW;
        const int k = (o / CW) % NACC;
        const int cgo = o / (CW * NACC);
        const long cc = c0 + cgo * CW + i;
        float s = 0.f;
        for (int q = 0; q < TJ; ++q) s += red[((q * CG + cgo) * NACC + k) * CW + i];
        if (k < K * K) atomicAdd(p.dker + (long)k * D + cc, s);
        else if (p.dbias) atomicAdd(p.dbias + cc, s);
    }
}

template <int K, typename E>
cudaError_t launch2d_bwd_ring(const ConvDev &p, cudaStream_t s) {
    const long ctiles = p.D / 64;
    const long jtiles = (p.dims[1] + R2B_TJ - 1) / R2B_TJ;
    const long strips = (p.dims[0] + R2B_TI - 1) / R2B_TI;
    const size_t smem = r2_smem_bytes<K, E>();
    auto kern = k_conv2d_bwd_ring<K, E>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)(ctiles * jtiles), (unsigned)strips, (unsigned)p.batch);
    kern<<<grid, R2B_NT, smem, s>>>(p, ctiles, jtiles, strips);
    return cudaGetLastError();
}

/*
 * Forward with the same streamed rows: stage m is input row r0-(K-1)+m
 * (R2_TJ + K-1 columns with the left halo); row r = r0+n reads stages
 * n .. n+K-1 from its K x K register window.
 */
template <int K>
__host__ __device__ constexpr int r2f_ws() { return R2_TJ + K - 1; }

template <int K, typename E>
__host__ __device__ constexpr size_t r2f_smem_bytes() {
    return (size_t)r2_nr<K, E>() * r2f_ws<K>() * R2_CG * 4 * sizeof(E);
}

template <int K, class V, typename E>
__global__ void __launch_bounds__(kThreads2d) k_conv2d_fwd_ring(ConvDev p, long ctiles) {
    using T = float4;
    constexpr int WS = r2f_ws<K>();
    constexpr int NR = r2_nr<K, E>();
    constexpr int PD = r2_pd<E>();
    constexpr int ROWF = WS * R2_CG * 4;             /* elements per ring row */
    constexpr int EPU = 16 / (int)sizeof(E);         /* elements per 16-byte copy */
    constexpr int UPC = R2_CG * 4 / EPU;             /* copies per column */
    constexpr int UNITS = WS * UPC;
    constexpr int CPT = (UNITS + kThreads2d - 1) / kThreads2d;
    extern __shared__ __align__(16) float smf[];
    E *sm = reinterpret_cast<E *>(smf);

    const int tid = threadIdx.x;
    const int cg = tid % R2_CG;
    const int jj = tid / R2_CG;
    const long H = p.dims[0], W = p.dims[1], D = p.D;
    const long ct = blockIdx.x % ctiles;
    const long jt = blockIdx.x / ctiles;
    const long c0 = ct * R2_CG * 4;
    const long j0 = jt * R2_TJ;
    const long j = j0 + jj;
    const long b = blockIdx.z;
    const long r0 = (long)blockIdx.y * R2_TI;
    const long rend = min(H, r0 + R2_TI);
    const int cnt = (int)(rend - r0);
    const int nstage = cnt + K - 1;
    const long jlo = j0 - (K - 1);
    const bool act = j < W;
    const E *ibase = reinterpret_cast<const E *>(p.in) + b * H * W * D + c0;

    long coff[CPT];
    bool cok[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        const int e = tid + c * kThreads2d;
        const long col = jlo + e / UPC;
        cok[c] = e < UNITS && col >= 0 && col < W;
        coff[c] = col * D + (e % UPC) * EPU;
    }
    const long rowst = W * D;
    auto issue = [&](int m) {
        if (m < nstage) {
            const long ri = r0 - (K - 1) + m;
            E *di = sm + (m % NR) * ROWF + tid * EPU;
            const E *si = ibase + ri * rowst;
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                if (tid + c * kThreads2d < UNITS) {
                    const bool ok = cok[c] && ri >= 0;
                    kmb_cp_async16(di + c * kThreads2d * EPU, ok ? si + coff[c] : ibase,
                                   ok ? 16 : 0);
                }
            }
        }
        kmb_cp_async_commit();
    };

    T wk[K * K];
#pragma unroll
    for (int k = 0; k < K * K; ++k) wk[k] = V::load(p.ker + k * D + c0 + cg * 4);
    const T bias = p.bias ? V::load(p.bias + c0 + cg * 4) : V::zero();
    T iw[K][K]; /* [stage % K][column] */
    auto fetch = [&](int m, T (&iv)[K]) {
        const E *si = sm + (m % NR) * ROWF + (jj * R2_CG + cg) * 4;
#pragma unroll
        for (int q = 0; q < K; ++q) iv[q] = CIO<E>::ld4(si + q * R2_CG * 4);
    };

#pragma unroll 1
    for (int m = 0; m < PD; ++m) issue(m);
    kmb_cp_async_wait<PD - (K - 1)>();
    __syncthreads();
#pragma unroll
    for (int m = 0; m < K - 1; ++m) fetch(m, iw[m % K]);

    E *obase = reinterpret_cast<E *>(p.out) + b * H * W * D + c0 + cg * 4;
    auto row = [&](int n, auto ph_tag) {
        constexpr int PH = decltype(ph_tag)::value;
        fetch(n + K - 1, iw[(PH + K - 1) % K]);
        if (act) {
            T s = bias;
#pragma unroll
            for (int k0 = 0; k0 < K; ++k0)
#pragma unroll
                for (int k1 = 0; k1 < K; ++k1)
                    s = V::fma(iw[(PH + k0) % K][k1], wk[k0 * K + k1], s);
            CIO<E>::st4(obase + ((r0 + n) * W + j) * D, s);
        }
    };
    for (int n = 0; n < cnt; n += K) {
#pragma unroll
        for (int i = 0; i < K; ++i) issue(n + PD + i);
        kmb_cp_async_wait<PD - K + 1>();
        __syncthreads();
        row(n, std::integral_constant<int, 0>{});
        if (K > 1 && n + 1 < cnt) row(n + 1, std::integral_constant<int, 1 % K>{});
        if (K > 2 && n + 2 < cnt) row(n + 2, std::integral_constant<int, 2 % K>{});
    }
    kmb_cp_async_wait<0>();
}

template <int K, typename E>
cudaError_t launch2d_fwd_ring(const ConvDev &p, cudaStream_t s) {
    const long ctiles = p.D / (4 * R2_CG);
    const long jtiles = (p.dims[1] + R2_TJ - 1) / R2_TJ;
    const long strips = (p.dims[0] + R2_TI - 1) / R2_TI;
    const size_t smem = r2f_smem_bytes<K, E>();
    auto kern = k_conv2d_fwd_ring<K, Vec4p, E>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)(ctiles * jtiles), (unsigned)strips, (unsigned)p.batch);
    kern<<<grid, kThreads2d, smem, s>>>(p, ctiles);
    return cudaGetLastError();
}

/* K <= 3: the two K x K float4 windows, the taps and the accumulators fit
 * the register file without spills up to K = 3 */
constexpr int R2_KMAX = 3;

template <typename E>
cudaError_t dispatch2d_fwd_ring(const ConvDev &p, cudaStream_t s) {
    switch (p.K) {
    case 1: return launch2d_fwd_ring<1, E>(p, s);
    case 2: return launch2d_fwd_ring<2, E>(p, s);
    case 3: return launch2d_fwd_ring<3, E>(p, s);
    default: return cudaErrorNotSupported;
    }
}

template <typename E>
cudaError_t dispatch2d_bwd_ring(const ConvDev &p, cudaStream_t s) {
    switch (p.K) {
    case 1: return launch2d_bwd_ring<1, E>(p, s);
    case 2: return launch2d_bwd_ring<2, E>(p, s);
    case 3: return launch2d_bwd_ring<3, E>(p, s);
    default: return cudaErrorNotSupported;
    }
}

/* ------------------------------------------------------------------ */
/* 3D (the Mamba-ND volumes)                                           */
/* ------------------------------------------------------------------ */

/*
 * 3D causal depthwise convolution (the Mamba-ND volumes) for K <= 3, D a
 * multiple of 4 and 16-byte aligned tensors.  A warp owns two x-adjacent
 * (y, x) columns of the volume and 64 channels (2 per lane); a CTA is a
 * 4 x 8 tile of columns, and channel blocks are the fastest grid dimension
 * (a tile's CTAs read whole point vectors together).  The lane keeps its
 * channels' K^3 taps in registers and walks z, so each input slice is
 * read once and feeds K rolling output accumulators per column:
 *   forward (z ascending)  out(z) = bias + sum_o in(z - oz, y - oy, x - ox) w[K-1-o]
 *   dinput  (z descending) din(z) = sum_o dy(z + oz, y + oy, x + ox) w[K-1-o]
 * after slice s the accumulator of the output at s is complete.  dkernel
 * keeps K^3 accumulators and a window of K dy slices per column instead:
 *   dker[K-1-o] += dy(s + oz, y, x) in(s, y - oy, x - ox),  dbias += dy(s)
 * and folds them over the CTA's warps, one atomic per (tap, channel).
 *
 * The slices are staged: the CTA's input slices (its columns and the K - 1
 * halo columns on each in-plane axis, 64 channels) stream through a ring
 * of ZS_R slices in shared memory (cp.async, 16-byte chunks, zero-filled
 * outside the volume), ZS_R - 1 slices ahead of the compute, so the loads
 * in flight cost no registers.  A lane reads the K x (K + 1) neighbours
 * of its column pair from the slice (8-byte reads of 256-byte column
 * rows).  dkernel stages the dy slice of its own columns K - 1 slices
 * ahead of the input slice, for its windows of dy.  HBM sees one read of
 * each input and one write of each output.
 */
constexpr int Z3_TY = 4, Z3_TX = 8;                      /* columns of a CTA */
constexpr int Z3_PX = 2;                                 /* x-adjacent columns of a warp */
constexpr int Z3_CH = 64;                                /* channels of a CTA (a warp) */
constexpr int Z3_THREADS = Z3_TY * Z3_TX / Z3_PX * 32;
constexpr int ZS_R = 8;                                  /* slices in the ring */

/* the warp's columns: tile origin (y0, x0), in-tile row wy and first
 * column wx, and per column the element offset of (b, z = 0, y, x, c) */
struct Tile3 {
    int Z, Y, X, y0, x0, wy, wx;
    int sz;                /* element stride of z (P * D < 2^31) */
    long c;                /* first of the lane's 2 channels */
    long base[Z3_PX];
    bool on[Z3_PX];        /* column and channels inside the volume */
};

__device__ __forceinline__ Tile3 tile3(const ConvDev &p) {
    Tile3 t;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    t.Z = (int)p.dims[0];
    t.Y = (int)p.dims[1];
    t.X = (int)p.dims[2];
    const int ntx = (t.X + Z3_TX - 1) / Z3_TX;
    t.y0 = (int)(blockIdx.y / ntx) * Z3_TY;
    t.x0 = (int)(blockIdx.y % ntx) * Z3_TX;
    t.wy = w / (Z3_TX / Z3_PX);
    t.wx = (w % (Z3_TX / Z3_PX)) * Z3_PX;
    t.c = (long)blockIdx.x * Z3_CH + lane * 2;
    t.sz = t.Y * t.X * (int)p.D;
    const int y = t.y0 + t.wy;
#pragma unroll
    for (int u = 0; u < Z3_PX; ++u) {
        const int x = t.x0 + t.wx + u;
        t.on[u] = y < t.Y && x < t.X && t.c < p.D;
        t.base[u] = (long)blockIdx.z * p.P * p.D + ((long)y * t.X + x) * p.D + t.c;
    }
    return t;
}

__device__ __forceinline__ float2 ld2(const float *a) {
    return __ldg(reinterpret_cast<const float2 *>(a));
}

template <int K, typename E>
struct ZSLayout {
    static constexpr int CY = Z3_TY + K - 1, CX = Z3_TX + K - 1; /* staged columns */
    static constexpr int NCOL = CY * CX;
    static constexpr int EPU = 16 / (int)sizeof(E);    /* elements per 16-byte chunk */
    static constexpr int UPC = Z3_CH / EPU;            /* chunks per column */
    static constexpr int SL = NCOL * Z3_CH;            /* elements of a staged input slice */
    static constexpr int SLD = Z3_TY * Z3_TX * Z3_CH;  /* elements of a dy slice (dkernel) */
    static constexpr int NJ = (NCOL * UPC + Z3_THREADS - 1) / Z3_THREADS; /* chunks a thread */
    static constexpr int NV = Z3_PX + K - 1;           /* neighbour columns of a warp per row */
    static constexpr int DYJ = Z3_TY * Z3_TX * UPC;    /* dy chunks of a slice (dkernel) */
    static_assert(DYJ <= Z3_THREADS, "at most one dy chunk a thread");
};

/* the 16-byte chunk jobs of a thread for one staged slice: element offset
 * of slice 0 (or -1 when the column or the channels are outside) and the
 * offset in the slot */
template <int K, int SGN, typename E>
struct ZSJobs {
    using L = ZSLayout<K, E>;
    long src[L::NJ];
    int dst[L::NJ];
    __device__ __forceinline__ void init(const ConvDev &p, int y0, int x0, long c0, int tid) {
        const int Y = (int)p.dims[1], X = (int)p.dims[2];
#pragma unroll
        for (int i = 0; i < L::NJ; ++i) {
            const int e = tid + i * Z3_THREADS;
            const int col = e / L::UPC, ch = e % L::UPC;
            const int cy = col / L::CX, cx = col % L::CX;
            const int y = SGN < 0 ? y0 - (K - 1) + cy : y0 + cy;
            const int x = SGN < 0 ? x0 - (K - 1) + cx : x0 + cx;
            const long c = c0 + ch * L::EPU;
            const bool ok = e < L::NCOL * L::UPC && y >= 0 && y < Y && x >= 0 && x < X &&
                            c < p.D;
            src[i] = ok ? (long)blockIdx.z * p.P * p.D + ((long)y * X + x) * p.D + c : -1;
            dst[i] = e < L::NCOL * L::UPC ? col * Z3_CH + ch * L::EPU : -1;
        }
    }
    __device__ __forceinline__ void issue(E *slot, const E *base, long zoff) const {
#pragma unroll
        for (int i = 0; i < L::NJ; ++i)
            if (dst[i] >= 0)
                kmb_cp_async16(slot + dst[i], base + (src[i] >= 0 ? src[i] + zoff : 0),
                               src[i] >= 0 ? 16 : 0);
    }
};

/* SGN = -1: forward (z ascending); SGN = +1: dinput (z descending) */
template <int K, int SGN, typename E>
__global__ void __launch_bounds__(Z3_THREADS, 1) k_conv3d_zring(ConvDev p) {
    using L = ZSLayout<K, E>;
    constexpr int KK = K * K, KV = K * KK, NV = L::NV;
    extern __shared__ __align__(16) float zsmf[];
    E *zsm = reinterpret_cast<E *>(zsmf);
    const int tid = threadIdx.x, lane = tid & 31;
    const Tile3 t = tile3(p);
    const long c0 = (long)blockIdx.x * Z3_CH;
    const bool cok = t.c < p.D;
    float2 wt[KV];
#pragma unroll
    for (int k = 0; k < KV; ++k) wt[k] = cok ? ld2(p.ker + k * p.D + t.c) : kmb_f2s(0.f);
    ZSJobs<K, SGN, E> jobs;
    jobs.init(p, t.y0, t.x0, c0, tid);
    const E *src = reinterpret_cast<const E *>(SGN < 0 ? p.in : p.dy);
    E *dst = reinterpret_cast<E *>(SGN < 0 ? p.out : p.din);
    const float2 b2 = (SGN < 0 && p.bias && cok) ? ld2(p.bias + t.c) : kmb_f2s(0.f);
    float2 acc[Z3_PX][K];
#pragma unroll
    for (int u = 0; u < Z3_PX; ++u)
#pragma unroll
        for (int i = 0; i < K; ++i) acc[u][i] = b2;
    /* slice t of the walk is z = t (forward) or Z - 1 - t (dinput) */
    auto zof = [&](int s) { return (long)(SGN < 0 ? s : t.Z - 1 - s) * t.sz; };
#pragma unroll 1
    for (int s = 0; s < ZS_R - 1; ++s) {
        if (s < t.Z) jobs.issue(zsm + s * L::SL, src, zof(s));
        kmb_cp_async_commit();
    }
    /* neighbour column i of in-plane row oy in a staged slice: forward
     * x0 + wx + i - (K - 1) at row y - oy; dinput x0 + wx + i at row y + oy */
    int nb[K];
#pragma unroll
    for (int oy = 0; oy < K; ++oy) {
        const int cy = SGN < 0 ? t.wy + (K - 1) - oy : t.wy + oy;
        nb[oy] = (cy * L::CX + t.wx) * Z3_CH + lane * 2;
    }
    int slot = 0;
#pragma unroll 1
    for (int s = 0; s < t.Z; ++s) {
        kmb_cp_async_wait<ZS_R - 2>();
        __syncthreads();
        if (s + ZS_R - 1 < t.Z) {
            const int ns = slot == 0 ? ZS_R - 1 : slot - 1; /* (s + ZS_R - 1) % ZS_R */
            jobs.issue(zsm + ns * L::SL, src, zof(s + ZS_R - 1));
        }
        kmb_cp_async_commit();
        const E *sl = zsm + slot * L::SL;
        slot = slot + 1 == ZS_R ? 0 : slot + 1;
        float2 v[K][NV];
#pragma unroll
        for (int oy = 0; oy < K; ++oy)
#pragma unroll
            for (int i = 0; i < NV; ++i)
                v[oy][i] = CIO<E>::ld2(sl + nb[oy] + i * Z3_CH);
#pragma unroll
        for (int u = 0; u < Z3_PX; ++u)
#pragma unroll
            for (int oz = 0; oz < K; ++oz)
#pragma unroll
                for (int oy = 0; oy < K; ++oy)
#pragma unroll
                    for (int ox = 0; ox < K; ++ox)
                        acc[u][oz] = kmb_fma2(v[oy][SGN < 0 ? u + (K - 1) - ox : u + ox],
                                              wt[KV - 1 - (oz * KK + oy * K + ox)], acc[u][oz]);
        const long zo = zof(s);
#pragma unroll
        for (int u = 0; u < Z3_PX; ++u) {
            if (t.on[u]) CIO<E>::st2(dst + t.base[u] + zo, acc[u][0]);
#pragma unroll
            for (int i = 0; i + 1 < K; ++i) acc[u][i] = acc[u][i + 1];
            acc[u][K - 1] = b2;
        }
    }
}

template <int K, typename E>
__global__ void __launch_bounds__(Z3_THREADS, 1) k_conv3d_zring_param(ConvDev p) {
    using L = ZSLayout<K, E>;
    constexpr int KK = K * K, KV = K * KK, NV = L::NV;
    constexpr int SLOT = L::SL + L::SLD;
    extern __shared__ __align__(16) float zsmf[];
    E *zsm = reinterpret_cast<E *>(zsmf);
    __shared__ float2 red[Z3_THREADS / 32][32];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const Tile3 t = tile3(p);
    const long c0 = (long)blockIdx.x * Z3_CH;
    ZSJobs<K, -1, E> jobs;
    jobs.init(p, t.y0, t.x0, c0, tid);
    const E *in = reinterpret_cast<const E *>(p.in), *dy = reinterpret_cast<const E *>(p.dy);
    /* dy of the CTA's own columns: at most one 16-byte chunk a thread */
    const bool djob = tid < L::DYJ;
    const int dcol = tid / L::UPC, dch = tid % L::UPC;
    const int dyy = t.y0 + dcol / Z3_TX, dxx = t.x0 + dcol % Z3_TX;
    const bool dok = djob && dyy < t.Y && dxx < t.X && c0 + dch * L::EPU < p.D;
    const long dsrc = dok ? (long)blockIdx.z * p.P * p.D + ((long)dyy * t.X + dxx) * p.D + c0 +
                                dch * L::EPU
                          : 0;
    const int ddst = L::SL + dcol * Z3_CH + dch * L::EPU;
    auto issue = [&](int s) { /* input slice s and dy slice s + K - 1 */
        E *slot = zsm + (s % ZS_R) * SLOT;
        jobs.issue(slot, in, (long)s * t.sz);
        const bool ok = dok && s + K - 1 < t.Z;
        if (djob)
            kmb_cp_async16(slot + ddst, dy + (ok ? dsrc + (long)(s + K - 1) * t.sz : 0),
                           ok ? 16 : 0);
    };
#pragma unroll 1
    for (int s = 0; s < ZS_R - 1; ++s) {
        if (s < t.Z) issue(s);
        kmb_cp_async_commit();
    }
    int nb[K];
#pragma unroll
    for (int oy = 0; oy < K; ++oy)
        nb[oy] = ((t.wy + (K - 1) - oy) * L::CX + t.wx) * Z3_CH + lane * 2;
    /* this lane's dy of its columns in a slot */
    const int dme = L::SL + (t.wy * Z3_TX + t.wx) * Z3_CH + lane * 2;
    float2 acc[KV], accb = kmb_f2s(0.f);
#pragma unroll
    for (int k = 0; k < KV; ++k) acc[k] = kmb_f2s(0.f);
    float2 dyw[Z3_PX][K]; /* dy of each column at slices s .. s + K - 1 */
#pragma unroll
    for (int u = 0; u < Z3_PX; ++u)
#pragma unroll
        for (int i = 0; i + 1 < K; ++i)
            dyw[u][i] = t.on[u] && i < t.Z ? CIO<E>::ldg2(dy + t.base[u] + (long)i * t.sz)
                                           : kmb_f2s(0.f);
#pragma unroll 1
    for (int s = 0; s < t.Z; ++s) {
        kmb_cp_async_wait<ZS_R - 2>();
        __syncthreads();
        if (s + ZS_R - 1 < t.Z) issue(s + ZS_R - 1);
        kmb_cp_async_commit();
        const E *sl = zsm + (s % ZS_R) * SLOT;
#pragma unroll
        for (int u = 0; u < Z3_PX; ++u) dyw[u][K - 1] = CIO<E>::ld2(sl + dme + u * Z3_CH);
        float2 v[K][NV];
#pragma unroll
        for (int oy = 0; oy < K; ++oy)
#pragma unroll
            for (int i = 0; i < NV; ++i) v[oy][i] = CIO<E>::ld2(sl + nb[oy] + i * Z3_CH);
#pragma unroll
        for (int u = 0; u < Z3_PX; ++u) {
#pragma unroll
            for (int oz = 0; oz < K; ++oz)
#pragma unroll
                for (int oy = 0; oy < K; ++oy)
#pragma unroll
                    for (int ox = 0; ox < K; ++ox) {
                        const int k = KV - 1 - (oz * KK + oy * K + ox);
                        acc[k] = kmb_fma2(dyw[u][oz], v[oy][u + (K - 1) - ox], acc[k]);
                    }
            accb = kmb_add2(accb, dyw[u][0]);
#pragma unroll
            for (int i = 0; i + 1 < K; ++i) dyw[u][i] = dyw[u][i + 1];
        }
    }
    /* fold the CTA's warps, one tap at a time (columns outside the volume
     * and channels past D hold zeros) */
    const int ntap = p.dbias ? KV + 1 : KV;
#pragma unroll
    for (int k = 0; k < KV + 1; ++k) {
        if (k < ntap) {
            red[w][lane] = k < KV ? acc[k] : accb;
            __syncthreads();
            if (w == 0 && t.c < p.D) {
                float2 r = red[0][lane];
                for (int ww = 1; ww < Z3_THREADS / 32; ++ww) r = kmb_add2(r, red[ww][lane]);
                float *d = k < KV ? p.dker + k * p.D + t.c : p.dbias + t.c;
                if (((uintptr_t)d & 7u) == 0) {
                    atomicAdd(reinterpret_cast<float2 *>(d), r);
                } else { /* dkernel / dbias need not be 8-byte aligned */
                    atomicAdd(d, r.x);
                    atomicAdd(d + 1, r.y);
                }
            }
            __syncthreads();
        }
    }
}

template <int K, typename E>
cudaError_t launch3d_zring(const ConvDev &p, bool bwd, cudaStream_t s) {
    using L = ZSLayout<K, E>;
    const unsigned tiles = (unsigned)(((p.dims[1] + Z3_TY - 1) / Z3_TY) *
                                      ((p.dims[2] + Z3_TX - 1) / Z3_TX));
    dim3 grid((unsigned)((p.D + Z3_CH - 1) / Z3_CH), tiles, (unsigned)p.batch);
    const size_t sm1 = sizeof(E) * ZS_R * L::SL;
    const size_t sm2 = sizeof(E) * ZS_R * (L::SL + L::SLD);
    cudaError_t e;
    if (!bwd) {
        auto fk = k_conv3d_zring<K, -1, E>;
        e = cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
        if (e != cudaSuccess) return e;
        fk<<<grid, Z3_THREADS, sm1, s>>>(p);
        return cudaGetLastError();
    }
    auto bk = k_conv3d_zring<K, +1, E>;
    e = cudaFuncSetAttribute(bk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
    if (e != cudaSuccess) return e;
    bk<<<grid, Z3_THREADS, sm1, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    auto pk = k_conv3d_zring_param<K, E>;
    e = cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
    if (e != cudaSuccess) return e;
    pk<<<grid, Z3_THREADS, sm2, s>>>(p);
    return cudaGetLastError();
}

template <typename E>
cudaError_t dispatch3d(const ConvDev &p, bool bwd, cudaStream_t s) {
    switch (p.K) {
    case 1: return launch3d_zring<1, E>(p, bwd, s);
    case 2: return launch3d_zring<2, E>(p, bwd, s);
    case 3: return launch3d_zring<3, E>(p, bwd, s);
    default: return cudaErrorNotSupported;
    }
}

bool use_3d(const ConvDev &p) { return p.nd == 3 && p.K >= 1 && p.K <= 3; }

/* ------------------------------------------------------------------ */
/* generic ND                                                          */
/* ------------------------------------------------------------------ */

__device__ __forceinline__ void unravel(const ConvDev &p, long lin, long *co) {
#pragma unroll
    for (int a = 0; a < kMaxNd; ++a)
        if (a < p.nd) co[a] = (lin / p.strides[a]) % p.dims[a];
}

/* Offset of the tap kl neighbour of `co` in direction sgn (-1: causal
 * source for forward / dkernel, +1: output for the dinput gather), or -1. */
__device__ __forceinline__ long tap_neighbor(const ConvDev &p, const long *co, long kl, int sgn) {
    long off = 0;
    for (int a = p.nd - 1; a >= 0; --a) {
        const long ka = kl % p.K;
        kl /= p.K;
        const long v = co[a] + sgn * (p.K - 1 - ka);
        if (v < 0 || v >= p.dims[a]) return -1;
        off += v * p.strides[a];
    }
    return off;
}

__global__ void k_convnd_fwd_generic(ConvDev p) {
    const long total = p.batch * p.P * p.D;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long)gridDim.x * blockDim.x) {
        const long d = e % p.D;
        const long pt = (e / p.D) % p.P;
        const long b = e / (p.D * p.P);
        long co[kMaxNd];
        unravel(p, pt, co);
        const float *ib = p.in + b * p.P * p.D;
        float s = p.bias ? p.bias[d] : 0.f;
        for (long kl = 0; kl < p.KV; ++kl) {
            const long src = tap_neighbor(p, co, kl, -1);
            if (src >= 0) s = fmaf(ib[src * p.D + d], p.ker[kl * p.D + d], s);
        }
        p.out[e] = s;
    }
}

__global__ void k_convnd_bwd_input_generic(ConvDev p) {
    const long total = p.batch * p.P * p.D;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long)gridDim.x * blockDim.x) {
        const long d = e % p.D;
        const long pt = (e / p.D) % p.P;
        const long b = e / (p.D * p.P);
        long co[kMaxNd];
        unravel(p, pt, co);
        const float *gb = p.dy + b * p.P * p.D;
        float s = 0.f;
        for (long kl = 0; kl < p.KV; ++kl) {
            const long o = tap_neighbor(p, co, kl, +1);
            if (o >= 0) s = fmaf(gb[o * p.D + d], p.ker[kl * p.D + d], s);
        }
        p.din[e] = s;
    }
}

/* blockIdx.y = channel d, blockIdx.z = tap kl (KV) or KV for dbias;
 * blockIdx.x strides over the batch x points. */
__global__ void __launch_bounds__(256) k_convnd_bwd_param_generic(ConvDev p) {
    __shared__ float wsum[8];
    const long d = blockIdx.y;
    const long kl = blockIdx.z;
    const long total = p.batch * p.P;
    float s = 0.f;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long)gridDim.x * blockDim.x) {
        const long pt = e % p.P;
        const long b = e / p.P;
        const float gy = p.dy[(b * p.P + pt) * p.D + d];
        if (kl == p.KV) {
            s += gy;
        } else {
            long co[kMaxNd];
            unravel(p, pt, co);
            const long src = tap_neighbor(p, co, kl, -1);
            if (src >= 0) s = fmaf(gy, p.in[(b * p.P + src) * p.D + d], s);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += wsum[w];
        if (kl == p.KV) {
            if (p.dbias) atomicAdd(p.dbias + d, t);
        } else {
            atomicAdd(p.dker + kl * p.D + d, t);
        }
    }
}

/* ------------------------------------------------------------------ */
/* launch                                                              */
/* ------------------------------------------------------------------ */

bool make_dev(const KmbConvND *a, ConvDev *p) {
    memset(p, 0, sizeof *p);
    p->in = a->input; p->ker = a->kernel; p->bias = a->bias; p->dy = a->dy;
    p->out = a->output; p->din = a->dinput; p->dker = a->dkernel; p->dbias = a->dbias;
    p->batch = a->batch; p->D = a->D; p->K = a->K; p->nd = (int)a->ndims;
    long s = 1;
    for (int ax = p->nd - 1; ax >= 0; --ax) {
        p->dims[ax] = a->dims[ax];
        p->strides[ax] = s;
        s *= a->dims[ax];
    }
    p->P = s;
    long kv = 1;
    for (int ax = 0; ax < p->nd; ++ax) kv *= a->K;
    p->KV = kv;
    return true;
}

Geo2d geo2d(const ConvDev &p, int cw, int ti) {
    Geo2d g;
    const long groups = (p.D + cw - 1) / cw;
    g.cgt = (int)(groups < 16 ? groups : 16);
    g.tj = kThreads2d / g.cgt;
    g.ti = ti;
    g.ctiles = (groups + g.cgt - 1) / g.cgt;
    g.jtiles = (p.dims[1] + g.tj - 1) / g.tj;
    g.strips = (p.dims[0] + ti - 1) / ti;
    return g;
}

template <int K, int CW>
cudaError_t launch2d(const ConvDev &p, bool bwd, cudaStream_t s) {
    const Geo2d g = geo2d(p, CW, bwd ? 64 : 32);
    dim3 grid((unsigned)(g.ctiles * g.jtiles), (unsigned)g.strips, (unsigned)p.batch);
    if (!bwd) {
        k_conv2d_fwd<K, CW><<<grid, kThreads2d, 0, s>>>(p, g);
    } else {
        const size_t smem = sizeof(float) * kThreads2d * (K * K + 1) * CW;
        auto kern = k_conv2d_bwd<K, CW>;
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem);
            if (e != cudaSuccess) return e;
        }
        kern<<<grid, kThreads2d, smem, s>>>(p, g);
    }
    return cudaGetLastError();
}

template <int CW>
cudaError_t dispatch2d(const ConvDev &p, bool bwd, cudaStream_t s) {
    switch (p.K) {
    case 1: return launch2d<1, CW>(p, bwd, s);
    case 2: return launch2d<2, CW>(p, bwd, s);
    case 3: return launch2d<3, CW>(p, bwd, s);
    case 4: return launch2d<4, CW>(p, bwd, s);
    case 5: return launch2d<5, CW>(p, bwd, s);
    default: return cudaErrorNotSupported;
    }
}

bool use_2d(const ConvDev &p) { return p.nd == 2 && p.K >= 1 && p.K <= 5; }

bool aligned4(const KmbConvND *a, bool bwd) {
    auto al = [](const void *q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
    if (a->D % 4) return false;
    if (!al(a->input) || !al(a->kernel) || !al(a->bias)) return false;
    if (!bwd) return al(a->output);
    return al(a->dy) && al(a->dinput);
}

unsigned grid_for(long total, int threads) {
    long blocks = (total + threads - 1) / threads;
    if (blocks > 148L * 64) blocks = 148L * 64;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

} // namespace

extern "C" int kmb_launch_convnd_fwd(const KmbConvND *a, cudaStream_t s) {
    ConvDev p;
    make_dev(a, &p);
    cudaError_t e;
    if (use_2d(p)) {
        if (aligned4(a, false) && p.D % (4 * R2_CG) == 0 && p.K <= R2_KMAX)
            e = dispatch2d_fwd_ring<float>(p, s);
        else
            e = aligned4(a, false) ? dispatch2d<4>(p, false, s) : dispatch2d<1>(p, false, s);
    } else if (use_3d(p) && aligned4(a, false) && p.P * p.D < (1L << 31)) {
        e = dispatch3d<float>(p, false, s);
    } else {
        k_convnd_fwd_generic<<<grid_for(p.batch * p.P * p.D, 256), 256, 0, s>>>(p);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return kmb_cuda_fail(e, "convnd forward launch");
    return KMB_OK;
}

extern "C" int kmb_launch_convnd_bwd(const KmbConvND *a, cudaStream_t s) {
    ConvDev p;
    make_dev(a, &p);
    cudaError_t e = cudaMemsetAsync(a->dkernel, 0, sizeof(float) * p.KV * p.D, s);
    if (e == cudaSuccess && a->dbias) e = cudaMemsetAsync(a->dbias, 0, sizeof(float) * p.D, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "convnd backward memset");
    if (use_2d(p)) {
        if (aligned4(a, true) && p.D % (4 * R2_CG) == 0 && p.K <= R2_KMAX)
            e = dispatch2d_bwd_ring<float>(p, s);
        else e = aligned4(a, true) ? dispatch2d<4>(p, true, s) : dispatch2d<1>(p, true, s);
    } else if (use_3d(p) && aligned4(a, true) && p.P * p.D < (1L << 31)) {
        e = dispatch3d<float>(p, true, s);
    } else {
        k_convnd_bwd_input_generic<<<grid_for(p.batch * p.P * p.D, 256), 256, 0, s>>>(p);
        e = cudaGetLastError();
        if (e == cudaSuccess) {
            long per = p.batch * p.P;
            unsigned bx = (unsigned)((per + 255) / 256);
            if (bx > 64) bx = 64;
            dim3 grid(bx, (unsigned)p.D, (unsigned)(p.KV + 1));
            k_convnd_bwd_param_generic<<<grid, 256, 0, s>>>(p);
            e = cudaGetLastError();
        }
    }
    if (e != cudaSuccess) return kmb_cuda_fail(e, "convnd backward launch");
    return KMB_OK;
}

/* bf16 activations (input, output, dy, dinput), fp32 taps, bias, dkernel
 * and dbias: the streamed 2D kernels (D a multiple of 64) and the 3D
 * kernels (D a multiple of 8), K <= 3, 16-byte aligned device tensors. */
extern "C" int kmb_convnd_bf16_supported(const KmbConvND *a, int bwd) {
    auto al = [](const void *q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
    if (a->K < 1 || a->K > 3 || !al(a->input) || !al(a->kernel) || !al(a->bias)) return 0;
    if (bwd ? !(al(a->dy) && al(a->dinput)) : !al(a->output)) return 0;
    long P = 1;
    for (long i = 0; i < a->ndims; ++i) P *= a->dims[i];
    if (a->ndims == 2) return a->D % 64 == 0; /* the streamed kernels' 64-channel tiles */
    if (a->ndims == 3) return a->D % 8 == 0 && P * a->D < (1L << 31);
    return 0;
}

extern "C" int kmb_launch_convnd_fwd_bf16(const KmbConvND *a, cudaStream_t s) {
    ConvDev p;
    make_dev(a, &p);
    const cudaError_t e = p.nd == 2 ? dispatch2d_fwd_ring<__nv_bfloat16>(p, s)
                                    : dispatch3d<__nv_bfloat16>(p, false, s);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "convnd bf16 forward launch");
}

extern "C" int kmb_launch_convnd_bwd_bf16(const KmbConvND *a, cudaStream_t s) {
    ConvDev p;
    make_dev(a, &p);
    cudaError_t e = cudaMemsetAsync(a->dkernel, 0, sizeof(float) * p.KV * p.D, s);
    if (e == cudaSuccess && a->dbias) e = cudaMemsetAsync(a->dbias, 0, sizeof(float) * p.D, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "convnd bf16 backward memset");
    e = p.nd == 2 ? dispatch2d_bwd_ring<__nv_bfloat16>(p, s)
                  : dispatch3d<__nv_bfloat16>(p, true, s);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "convnd bf16 backward launch");
}
