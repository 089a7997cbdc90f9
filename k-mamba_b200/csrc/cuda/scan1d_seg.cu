/*
 * 1D selective scan split along the sequence, for the channel-shared
 * layout of the headline configuration (B and C shared by all channels,
 * N = 16 states, D a multiple of 32), with fp32 or bf16 inputs and outputs.
 *
 * Recurrence and adjoint as in scan1d.cu (reference cpu/scan1d.asm:88-152,
 * cpu/scan1d_backward.c:248-295).  Lanes: 4 lanes per channel, 4 states per
 * lane, 32 channels per CTA of 128 threads.
 *
 * Parallelism over L.  The sequence is cut into S segments and every
 * (batch item, 32-channel group, segment) is a CTA, so a small batch still
 * fills the GPU.  A segment starts from an exact state only at the
 * sequence start; elsewhere it starts kBurnSteps steps earlier from a zero
 * state (the forward) or kBurnSteps steps later from a zero adjoint (the
 * backward) and lets that warm-up window absorb the unknown carry: the
 * carry's contribution to the segment's first state is scaled by the
 * product of the window's decays, exp(A sum dt), for every state.  A CTA
 * accepts its warm-up only when that product is at most 2^-40 for every
 * state it owns (sum over the window of dt A log2 e <= -40, accumulated
 * from the same w = dt A log2 e the decays use), and in the forward only
 * when no state reached the +-1000 clamp (the clamp makes the recurrence
 * nonlinear).  Otherwise it records a flag and writes nothing; a second
 * launch (the fixer, one CTA per batch item and channel group) then redoes
 * the flagged segments in order from the exact boundary states the
 * neighbouring segments left in `seg_state`, so the results are the exact
 * sequential recurrence in every case and the warm-up is only ever a
 * shortcut.  Flag codes: 1 = warm-up decay too weak, 2 = clamp reached
 * (forward; also redoes the next segment, whose warm-up crossed it).
 *
 * Outputs: forward y (T), the checkpoints every KMB_SCAN1D_CHUNK steps
 * (fp32, the backward's restart points), h_last; backward dx, ddt (T), dA,
 * and dB / dC channel sums accumulated in fp32 (the host converts them to
 * bf16 for bf16 outputs).
 */
#include <stdint.h>

#include <cuda_bf16.h>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kNT = 128;
constexpr int kP = 4;                 /* lanes per channel */
constexpr int kDT = kNT / kP;         /* channels per CTA */
constexpr int kN = 16;                /* states */
constexpr int kTT = 32;               /* forward tile (steps) */
constexpr int kST = 3;                /* forward pipeline stages */
constexpr int kCh = KMB_SCAN1D_CHUNK; /* backward chunk = checkpoint interval */
constexpr int kBurnSteps = 256;
constexpr float kBurnLog2 = -40.f;
constexpr unsigned kFull = 0xffffffffu;
/* State pairs per lane (of 2) whose decays the fast paths compute on the
 * FMA pipe (kmb_exp2_fma2) instead of MUFU ex2.  Off: both kernels are
 * bound by instruction issue, not by the 16-per-clock MUFU rate, and the
 * FMA-pipe exponential issues more instructions (one pair of two per lane
 * measured forward 0.503 -> 0.555 ms and backward 1.141 -> 1.206 ms at
 * config 2).  Kept as a build option for issue-light variants. */
#ifndef KMB_SEG_FMA_PAIRS_FWD
#define KMB_SEG_FMA_PAIRS_FWD 0
#endif
#ifndef KMB_SEG_FMA_PAIRS_BWD
#define KMB_SEG_FMA_PAIRS_BWD 0
#endif
constexpr int kFmaFwd = KMB_SEG_FMA_PAIRS_FWD, kFmaBwd = KMB_SEG_FMA_PAIRS_BWD;

/* Largest |A log2 e| over the lane's FMA-pipe state pairs, or +inf when
 * one of them is not finite (the range check then fails at once). */
template <int NP>
__device__ __forceinline__ float fma_pairs_amax(const float2 (&A2p)[2]) {
    float m = 0.f;
#pragma unroll
    for (int jp = 2 - NP; jp < 2; ++jp) {
        const float a = fabsf(A2p[jp].x), b = fabsf(A2p[jp].y);
        m = (a <= 3.0e38f && b <= 3.0e38f) ? fmaxf(m, fmaxf(a, b)) : __int_as_float(0x7f800000);
    }
    return m;
}

/* The decays of pair jp: FMA pipe for the last NP pairs, else MUFU ex2 with
 * the weak-decay polynomial. */
template <int NP>
__device__ __forceinline__ float2 decay_pair(float2 w, int jp) {
    return jp >= 2 - NP ? kmb_exp2_fma2(w) : kmb_exp2_decay2(w);
}

template <typename T> struct IO;
template <> struct IO<float> {
    static __device__ __forceinline__ float f(float v) { return v; }
    /* 4 consecutive values of a 16-byte aligned row */
    static __device__ __forceinline__ float4 f4(const float *r) {
        return *reinterpret_cast<const float4 *>(r);
    }
};
template <> struct IO<__nv_bfloat16> {
    static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ float4 f4(const __nv_bfloat16 *r) {
        const uint2 u = *reinterpret_cast<const uint2 *>(r);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
};

struct SegArgs {
    const void *x, *dt, *B, *C, *dy;
    const float *A, *h0, *ckpt_in;
    void *y, *dx, *ddt;
    float *dB, *dC, *dA;
    float *h_last, *ckpt;
    float *seg_state; /* [batch, S, D, N] */
    int *flag;        /* [batch, D / 32, S] */
    long L, D, nslots;
    int S, seg_len;   /* segments, steps per segment (a multiple of kTT) */
    int fix;          /* 0: segment launch, 1: fixer launch */
};

__device__ __forceinline__ float clamp1000(float v) { return fmaxf(fminf(v, 1000.f), -1000.f); }

/* Reduce-scatter of 4 values across the 4 lanes of a channel: lane
 * (lane & 3) receives the sum of value index (lane & 3). */
__device__ __forceinline__ float rs4(float (&v)[4], int lane) {
#pragma unroll
    for (int h = 2; h > 0; h >>= 1) {
        const bool up = (lane & h) != 0;
#pragma unroll
        for (int k = 0; k < h; ++k) {
            const float send = up ? v[k] : v[k + h];
            const float keep = up ? v[k + h] : v[k];
            v[k] = keep + __shfl_xor_sync(kFull, send, h);
        }
    }
    return v[0];
}

/* cp.async copy of `rows` x `cols` elements of T (cols * sizeof(T) a
 * multiple of 16) into a dense shared tile; rows past `rows_valid` are
 * zero-filled.  `ld` is the global row stride in elements. */
template <typename T, int ROWS, int COLS>
__device__ __forceinline__ void tile_copy(T *s, const T *g, long ld, int rows_valid, int tid) {
    constexpr int UPR = COLS * (int)sizeof(T) / 16; /* 16-byte units per row */
    constexpr int E = 16 / (int)sizeof(T);
#pragma unroll
    for (int u = tid; u < ROWS * UPR; u += kNT) {
        const int r = u / UPR, c = (u - r * UPR) * E;
        const bool ok = r < rows_valid;
        kmb_cp_async16(s + r * COLS + c, ok ? (const void *)(g + (long)r * ld + c) : (const void *)g,
                       ok ? 16 : 0);
    }
}

/* ------------------------------------------------------------------ */
/* forward                                                             */
/* ------------------------------------------------------------------ */

template <typename T>
struct FwdLayout {
    static constexpr int XS = kTT * kDT * (int)sizeof(T); /* x or dt tile [TT][DT] */
    static constexpr int BS = kTT * kN * (int)sizeof(T);  /* B or C rows [TT][N] */
    static constexpr int YS = kTT * kDT * 4;              /* y tile (fp32) */
    static constexpr int STAGE = 2 * XS + 2 * BS + YS;
    static constexpr int SMEM = kST * STAGE + 16;
};

/*
 * Runs the tiles [kb, ke) of one (batch item, channel group) starting from
 * state h; tiles before ko are warm-up (no outputs).  Returns 0, or a flag
 * code when `seg` (a segment launch) and the warm-up was rejected (1) or a
 * state reached the clamp (2).  With `check` the warm-up decays are tested
 * at tile ko; without it the warm-up (if any) started from an exact state.
 */
template <typename T, bool CLAMP>
__device__ __forceinline__ int fwd_run(const SegArgs &p, unsigned char *smem, int *sflag, long b,
                                       long d0, int kb, int ko, int ke, float (&h)[4],
                                       bool seg, bool check) {
    using LY = FwdLayout<T>;
    const int tid = threadIdx.x, lane = tid & 31, g = tid & 3, dl = tid >> 2, n0 = g * 4;
    const long D = p.D, L = p.L;
    const long d = d0 + dl;
    float2 A2p[2];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp)
        A2p[jp] = kmb_f2(__ldg(p.A + d * kN + n0 + 2 * jp) * KMB_LOG2E,
                         __ldg(p.A + d * kN + n0 + 2 * jp + 1) * KMB_LOG2E);
    const T *xg = static_cast<const T *>(p.x) + b * L * D + d0;
    const T *dg = static_cast<const T *>(p.dt) + b * L * D + d0;
    const T *Bg = static_cast<const T *>(p.B) + b * L * kN;
    const T *Cg = static_cast<const T *>(p.C) + b * L * kN;
    T *yg = static_cast<T *>(p.y);
    float *ck = p.ckpt ? p.ckpt + (b * p.nslots * D + d) * kN + n0 : nullptr;
    const float amaxF = fma_pairs_amax<kFmaFwd>(A2p);

    auto stage = [&](int k) { return smem + (k % kST) * LY::STAGE; };
    auto load = [&](int k) {
        unsigned char *st = stage(k);
        const long t0 = (long)k * kTT;
        const int rv = (int)min((long)kTT, L - t0);
        tile_copy<T, kTT, kDT>(reinterpret_cast<T *>(st), xg + t0 * D, D, rv, tid);
        tile_copy<T, kTT, kDT>(reinterpret_cast<T *>(st + LY::XS), dg + t0 * D, D, rv, tid);
        tile_copy<T, kTT, kN>(reinterpret_cast<T *>(st + 2 * LY::XS), Bg + t0 * kN, kN, rv, tid);
        tile_copy<T, kTT, kN>(reinterpret_cast<T *>(st + 2 * LY::XS + LY::BS), Cg + t0 * kN, kN,
                              rv, tid);
    };
    auto flush_y = [&](int k) {
        const float *ys = reinterpret_cast<const float *>(stage(k) + 2 * LY::XS + 2 * LY::BS);
        const long t0 = (long)k * kTT;
        const int rv = (int)min((long)kTT, L - t0);
        constexpr int E = 16 / (int)sizeof(T), UPR = kDT / E;
        for (int u = tid; u < rv * UPR; u += kNT) {
            const int r = u / UPR, c = (u - r * UPR) * E;
            T *dst = yg + (b * L + t0 + r) * D + d0 + c;
            if constexpr (sizeof(T) == 4) {
                *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(ys + r * kDT + c);
            } else {
                const float *src = ys + r * kDT + c;
                uint4 w;
                __nv_bfloat162 q0 = __floats2bfloat162_rn(src[0], src[1]);
                __nv_bfloat162 q1 = __floats2bfloat162_rn(src[2], src[3]);
                __nv_bfloat162 q2 = __floats2bfloat162_rn(src[4], src[5]);
                __nv_bfloat162 q3 = __floats2bfloat162_rn(src[6], src[7]);
                w.x = *reinterpret_cast<unsigned *>(&q0);
                w.y = *reinterpret_cast<unsigned *>(&q1);
                w.z = *reinterpret_cast<unsigned *>(&q2);
                w.w = *reinterpret_cast<unsigned *>(&q3);
                *reinterpret_cast<uint4 *>(dst) = w;
            }
        }
    };

#pragma unroll
    for (int k = kb; k < kb + kST - 1; ++k) {
        if (k < ke) load(k);
        kmb_cp_async_commit();
    }
    float2 wsum[2] = {kmb_f2s(0.f), kmb_f2s(0.f)};
    int status = 0;
    for (int k = kb; k < ke; ++k) {
        kmb_cp_async_wait<kST - 2>();
        __syncthreads();
        if (seg && *sflag) { /* a warp reached the clamp in the previous tile */
            status = 2;
            break;
        }
        if (k == ko && check) {
            /* the warm-up window's decays must bound the unknown carry */
            bool ok = true;
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) ok = ok && wsum[jp].x <= kBurnLog2 && wsum[jp].y <= kBurnLog2;
            if (!__syncthreads_and(ok)) {
                status = 1;
                break;
            }
        }
        if (k - 1 >= ko && yg) flush_y(k - 1);
        if (k + kST - 1 < ke) load(k + kST - 1);
        kmb_cp_async_commit();

        const unsigned char *st = stage(k);
        const T *xs = reinterpret_cast<const T *>(st) + dl;
        const T *ds = reinterpret_cast<const T *>(st + LY::XS) + dl;
        const T *bs = reinterpret_cast<const T *>(st + 2 * LY::XS) + n0;
        const T *cs = reinterpret_cast<const T *>(st + 2 * LY::XS + LY::BS) + n0;
        float *ys = reinterpret_cast<float *>(const_cast<unsigned char *>(st) + 2 * LY::XS +
                                              2 * LY::BS) + dl;
        const long t0 = (long)k * kTT;
        const int rv = (int)min((long)kTT, L - t0);
        const bool warm = k < ko;

        /* exact path: per-step clamp (partial tiles, replays) */
        auto exact_tile = [&](int rows) {
            for (int i = 0; i < rows; ++i) {
                const float dv = IO<T>::f(ds[i * kDT]);
                const float u = dv * IO<T>::f(xs[i * kDT]);
                const float4 b4 = IO<T>::f4(bs + i * kN);
                const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
                float cv[4] = {0.f, 0.f, 0.f, 0.f};
                if (!warm) {
                    const float4 c4 = IO<T>::f4(cs + i * kN);
                    cv[0] = c4.x; cv[1] = c4.y; cv[2] = c4.z; cv[3] = c4.w;
                }
                float yp = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float w = dv * (j & 1 ? A2p[j >> 1].y : A2p[j >> 1].x);
                    if (warm) {
                        if (j & 1) wsum[j >> 1].y += w;
                        else wsum[j >> 1].x += w;
                    }
                    float hn = fmaf(kmb_exp2_decay(w), h[j], bv[j] * u);
                    if (CLAMP) hn = clamp1000(hn);
                    h[j] = hn;
                    yp = fmaf(cv[j], hn, yp);
                }
                if (!warm) {
#pragma unroll
                    for (int o = 2; o > 0; o >>= 1) yp += __shfl_xor_sync(kFull, yp, o);
                    if (g == 0) ys[i * kDT] = yp;
                    if (((t0 + i + 1) % kCh) == 0 && ck)
                        *reinterpret_cast<float4 *>(ck + ((t0 + i) / kCh) * D * kN) =
                            make_float4(h[0], h[1], h[2], h[3]);
                }
            }
        };

        if (rv == kTT) {
            float hst[4] = {h[0], h[1], h[2], h[3]};
            const float2 wst[2] = {wsum[0], wsum[1]};
            float2 sq = kmb_f2s(0.f);
            float dmax = 0.f; /* max |dt| of the tile: bounds |w| of the FMA-pipe pairs */
#pragma unroll
            for (int i0 = 0; i0 < kTT; i0 += kP) {
                float yq[kP];
#pragma unroll
                for (int s4 = 0; s4 < kP; ++s4) {
                    const int i = i0 + s4;
                    const float dv = IO<T>::f(ds[i * kDT]);
                    if (kFmaFwd > 0) dmax = fmaxf(dmax, fabsf(dv));
                    const float2 dv2 = kmb_f2s(dv), u2 = kmb_f2s(dv * IO<T>::f(xs[i * kDT]));
                    const float4 b4 = IO<T>::f4(bs + i * kN);
                    const float2 bp[2] = {kmb_f2(b4.x, b4.y), kmb_f2(b4.z, b4.w)};
                    float2 w[2], a[2];
#pragma unroll
                    for (int jp = 0; jp < 2; ++jp) {
                        w[jp] = kmb_mul2(dv2, A2p[jp]);
                        a[jp] = decay_pair<kFmaFwd>(w[jp], jp);
                    }
                    float2 hn[2];
#pragma unroll
                    for (int jp = 0; jp < 2; ++jp) {
                        hn[jp] = kmb_fma2(a[jp], kmb_f2(h[2 * jp], h[2 * jp + 1]),
                                          kmb_mul2(bp[jp], u2));
                        if (CLAMP) sq = kmb_fma2(hn[jp], hn[jp], sq);
                        h[2 * jp] = hn[jp].x;
                        h[2 * jp + 1] = hn[jp].y;
                    }
                    if (warm) {
                        wsum[0] = kmb_add2(wsum[0], w[0]);
                        wsum[1] = kmb_add2(wsum[1], w[1]);
                        yq[s4] = 0.f;
                    } else {
                        const float4 c4 = IO<T>::f4(cs + i * kN);
                        float2 y2 = kmb_mul2(kmb_f2(c4.x, c4.y), hn[0]);
                        y2 = kmb_fma2(kmb_f2(c4.z, c4.w), hn[1], y2);
                        yq[s4] = y2.x + y2.y;
                        if ((i + 1) % kCh == 0 && ck)
                            *reinterpret_cast<float4 *>(ck + ((t0 + i) / kCh) * D * kN) =
                                make_float4(h[0], h[1], h[2], h[3]);
                    }
                }
                if (!warm) ys[(i0 + g) * kDT] = rs4(yq, lane);
            }
            /* replay the tile exactly (clamped, MUFU / polynomial decays)
             * when a state may have reached the clamp or a FMA-pipe decay
             * argument may have left its range */
            bool bad = false;
            if (CLAMP) bad = !(sq.x + sq.y < 1e6f);
            if (kFmaFwd > 0) bad = bad || !(dmax * amaxF <= KMB_EXP2_FMA_MAX);
            if ((CLAMP || kFmaFwd > 0) && __any_sync(kFull, bad)) {
                if (seg) {
                    *sflag = 1; /* the CTA stops at the next tile boundary */
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) h[j] = hst[j];
                    wsum[0] = wst[0];
                    wsum[1] = wst[1];
                    exact_tile(kTT);
                }
            }
        } else {
            exact_tile(rv);
        }
    }
    kmb_cp_async_wait<0>();
    __syncthreads();
    if (status == 0 && seg && *sflag) status = 2;
    if (status == 0 && ke - 1 >= ko && yg) flush_y(ke - 1);
    return status;
}

/* MINB CTAs per SM: 4 (128 registers) for grids of more than two waves of
 * 3, where it measured faster (config 2 at batch 8, 1152 CTAs: 0.503 ->
 * 0.489 ms); 3 (168 registers, more room for the tile's loads in flight)
 * for the smaller grids of small batches, where fewer resident warps make
 * the per-CTA latency count (batch 1, 384 CTAs: 0.130 ms with 3). */
template <typename T, bool CLAMP, int MINB>
__global__ void __launch_bounds__(kNT, MINB) k_scan1d_fwd_seg(SegArgs p) {
    extern __shared__ __align__(16) unsigned char smem[];
    int *sflag = reinterpret_cast<int *>(smem + kST * FwdLayout<T>::STAGE);
    const int tid = threadIdx.x, n0 = (tid & 3) * 4;
    const long b = blockIdx.y, dg = blockIdx.x, d0 = dg * kDT, d = d0 + (tid >> 2);
    const long D = p.D;
    const int ntiles = (int)((p.L + kTT - 1) / kTT);
    const int seg_tiles = p.seg_len / kTT;
    int *flags = p.flag + (b * (D / kDT) + dg) * p.S;
    auto state_at = [&](int s) { return p.seg_state + ((b * p.S + s) * D + d) * kN + n0; };
    auto finish = [&](int s, const float (&h)[4]) {
        *reinterpret_cast<float4 *>(state_at(s)) = make_float4(h[0], h[1], h[2], h[3]);
        if (s == p.S - 1 && p.h_last)
            *reinterpret_cast<float4 *>(p.h_last + (b * D + d) * kN + n0) =
                make_float4(h[0], h[1], h[2], h[3]);
    };
    auto initial = [&](float (&h)[4]) {
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = p.h0 ? p.h0[(b * D + d) * kN + n0 + j] : 0.f;
    };
    if (!p.fix) {
        const int s = blockIdx.z;
        const int ko = s * seg_tiles, ke = min(ko + seg_tiles, ntiles);
        const int kb = s == 0 ? 0 : max(0, ko - kBurnSteps / kTT);
        float h[4] = {0.f, 0.f, 0.f, 0.f};
        if (kb == 0) initial(h); /* the warm-up reaches the sequence start: exact */
        if (tid == 0) *sflag = 0;
        __syncthreads();
        const int st = fwd_run<T, CLAMP>(p, smem, sflag, b, d0, kb, ko, ke, h, true, kb > 0);
        if (tid == 0) flags[s] = st;
        if (st == 0) finish(s, h);
        return;
    }
    /* fixer: redo the flagged segments in order from exact boundary states */
    bool redo_next = false;
    for (int s = 0; s < p.S; ++s) {
        const int f = flags[s];
        const bool redo = f != 0 || redo_next;
        redo_next = (f & 2) != 0;
        if (!redo) continue;
        float h[4];
        if (s == 0) {
            initial(h);
        } else {
            const float4 v = *reinterpret_cast<const float4 *>(state_at(s - 1));
            h[0] = v.x; h[1] = v.y; h[2] = v.z; h[3] = v.w;
        }
        const int ko = s * seg_tiles, ke = min(ko + seg_tiles, ntiles);
        fwd_run<T, CLAMP>(p, smem, sflag, b, d0, ko, ko, ke, h, false, false);
        finish(s, h);
        __syncthreads();
    }
}

/* ------------------------------------------------------------------ */
/* backward                                                            */
/* ------------------------------------------------------------------ */

template <typename T>
struct BwdLayout {
    static constexpr int XS = kCh * kDT * (int)sizeof(T); /* x, dt, dy [T][DT] */
    static constexpr int BS = kCh * kN * (int)sizeof(T);  /* B, C [T][N] */
    static constexpr int CK = kDT * kN * 4;               /* chunk-start states (fp32) */
    static constexpr int STAGE = 3 * XS + 2 * BS + CK;
    static constexpr int PART = kCh * kDT * kN * 4;       /* dB or dC partials (fp32) */
    static constexpr int PX = kCh * kDT * kP * 8;         /* dx / ddt partials (float2) */
    static constexpr int SMEM = 2 * STAGE + 2 * PART + PX + 16;
};

/*
 * Reverse sweep of the chunks [cb, ct] (ct first) of one (batch item,
 * channel group) from adjoint carry g; chunks above ce - 1 are warm-up (no
 * outputs).  Returns 1 when `check` and the warm-up decays were too weak.
 */
template <typename T, bool CLAMP>
__device__ __forceinline__ int bwd_run(const SegArgs &p, unsigned char *smem, long b, long d0,
                                       int cb, int ce, int ct, float2 (&gcp)[2], bool check,
                                       float2 (&dAp)[2]) {
    using LY = BwdLayout<T>;
    const int tid = threadIdx.x, g = tid & 3, dl = tid >> 2, n0 = g * 4;
    const long D = p.D, L = p.L;
    const long d = d0 + dl;
    float *partB = reinterpret_cast<float *>(smem + 2 * LY::STAGE);
    float *partC = partB + kCh * kDT * kN;
    float2 *partX = reinterpret_cast<float2 *>(partC + kCh * kDT * kN);

    float2 A2p[2], Arp[2];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        const float a0 = __ldg(p.A + d * kN + n0 + 2 * jp), a1 = __ldg(p.A + d * kN + n0 + 2 * jp + 1);
        Arp[jp] = kmb_f2(a0, a1);
        A2p[jp] = kmb_f2(a0 * KMB_LOG2E, a1 * KMB_LOG2E);
    }
    const T *xg = static_cast<const T *>(p.x) + b * L * D + d0;
    const T *dtg = static_cast<const T *>(p.dt) + b * L * D + d0;
    const T *dyg = static_cast<const T *>(p.dy) + b * L * D + d0;
    const T *Bg = static_cast<const T *>(p.B) + b * L * kN;
    const T *Cg = static_cast<const T *>(p.C) + b * L * kN;

    auto load = [&](int c, int sidx) {
        unsigned char *st = smem + sidx * LY::STAGE;
        const long t0 = (long)c * kCh;
        const int rv = (int)min((long)kCh, L - t0);
        tile_copy<T, kCh, kDT>(reinterpret_cast<T *>(st), xg + t0 * D, D, rv, tid);
        tile_copy<T, kCh, kDT>(reinterpret_cast<T *>(st + LY::XS), dtg + t0 * D, D, rv, tid);
        tile_copy<T, kCh, kDT>(reinterpret_cast<T *>(st + 2 * LY::XS), dyg + t0 * D, D, rv, tid);
        tile_copy<T, kCh, kN>(reinterpret_cast<T *>(st + 3 * LY::XS), Bg + t0 * kN, kN, rv, tid);
        tile_copy<T, kCh, kN>(reinterpret_cast<T *>(st + 3 * LY::XS + LY::BS), Cg + t0 * kN, kN,
                              rv, tid);
        if (c > 0) /* the forward's checkpoint before chunk c: [DT][N] contiguous */
            tile_copy<float, kDT, kN>(
                reinterpret_cast<float *>(st + 3 * LY::XS + 2 * LY::BS),
                p.ckpt_in + ((b * p.nslots + c - 1) * D + d0) * kN, kN, kDT, tid);
    };

    float2 wsum[2] = {kmb_f2s(0.f), kmb_f2s(0.f)};
    const float amaxF = fma_pairs_amax<kFmaBwd>(A2p);
    load(ct, 0);
    kmb_cp_async_commit();
    int status = 0;
    const int xdd = tid % kDT;
    for (int c = ct, it = 0; c >= cb; --c, ++it) {
        kmb_cp_async_wait<0>();
        __syncthreads();
        const bool warm = c >= ce;
        if (!warm && c == ce - 1 && check) {
            bool ok = true;
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) ok = ok && wsum[jp].x <= kBurnLog2 && wsum[jp].y <= kBurnLog2;
            if (!__syncthreads_and(ok)) {
                status = 1;
                break;
            }
        }
        if (c > cb) load(c - 1, (it + 1) & 1);
        kmb_cp_async_commit();

        const unsigned char *st = smem + (it & 1) * LY::STAGE;
        const T *xs = reinterpret_cast<const T *>(st) + dl;
        const T *ds = reinterpret_cast<const T *>(st + LY::XS) + dl;
        const T *dys = reinterpret_cast<const T *>(st + 2 * LY::XS) + dl;
        const T *bs = reinterpret_cast<const T *>(st + 3 * LY::XS) + n0;
        const T *cs = reinterpret_cast<const T *>(st + 3 * LY::XS + LY::BS) + n0;
        const long t0 = (long)c * kCh;
        const int len = (int)min((long)kCh, L - t0);

        float2 hsp[2];
        if (c > 0) {
            const float4 v = *reinterpret_cast<const float4 *>(
                reinterpret_cast<const float *>(st + 3 * LY::XS + 2 * LY::BS) + dl * kN + n0);
            hsp[0] = kmb_f2(v.x, v.y);
            hsp[1] = kmb_f2(v.z, v.w);
        } else {
            float hs[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) hs[j] = p.h0 ? p.h0[(b * D + d) * kN + n0 + j] : 0.f;
            hsp[0] = kmb_f2(hs[0], hs[1]);
            hsp[1] = kmb_f2(hs[2], hs[3]);
        }

        /* recompute the chunk's states and decays (rows past L are zero:
         * identity steps with zero gradient terms) */
        float2 hr[kCh][2], ar[kCh][2];
        auto recompute = [&](auto exact_tag) {
            constexpr bool EXACT = decltype(exact_tag)::value;
            float2 hh[2] = {hsp[0], hsp[1]};
            float2 sq = kmb_f2s(0.f);
            float dmax = 0.f;
#pragma unroll
            for (int i = 0; i < kCh; ++i) {
                const float dv = IO<T>::f(ds[i * kDT]);
                if (!EXACT && kFmaBwd > 0) dmax = fmaxf(dmax, fabsf(dv));
                const float2 dv2 = kmb_f2s(dv), u2 = kmb_f2s(dv * IO<T>::f(xs[i * kDT]));
                const float4 b4 = IO<T>::f4(bs + i * kN);
                const float2 bp[2] = {kmb_f2(b4.x, b4.y), kmb_f2(b4.z, b4.w)};
#pragma unroll
                for (int jp = 0; jp < 2; ++jp) {
                    const float2 w = kmb_mul2(dv2, A2p[jp]);
                    if (warm && !EXACT) wsum[jp] = kmb_add2(wsum[jp], w);
                    const float2 a = EXACT ? kmb_exp2_decay2(w) : decay_pair<kFmaBwd>(w, jp);
                    float2 hn = kmb_fma2(a, hh[jp], kmb_mul2(bp[jp], u2));
                    if (EXACT && CLAMP) {
                        hn.x = clamp1000(hn.x);
                        hn.y = clamp1000(hn.y);
                    } else if (CLAMP) {
                        sq = kmb_fma2(hn, hn, sq);
                    }
                    hh[jp] = hn;
                    hr[i][jp] = hn;
                    ar[i][jp] = a;
                }
            }
            if (EXACT) return false;
            bool bad = CLAMP && !(sq.x + sq.y < 1e6f);
            if (kFmaBwd > 0) bad = bad || !(dmax * amaxF <= KMB_EXP2_FMA_MAX);
            return bad;
        };
        if (__any_sync(kFull, recompute(std::false_type{}))) recompute(std::true_type{});

        if (warm) {
            /* warm-up: only the adjoint carry moves */
#pragma unroll
            for (int i = kCh - 1; i >= 0; --i) {
                const float2 dyv2 = kmb_f2s(IO<T>::f(dys[i * kDT]));
                const float4 c4 = IO<T>::f4(cs + i * kN);
                const float2 cp[2] = {kmb_f2(c4.x, c4.y), kmb_f2(c4.z, c4.w)};
#pragma unroll
                for (int jp = 0; jp < 2; ++jp)
                    gcp[jp] = kmb_mul2(kmb_fma2(dyv2, cp[jp], gcp[jp]), ar[i][jp]);
            }
            continue;
        }

#pragma unroll
        for (int i = kCh - 1; i >= 0; --i) {
            const float xv = IO<T>::f(xs[i * kDT]);
            const float dv = IO<T>::f(ds[i * kDT]);
            const float dyv = IO<T>::f(dys[i * kDT]);
            const float2 dv2 = kmb_f2s(dv), dyv2 = kmb_f2s(dyv), u2 = kmb_f2s(dv * xv);
            const float4 b4 = IO<T>::f4(bs + i * kN);
            const float4 c4 = IO<T>::f4(cs + i * kN);
            const float2 bp[2] = {kmb_f2(b4.x, b4.y), kmb_f2(b4.z, b4.w)};
            const float2 cp[2] = {kmb_f2(c4.x, c4.y), kmb_f2(c4.z, c4.w)};
            float2 dxs2 = kmb_f2s(0.f), dts2 = kmb_f2s(0.f), vb[2], vc[2];
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) {
                const float2 hp = i > 0 ? hr[i > 0 ? i - 1 : 0][jp] : hsp[jp];
                const float2 ah = kmb_fma2(dyv2, cp[jp], gcp[jp]);
                const float2 q = kmb_mul2(ah, ar[i][jp]);
                const float2 qh = kmb_mul2(q, hp);
                dAp[jp] = kmb_fma2(dv2, qh, dAp[jp]);
                dts2 = kmb_fma2(Arp[jp], qh, dts2);
                dxs2 = kmb_fma2(ah, bp[jp], dxs2);
                vb[jp] = kmb_mul2(ah, u2);
                vc[jp] = kmb_mul2(dyv2, hr[i][jp]);
                gcp[jp] = q;
            }
            partX[(i * kDT + dl) * kP + g] = kmb_f2(dxs2.x + dxs2.y, dts2.x + dts2.y);
            const int o = (i * kDT + dl) * kN + n0;
            *reinterpret_cast<float4 *>(partB + o) = make_float4(vb[0].x, vb[0].y, vb[1].x, vb[1].y);
            *reinterpret_cast<float4 *>(partC + o) = make_float4(vc[0].x, vc[0].y, vc[1].x, vc[1].y);
        }
        __syncthreads();

        /* dx / ddt of the chunk: 2 outputs per thread, coalesced rows */
#pragma unroll
        for (int r = 0; r < kCh * kDT / kNT; ++r) {
            const int o = tid + r * kNT;
            const int i = o / kDT;
            const float2 *src = partX + o * kP;
            float2 sum = kmb_add2(kmb_add2(src[0], src[1]), kmb_add2(src[2], src[3]));
            if (i < len) {
                const long t = (b * L + t0 + i) * D + d0 + xdd;
                const float dtv = IO<T>::f(reinterpret_cast<const T *>(st + LY::XS)[o]);
                const float xv = IO<T>::f(reinterpret_cast<const T *>(st)[o]);
                const float dxv = sum.x * dtv, ddtv = fmaf(xv, sum.x, sum.y);
                if constexpr (sizeof(T) == 4) {
                    static_cast<float *>(p.dx)[t] = dxv;
                    static_cast<float *>(p.ddt)[t] = ddtv;
                } else {
                    static_cast<__nv_bfloat16 *>(p.dx)[t] = __float2bfloat16_rn(dxv);
                    static_cast<__nv_bfloat16 *>(p.ddt)[t] = __float2bfloat16_rn(ddtv);
                }
            }
        }
        /* dB / dC: channel sums of the chunk, 2 threads per 4-state output
         * (every other channel), folded by a shuffle; one 128-bit atomic
         * per output and CTA */
        {
            const int e = tid;             /* 2 arrays x 8 steps x 4 quads x 2 halves = 128 */
            const int o = e >> 1, hh = e & 1;
            const int arr = o / (kCh * 4), i = (o >> 2) % kCh, q = o & 3;
            const float *src = (arr ? partC : partB) + i * kDT * kN + q * 4;
            float2 lo = kmb_f2s(0.f), hi = kmb_f2s(0.f);
#pragma unroll
            for (int k = 0; k < kDT / 2; ++k) {
                const float4 t4 = *reinterpret_cast<const float4 *>(src + (2 * k + hh) * kN);
                lo = kmb_add2(lo, kmb_f2(t4.x, t4.y));
                hi = kmb_add2(hi, kmb_f2(t4.z, t4.w));
            }
            lo.x += __shfl_xor_sync(kFull, lo.x, 1);
            lo.y += __shfl_xor_sync(kFull, lo.y, 1);
            hi.x += __shfl_xor_sync(kFull, hi.x, 1);
            hi.y += __shfl_xor_sync(kFull, hi.y, 1);
            if (hh == 0 && i < len) {
                float *dst = (arr ? p.dC : p.dB) + (b * L + t0 + i) * kN + q * 4;
                atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(lo.x, lo.y, hi.x, hi.y));
            }
        }
    }
    kmb_cp_async_wait<0>();
    __syncthreads();
    return status;
}

template <typename T, bool CLAMP>
__global__ void __launch_bounds__(kNT, 3) k_scan1d_bwd_seg(SegArgs p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, n0 = (tid & 3) * 4;
    const long b = blockIdx.y, dg = blockIdx.x, d0 = dg * kDT, d = d0 + (tid >> 2);
    const long D = p.D;
    const int nch = (int)((p.L + kCh - 1) / kCh);
    const int seg_ch = p.seg_len / kCh;
    int *flags = p.flag + (b * (D / kDT) + dg) * p.S;
    auto state_at = [&](int s) { return p.seg_state + ((b * p.S + s) * D + d) * kN + n0; };
    float2 dAp[2] = {kmb_f2s(0.f), kmb_f2s(0.f)};
    bool any = false;
    if (!p.fix) {
        const int s = blockIdx.z;
        const int cb = s * seg_ch, ce = min(cb + seg_ch, nch);
        const int top = min(nch, ce + kBurnSteps / kCh); /* warm-up from the top down */
        float2 gcp[2] = {kmb_f2s(0.f), kmb_f2s(0.f)};
        const int st = bwd_run<T, CLAMP>(p, smem, b, d0, cb, ce, top - 1, gcp, top < nch, dAp);
        if (tid == 0) flags[s] = st;
        if (st == 0) {
            *reinterpret_cast<float4 *>(state_at(s)) = make_float4(gcp[0].x, gcp[0].y, gcp[1].x, gcp[1].y);
            any = true;
        }
    } else {
        for (int s = p.S - 1; s >= 0; --s) {
            if (!flags[s]) continue;
            float2 gcp[2] = {kmb_f2s(0.f), kmb_f2s(0.f)};
            if (s + 1 < p.S) {
                const float4 v = *reinterpret_cast<const float4 *>(state_at(s + 1));
                gcp[0] = kmb_f2(v.x, v.y);
                gcp[1] = kmb_f2(v.z, v.w);
            }
            const int cb = s * seg_ch, ce = min(cb + seg_ch, nch);
            bwd_run<T, CLAMP>(p, smem, b, d0, cb, ce, ce - 1, gcp, false, dAp);
            *reinterpret_cast<float4 *>(state_at(s)) = make_float4(gcp[0].x, gcp[0].y, gcp[1].x, gcp[1].y);
            any = true;
        }
    }
    if (any) {
        atomicAdd(p.dA + d * kN + n0 + 0, dAp[0].x);
        atomicAdd(p.dA + d * kN + n0 + 1, dAp[0].y);
        atomicAdd(p.dA + d * kN + n0 + 2, dAp[1].x);
        atomicAdd(p.dA + d * kN + n0 + 3, dAp[1].y);
    }
}

__global__ void k_exp2_fma_eval(const float *w, float *out, long n) {
    for (long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 2; i < n;
         i += (long)gridDim.x * blockDim.x * 2) {
        const float2 r = kmb_exp2_fma2(kmb_f2(w[i], i + 1 < n ? w[i + 1] : 0.f));
        out[i] = r.x;
        if (i + 1 < n) out[i + 1] = r.y;
    }
}

__global__ void k_f32_to_bf16(const float *src, __nv_bfloat16 *dst, long n) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

template <typename T>
int launch_fwd(const SegArgs &p, long batch, int clamp, cudaStream_t s) {
    const size_t smem = FwdLayout<T>::SMEM;
    const long ctas = (p.D / kDT) * batch * p.S;
    const bool big = ctas > 2L * 3 * 148;
    auto kern = big ? (clamp ? k_scan1d_fwd_seg<T, true, 4> : k_scan1d_fwd_seg<T, false, 4>)
                    : (clamp ? k_scan1d_fwd_seg<T, true, 3> : k_scan1d_fwd_seg<T, false, 3>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg forward smem");
    SegArgs q = p;
    q.fix = 0;
    kern<<<dim3((unsigned)(p.D / kDT), (unsigned)batch, (unsigned)p.S), kNT, smem, s>>>(q);
    if ((e = cudaGetLastError()) != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg forward");
    if (p.S > 1) {
        q.fix = 1;
        kern<<<dim3((unsigned)(p.D / kDT), (unsigned)batch, 1), kNT, smem, s>>>(q);
        if ((e = cudaGetLastError()) != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg forward fixer");
    }
    return KMB_OK;
}

template <typename T>
int launch_bwd(const SegArgs &p, long batch, int clamp, cudaStream_t s) {
    const size_t smem = BwdLayout<T>::SMEM;
    auto kern = clamp ? k_scan1d_bwd_seg<T, true> : k_scan1d_bwd_seg<T, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg backward smem");
    SegArgs q = p;
    q.fix = 0;
    kern<<<dim3((unsigned)(p.D / kDT), (unsigned)batch, (unsigned)p.S), kNT, smem, s>>>(q);
    if ((e = cudaGetLastError()) != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg backward");
    if (p.S > 1) {
        q.fix = 1;
        kern<<<dim3((unsigned)(p.D / kDT), (unsigned)batch, 1), kNT, smem, s>>>(q);
        if ((e = cudaGetLastError()) != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg backward fixer");
    }
    return KMB_OK;
}

SegArgs make_args(const KmbScan1D *a, int S, int seg_len, float *seg_state, int *flag) {
    SegArgs p;
    p.x = a->x; p.dt = a->dt; p.B = a->B; p.C = a->C; p.dy = a->dy;
    p.A = a->A; p.h0 = a->h0; p.ckpt_in = nullptr;
    p.y = a->y; p.dx = a->dx; p.ddt = a->ddt;
    p.dB = a->dB; p.dC = a->dC; p.dA = a->dA;
    p.h_last = a->h_last; p.ckpt = a->ckpt;
    p.seg_state = seg_state; p.flag = flag;
    p.L = a->L; p.D = a->D; p.nslots = (a->L + kCh - 1) / kCh;
    p.S = S; p.seg_len = seg_len; p.fix = 0;
    return p;
}

} // namespace

extern "C" int kmb_scan1d_seg_supported(const KmbScan1D *a, int elem_bytes) {
    auto al = [](const void *q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
    const int E = 16 / elem_bytes;
    return a->bc_shared && a->N == kN && a->D % kDT == 0 && a->D % E == 0 && !a->h_all &&
           a->L < (1L << 30) && al(a->x) && al(a->dt) && al(a->B) && al(a->C) && al(a->dy) &&
           al(a->y) && al(a->dx) && al(a->ddt) && al(a->dB) && al(a->dC) && al(a->h0) &&
           al(a->h_last) && al(a->ckpt) && al(a->A);
}

extern "C" int kmb_scan1d_seg_plan(long batch, long L, long D, int *S_out, int *seg_len_out) {
    /* enough CTAs for about two full waves of 3 per SM, segments of at
     * least 512 steps (the 256-step warm-up stays under half), at most 64 */
    const long groups = batch * (D / kDT);
    const long want = (2L * 3 * 148 + groups - 1) / groups;
    long S = want < 1 ? 1 : want;
    const long max_s = L / 512 > 1 ? L / 512 : 1;
    if (S > max_s) S = max_s;
    if (S > 64) S = 64;
    const char *env = getenv("KMB_SCAN1D_SEGMENTS");
    if (env && *env) {
        const long v = strtol(env, nullptr, 10);
        if (v >= 1 && v <= 64) S = v;
    }
    /* segment length: a multiple of the forward tile, covering L */
    const long tiles = (L + kTT - 1) / kTT;
    const long seg_tiles = (tiles + S - 1) / S;
    *seg_len_out = (int)(seg_tiles * kTT);
    *S_out = (int)((tiles + seg_tiles - 1) / seg_tiles);
    return KMB_OK;
}

extern "C" int kmb_launch_scan1d_fwd_seg(const KmbScan1D *a, int bf16, int S, int seg_len,
                                         float *seg_state, int *flag, cudaStream_t s) {
    const SegArgs p = make_args(a, S, seg_len, seg_state, flag);
    return bf16 ? launch_fwd<__nv_bfloat16>(p, a->batch, a->clamp, s)
                : launch_fwd<float>(p, a->batch, a->clamp, s);
}

extern "C" int kmb_launch_scan1d_bwd_seg(const KmbScan1D *a, const float *ckpt_in, int bf16,
                                         int S, int seg_len, float *seg_state, int *flag,
                                         float *dB32, float *dC32, cudaStream_t s) {
    SegArgs p = make_args(a, S, seg_len, seg_state, flag);
    p.ckpt_in = ckpt_in;
    p.dB = dB32;
    p.dC = dC32;
    const size_t nbc = sizeof(float) * (size_t)a->batch * a->L * kN;
    cudaError_t e = cudaMemsetAsync(a->dA, 0, sizeof(float) * a->D * kN, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dB32, 0, nbc, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dC32, 0, nbc, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d seg backward memset");
    int rc = bf16 ? launch_bwd<__nv_bfloat16>(p, a->batch, a->clamp, s)
                  : launch_bwd<float>(p, a->batch, a->clamp, s);
    if (rc || !bf16) return rc;
    const long n = a->batch * a->L * kN;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    k_f32_to_bf16<<<blocks, 256, 0, s>>>(dB32, static_cast<__nv_bfloat16 *>((void *)a->dB), n);
    k_f32_to_bf16<<<blocks, 256, 0, s>>>(dC32, static_cast<__nv_bfloat16 *>((void *)a->dC), n);
    e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "scan1d seg dB/dC conversion");
}

extern "C" int kmb_exp2_fma_eval(const float *w, float *out, long n) {
    if (!w || !out || n < 0) return kmb_fail(KMB_EINVAL, "exp2_fma_eval: bad arguments");
    if (n == 0) return KMB_OK;
    cudaStream_t s = kmb_stream();
    const long blocks = (n / 2 + 255) / 256 < 1024 ? (n / 2 + 255) / 256 + 1 : 1024;
    k_exp2_fma_eval<<<(unsigned)blocks, 256, 0, s>>>(w, out, n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && kmb_sync_enabled()) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "exp2_fma_eval");
}
