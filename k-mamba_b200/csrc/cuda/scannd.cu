/*
 * ND selective scan over a causal grid, forward and backward (sm_100a),
 * for the reference API (scan_nd.h, scan2d of scan.h) where the full state
 * history h [P,D,M] is an output.
 *
 * Semantics of the reference src/scan_nd.c:86-230 (theta = lambda = NULL):
 *   dt_bar(p,d) = mean_axis delta_axis(p,d)
 *   h(p,d,m)    = dt_bar B(p,d,m) x(p,d)
 *               + sum_axis exp(delta_axis(p,d) A_axis(d,m)) h(p - e_axis,d,m)
 *   y(p,d)      = sum_m C(p,d,m) h(p,d,m)
 *
 * One persistent CTA per (batch item, channel tile) walks every wavefront
 * level of the grid in order, with a CTA barrier between levels instead of
 * one launch per level: all chains of a channel tile live in one CTA, so
 * no grid-wide synchronisation is needed.  Points of a level come from the
 * KMWavefrontPlan (uploaded once per grid shape); predecessor offsets are
 * precomputed per point.  A thread always serves the same channel (items
 * are (point, channel) with the channel fastest and DTILE | 256), loops
 * over the M states in registers and reads predecessors' states back from
 * global memory (L2) after the barrier.
 *
 * Backward (no reference implementation; adjoint of the recurrence):
 *   G(p)      = C(p) dy(p) + sum_axis exp(delta_axis(p+e) A_axis) G(p+e)
 *   dC = dy h,  dB = G dt_bar x,  dx = sum_m G dt_bar B,
 *   ddelta_axis(p) = (sum_m G B x) / ndims + sum_m G h(p-e) A_axis e_axis(p)
 *   dA_axis   = sum_p G h(p-e) delta_axis(p) e_axis(p)
 * walked in reverse level order; G is kept in a [P,D,M] scratch buffer and
 * dA in shared memory per CTA.
 */
#include <type_traits>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxAxes = 8;

struct NDDev {
    const float *x, *B, *C, *dy;
    float *h, *y, *G;
    float *dx, *dB, *dC;
    float *dA[kMaxAxes];
    float *ddelta[kMaxAxes];
    const float *delta[kMaxAxes];
    const float *A[kMaxAxes];
    const int *lvl_start, *lvl_off, *prev, *next;
    const int *sprev, *snext; /* prev / next in level-slot order */
    long P, D, M;
    long x_bs;      /* batch stride of x, y, dx (P*D) */
    long dl_bs;     /* batch stride of every delta / ddelta axis */
    long bc_bs, bc_ps, bc_ds; /* B / C / dB / dC strides: batch, point, channel */
    long h_bs;      /* batch stride of h and G (P*D*M) */
    int nd, nlevels, dtile;
};

__global__ void __launch_bounds__(kThreads) k_scannd_fwd(NDDev p) {
    const long b = blockIdx.y;
    const long d0 = (long)blockIdx.x * p.dtile;
    const int dd = threadIdx.x % p.dtile;
    const long d = d0 + dd;
    const bool dok = d < p.D;
    const long D = p.D, M = p.M;
    const int nd = p.nd;
    const float *x = p.x + b * p.x_bs;
    float *h = p.h + b * p.h_bs;
    float *y = p.y + b * p.x_bs;
    const float *Bb = p.B + b * p.bc_bs;
    const float *Cb = p.C + b * p.bc_bs;
    const int per = kThreads / p.dtile; /* points handled concurrently */
    const int pi0 = threadIdx.x / p.dtile;

    for (int l = 0; l < p.nlevels; ++l) {
        const int s0 = p.lvl_start[l], s1 = p.lvl_start[l + 1];
        if (dok) {
            for (int s = s0 + pi0; s < s1; s += per) {
                const long pt = p.lvl_off[s];
                const float xv = x[pt * D + d];
                float dta[kMaxAxes];
                float dt_bar = 0.f;
                for (int a = 0; a < nd; ++a) {
                    dta[a] = p.delta[a][b * p.dl_bs + pt * D + d];
                    dt_bar += dta[a];
                }
                dt_bar /= (float)nd;
                int pv[kMaxAxes];
                for (int a = 0; a < nd; ++a) pv[a] = p.prev[pt * nd + a];
                const long bcb = pt * p.bc_ps + d * p.bc_ds;
                float yacc = 0.f;
                for (long m = 0; m < M; ++m) {
                    float hn = dt_bar * (Bb[bcb + m] * xv);
                    for (int a = 0; a < nd; ++a) {
                        if (pv[a] >= 0) {
                            const float e = kmb_exp2_decay(dta[a] * (p.A[a][d * M + m] * KMB_LOG2E));
                            hn = fmaf(e, h[((long)pv[a] * D + d) * M + m], hn);
                        }
                    }
                    h[(pt * D + d) * M + m] = hn;
                    yacc = fmaf(Cb[bcb + m], hn, yacc);
                }
                y[pt * D + d] = yacc;
            }
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kThreads) k_scannd_bwd(NDDev p) {
    extern __shared__ float sdA[]; /* [nd][dtile][M] */
    const long b = blockIdx.y;
    const long d0 = (long)blockIdx.x * p.dtile;
    const int dd = threadIdx.x % p.dtile;
    const long d = d0 + dd;
    const bool dok = d < p.D;
    const long D = p.D, M = p.M;
    const int nd = p.nd;
    const int nsm = nd * p.dtile * (int)M;
    for (int i = threadIdx.x; i < nsm; i += kThreads) sdA[i] = 0.f;
    __syncthreads();

    const float *x = p.x + b * p.x_bs;
    const float *dy = p.dy + b * p.x_bs;
    const float *h = p.h + b * p.h_bs;
    float *G = p.G + b * p.h_bs;
    float *dx = p.dx + b * p.x_bs;
    const float *Bb = p.B + b * p.bc_bs;
    const float *Cb = p.C + b * p.bc_bs;
    float *dBb = p.dB + b * p.bc_bs;
    float *dCb = p.dC + b * p.bc_bs;
    const bool shared_bc = p.bc_ds == 0;
    const int per = kThreads / p.dtile;
    const int pi0 = threadIdx.x / p.dtile;

    for (int l = p.nlevels - 1; l >= 0; --l) {
        const int s0 = p.lvl_start[l], s1 = p.lvl_start[l + 1];
        if (dok) {
            for (int s = s0 + pi0; s < s1; s += per) {
                const long pt = p.lvl_off[s];
                const float xv = x[pt * D + d];
                const float gy = dy[pt * D + d];
                float dta[kMaxAxes], dtn[kMaxAxes];
                int pv[kMaxAxes], nx[kMaxAxes];
                float dt_bar = 0.f;
                for (int a = 0; a < nd; ++a) {
                    dta[a] = p.delta[a][b * p.dl_bs + pt * D + d];
                    dt_bar += dta[a];
                    pv[a] = p.prev[pt * nd + a];
                    nx[a] = p.next[pt * nd + a];
                    dtn[a] = nx[a] >= 0 ? p.delta[a][b * p.dl_bs + (long)nx[a] * D + d] : 0.f;
                }
                dt_bar /= (float)nd;
                const long bcb = pt * p.bc_ps + d * p.bc_ds;
                float sx = 0.f, sbar = 0.f;
                float sdt[kMaxAxes];
                for (int a = 0; a < nd; ++a) sdt[a] = 0.f;
                for (long m = 0; m < M; ++m) {
                    const float bv = Bb[bcb + m];
                    float gg = Cb[bcb + m] * gy;
                    for (int a = 0; a < nd; ++a) {
                        if (nx[a] >= 0) {
                            const float e = kmb_exp2_decay(dtn[a] * (p.A[a][d * M + m] * KMB_LOG2E));
                            gg = fmaf(e, G[((long)nx[a] * D + d) * M + m], gg);
                        }
                    }
                    G[(pt * D + d) * M + m] = gg;
                    const float hv = h[(pt * D + d) * M + m];
                    if (shared_bc) {
                        atomicAdd(dCb + bcb + m, gy * hv);
                        atomicAdd(dBb + bcb + m, gg * dt_bar * xv);
                    } else {
                        dCb[bcb + m] = gy * hv;
                        dBb[bcb + m] = gg * dt_bar * xv;
                    }
                    sx = fmaf(gg * dt_bar, bv, sx);
                    sbar = fmaf(gg * bv, xv, sbar);
                    for (int a = 0; a < nd; ++a) {
                        if (pv[a] >= 0) {
                            const float aa = p.A[a][d * M + m];
                            const float e = kmb_exp2_decay(dta[a] * (aa * KMB_LOG2E));
                            const float gh = gg * h[((long)pv[a] * D + d) * M + m] * e;
                            atomicAdd(&sdA[(a * p.dtile + dd) * M + m], gh * dta[a]);
                            sdt[a] = fmaf(gh, aa, sdt[a]);
                        }
                    }
                }
                dx[pt * D + d] = sx;
                for (int a = 0; a < nd; ++a)
                    p.ddelta[a][b * p.dl_bs + pt * D + d] = sdt[a] + sbar / (float)nd;
            }
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < nsm; i += kThreads) {
        const int a = i / (p.dtile * (int)M);
        const int r = i - a * p.dtile * (int)M;
        const int ddi = r / (int)M;
        const long dg = d0 + ddi;
        if (dg < D) atomicAdd(p.dA[a] + dg * M + (r - ddi * (int)M), sdA[i]);
    }
}

/* ------------------------------------------------------------------ */
/* warp-per-point kernels (channel-shared B/C, M % 4 == 0 <= 16,        */
/* D % 8 == 0, 3 or 4 axes: the Mamba-ND volumes)                       */
/* ------------------------------------------------------------------ */

/*
 * A CTA owns one batch item and 8 channels and walks the levels in order
 * (the backward's adjoint sweep: in reverse) with one CTA barrier per
 * level, as above.  A warp
 * handles one point at a time: lane 4c + q holds channel c of the group
 * and states 4q .. 4q+3, so the predecessor states h(p - e_axis) of the
 * warp are one coalesced 512-byte row per axis, B / C rows are one float4
 * per lane, and the sums over states fold over the 4 lanes of a channel.
 * The level's points are spread over the warps; predecessors were written
 * by this CTA before the last barrier, so they are read with plain
 * (L2-coherent) loads.
 */
constexpr int kWCh = 8;      /* channels per CTA */
/* warps per CTA of the forward and points a warp keeps in flight:
 * measured on 64^3 x 256 channels: 8 warps x 4 points 23.8 ms, 16 x 2
 * 16.6 ms, 32 x 1 11.8 ms */
constexpr int kWWarpsF = 32;
constexpr unsigned kWFull = 0xffffffffu;
/* warps per CTA of the pipelined sweeps (k_scannd_fwd_p / adj_p), 64^3 x
 * 1024 forward ms: 16 warps 9.8, 20 9.5, 24 8.2, 32 8.9 (at 32 the
 * 64-register cap makes the compiler recompute values in the loop) */
constexpr int kPW = 24;


template <int ND>
__global__ void __launch_bounds__(kWWarpsF * 32) k_scannd_fwd_w(NDDev p) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long b = blockIdx.y;
    const long d = (long)blockIdx.x * kWCh + c;
    const unsigned Du = (unsigned)p.D, Mu = (unsigned)p.M;
    const bool qok = q * 4u < Mu;
    float2 A2[ND][2];
#pragma unroll
    for (int a = 0; a < ND; ++a)
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            const unsigned m = q * 4 + 2 * jp;
            A2[a][jp] = kmb_f2(m < Mu ? p.A[a][d * Mu + m] * KMB_LOG2E : 0.f,
                               m + 1 < Mu ? p.A[a][d * Mu + m + 1] * KMB_LOG2E : 0.f);
        }
    /* per-lane bases: a point pt is element pt * D of the [P, D] tensors
     * (32-bit, P * D < 2^31) and row pt of the [P, M] ones; states of
     * point pt are at hq + (pt * D) * M */
    const float *xq = p.x + b * p.x_bs + d;
    const float *Bq = p.B + b * p.bc_bs + q * 4;
    const float *Cq = p.C + b * p.bc_bs + q * 4;
    float *hq = p.h + b * p.h_bs + d * Mu + q * 4;
    float *yq = p.y + b * p.x_bs + d;
    const float *dq[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) dq[a] = p.delta[a] + b * p.dl_bs + d;
    const int *lvl_off = p.lvl_off, *sprev = p.sprev, *lvl_start = p.lvl_start;
    const int nlevels = p.nlevels;

    __shared__ int sidx[kWWarpsF][32][ND + 1];
    for (int l = 0; l < nlevels; ++l) {
        const int s0 = lvl_start[l], s1 = lvl_start[l + 1];
        /* the warp's slots of the level are s0 + w + kWWarpsF j: lane j loads
         * the point and predecessor indices of slot j of each batch of 32 at
         * once into the warp's shared slot, from which they are read back
         * point by point */
        for (int base = s0 + w; base < s1; base += kWWarpsF * 32) {
            const int sl = base + kWWarpsF * lane;
            if (sl < s1) {
                sidx[w][lane][0] = lvl_off[sl];
#pragma unroll
                for (int a = 0; a < ND; ++a) sidx[w][lane][1 + a] = sprev[sl * ND + a];
            }
            __syncwarp();
            const int cnt = min(32, (s1 - base + kWWarpsF - 1) / kWWarpsF);
            for (int j = 0; j < cnt; ++j) {
                const unsigned pt = (unsigned)sidx[w][j][0];
                const unsigned od = pt * Du;
                int pv[ND];
#pragma unroll
                for (int a = 0; a < ND; ++a) pv[a] = sidx[w][j][1 + a];
                const float xv = xq[od];
                float dta[ND];
                float4 B4 = make_float4(0.f, 0.f, 0.f, 0.f), C4 = B4, hp[ND];
#pragma unroll
                for (int a = 0; a < ND; ++a) dta[a] = dq[a][od];
                if (qok) {
                    B4 = *reinterpret_cast<const float4 *>(Bq + (size_t)pt * Mu);
                    C4 = *reinterpret_cast<const float4 *>(Cq + (size_t)pt * Mu);
                }
#pragma unroll
                for (int a = 0; a < ND; ++a)
                    if (pv[a] >= 0 && qok)
                        hp[a] = *reinterpret_cast<const float4 *>(
                            hq + (size_t)((unsigned)pv[a] * Du) * Mu);
                float dt_bar = 0.f;
#pragma unroll
                for (int a = 0; a < ND; ++a) dt_bar += dta[a];
                dt_bar /= (float)ND;
                /* dt_bar (B x), in the reference's association */
                const float2 u2 = kmb_f2s(dt_bar), x2 = kmb_f2s(xv);
                float2 hn[2] = {kmb_mul2(u2, kmb_mul2(kmb_f2(B4.x, B4.y), x2)),
                                kmb_mul2(u2, kmb_mul2(kmb_f2(B4.z, B4.w), x2))};
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    if (pv[a] >= 0 && qok) {
                        const float2 dv2 = kmb_f2s(dta[a]);
                        const float2 e0 = kmb_exp2_decay2(kmb_mul2(dv2, A2[a][0]));
                        const float2 e1 = kmb_exp2_decay2(kmb_mul2(dv2, A2[a][1]));
                        hn[0] = kmb_fma2(e0, kmb_f2(hp[a].x, hp[a].y), hn[0]);
                        hn[1] = kmb_fma2(e1, kmb_f2(hp[a].z, hp[a].w), hn[1]);
                    }
                }
                const float2 y2 = kmb_fma2(kmb_f2(C4.z, C4.w), hn[1],
                                           kmb_mul2(kmb_f2(C4.x, C4.y), hn[0]));
                float yv = y2.x + y2.y;
                yv += __shfl_xor_sync(kWFull, yv, 1);
                yv += __shfl_xor_sync(kWFull, yv, 2);
                if (qok)
                    *reinterpret_cast<float4 *>(hq + (size_t)od * Mu) =
                        make_float4(hn[0].x, hn[0].y, hn[1].x, hn[1].y);
                if (q == 0) yq[od] = yv;
            }
            __syncwarp(); /* the slot is rewritten by the next batch */
        }
        __syncthreads();
    }
}

/* Smallest |A log2 e| over a lane's 4 states of one axis.  |delta| times
 * it bounds the lane's decay exponents |delta A log2 e| from below
 * (products round monotonically), so a bound >= KMB_DECAY_POLY_MAX means
 * kmb_exp2_decay2 returns the MUFU values for every state. */
__device__ __forceinline__ float lane_amin(const float2 (&A2)[2]) {
    return fminf(fminf(fabsf(A2[0].x), fabsf(A2[0].y)), fminf(fabsf(A2[1].x), fabsf(A2[1].y)));
}

/* k_scannd_fwd_w with each warp's loads pipelined, for M = 16.  After a
 * level's barrier the inputs of all its points and their predecessors'
 * states are in memory, so a warp streams its points of the level
 * through a ring of S point slots in shared memory (cp.async): the
 * predecessor rows (kWCh x 16 states), and x, delta, B and C of point j +
 * S - 1 are in flight while point j is computed from its slot.  Per
 * channel, the point's deltas and x sit side by side in the slot (one
 * 4-byte copy per lane, one 16-byte read per lane). */
template <int ND>
struct FwdPSlot {
    static constexpr int XW = ND + 1 <= 4 ? 4 : 8; /* floats per channel: delta_a, then x */
    static constexpr int HP = 0;                    /* [ND][128] predecessor rows */
    static constexpr int DX = ND * kWCh * 16;       /* [8][XW] */
    static constexpr int B = DX + kWCh * XW;        /* [16] */
    static constexpr int C = B + 16;                /* [16] */
    static constexpr int SIZE = C + 16;             /* floats, a multiple of 4 */
    static constexpr int NJ = (kWCh * (ND + 1) + 31) / 32; /* 4-byte copies a lane */
    static_assert(SIZE % 4 == 0, "slot layout");
};

/* the index row (point, then one neighbour per axis) of slot j */
template <int ND>
__device__ __forceinline__ void load_idx(const int (&row)[ND + 1], int (&ix)[ND + 1]) {
    if constexpr (ND == 3) {
        const int4 t = *reinterpret_cast<const int4 *>(row);
        ix[0] = t.x;
        ix[1] = t.y;
        ix[2] = t.z;
        ix[3] = t.w;
    } else {
#pragma unroll
        for (int i = 0; i <= ND; ++i) ix[i] = row[i];
    }
}

template <int ND, int S>
__global__ void __launch_bounds__(kPW * 32) k_scannd_fwd_p(NDDev p) {
    using L = FwdPSlot<ND>;
    constexpr float kInvND = 1.0f / ND;
    extern __shared__ __align__(16) float fsm[];
    __shared__ __align__(16) int sidx[kPW][32][ND + 1];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long b = blockIdx.y;
    const long d0 = (long)blockIdx.x * kWCh;
    const long d = d0 + c;
    const unsigned Du = (unsigned)p.D;
    float2 A2[ND][2];
#pragma unroll
    for (int a = 0; a < ND; ++a)
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            const float *ap = p.A[a] + d * 16 + q * 4 + 2 * jp;
            A2[a][jp] = kmb_f2(ap[0] * KMB_LOG2E, ap[1] * KMB_LOG2E);
        }
    float amin[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) amin[a] = lane_amin(A2[a]);
    float *wb = fsm + w * S * L::SIZE; /* this warp's ring of S slots */
    const unsigned wbs = (unsigned)__cvta_generic_to_shared(wb);
    const float *hg = p.h + b * p.h_bs + d0 * 16 + lane * 4; /* + point * D * 16 */
    float *hq = p.h + b * p.h_bs + d0 * 16 + lane * 4;
    float *yq = p.y + b * p.x_bs + d;
    /* this lane's 4-byte copies: value v of channel ch (delta_v, x for v = ND) */
    const float *vsrc[L::NJ];
    int vdst[L::NJ];
    bool vok[L::NJ];
#pragma unroll
    for (int i = 0; i < L::NJ; ++i) {
        const int e = lane + 32 * i, v = e / kWCh, ch = e % kWCh;
        vok[i] = v <= ND;
        const float *src = p.x + b * p.x_bs;
#pragma unroll
        for (int a = 0; a < ND; ++a)
            if (v == a) src = p.delta[a] + b * p.dl_bs;
        vsrc[i] = src + d0 + ch;
        vdst[i] = L::DX + ch * L::XW + v;
    }
    /* B (lanes 0-3) and C (lanes 4-7): one 16-byte chunk each */
    const float *bcsrc = (lane < 4 ? p.B : p.C) + b * p.bc_bs + (lane & 3) * 4;
    const int bcdst = (lane < 4 ? L::B : L::C) + (lane & 3) * 4;
    const int *lvl_off = p.lvl_off, *sprev = p.sprev, *lvl_start = p.lvl_start;
    const int nlevels = p.nlevels;

    for (int l = 0; l < nlevels; ++l) {
        const int s0 = lvl_start[l], s1 = lvl_start[l + 1];
        for (int base = s0 + w; base < s1; base += kPW * 32) {
            const int sl = base + kPW * lane;
            if (sl < s1) { /* the point; predecessors as element offsets (index x D,
                            * < 2^31) or -1 */
                sidx[w][lane][0] = lvl_off[sl];
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    const int pv = sprev[sl * ND + a];
                    sidx[w][lane][1 + a] = pv >= 0 ? pv * (int)Du : -1;
                }
            }
            __syncwarp();
            const int cnt = min(32, (s1 - base + kPW - 1) / kPW);
            auto issue = [&](int j, int slot) {
                const unsigned bs = wbs + slot * (L::SIZE * 4); /* shared address of the slot */
                int ix[ND + 1];
                load_idx<ND>(sidx[w][j], ix);
                /* a missing predecessor's row is zero-filled: it adds exactly 0 */
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    const bool ok = ix[1 + a] >= 0;
                    kmb_cp_async16_s(bs + (L::HP + a * kWCh * 16 + lane * 4) * 4,
                                     hg + (size_t)(unsigned)(ok ? ix[1 + a] : 0) * 16,
                                     ok ? 16 : 0);
                }
                const unsigned od = (unsigned)ix[0] * Du;
#pragma unroll
                for (int i = 0; i < L::NJ; ++i)
                    if (vok[i]) kmb_cp_async4_s(bs + vdst[i] * 4, vsrc[i] + od, 4);
                if (lane < 8) kmb_cp_async16_s(bs + bcdst * 4, bcsrc + (unsigned)ix[0] * 16, 16);
            };
            int si = 0, sc = 0; /* ring slots of the next issue and of the next compute */
#pragma unroll
            for (int j = 0; j < S - 1; ++j) {
                if (j < cnt) {
                    issue(j, si);
                    si = si + 1 == S ? 0 : si + 1;
                }
                kmb_cp_async_commit();
            }
            for (int j = 0; j < cnt; ++j) {
                if (j + S - 1 < cnt) {
                    issue(j + S - 1, si);
                    si = si + 1 == S ? 0 : si + 1;
                }
                kmb_cp_async_commit();
                kmb_cp_async_wait<S - 1>();
                __syncwarp();
                const float *bf = wb + sc * L::SIZE;
                sc = sc + 1 == S ? 0 : sc + 1;
                int ix[ND + 1];
                load_idx<ND>(sidx[w][j], ix);
                const unsigned od = (unsigned)ix[0] * Du;
                float dx[L::XW];
#pragma unroll
                for (int i = 0; i < L::XW; i += 4)
                    *reinterpret_cast<float4 *>(dx + i) =
                        *reinterpret_cast<const float4 *>(bf + L::DX + c * L::XW + i);
                bool weak = false;
                float dt_bar = 0.f;
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    dt_bar += dx[a];
                    weak |= fabsf(dx[a]) * amin[a] < KMB_DECAY_POLY_MAX;
                }
                dt_bar *= kInvND;
                /* MUFU only where no lane of the warp needs the polynomial */
                const bool fast = !__any_sync(kWFull, weak);
                const float4 B4 = *reinterpret_cast<const float4 *>(bf + L::B + q * 4);
                const float4 C4 = *reinterpret_cast<const float4 *>(bf + L::C + q * 4);
                /* dt_bar (B x), in the reference's association */
                const float2 u2 = kmb_f2s(dt_bar), x2 = kmb_f2s(dx[ND]);
                float2 hn[2] = {kmb_mul2(u2, kmb_mul2(kmb_f2(B4.x, B4.y), x2)),
                                kmb_mul2(u2, kmb_mul2(kmb_f2(B4.z, B4.w), x2))};
                auto carry = [&](auto fast_tag) {
                    constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
                    for (int a = 0; a < ND; ++a) { /* zero rows for missing predecessors */
                        const float4 hp = *reinterpret_cast<const float4 *>(
                            bf + L::HP + a * kWCh * 16 + lane * 4);
                        const float2 dv2 = kmb_f2s(dx[a]);
                        const float2 w0 = kmb_mul2(dv2, A2[a][0]);
                        const float2 w1 = kmb_mul2(dv2, A2[a][1]);
                        const float2 e0 = FAST ? kmb_ex2_2(w0) : kmb_exp2_decay2(w0);
                        const float2 e1 = FAST ? kmb_ex2_2(w1) : kmb_exp2_decay2(w1);
                        hn[0] = kmb_fma2(e0, kmb_f2(hp.x, hp.y), hn[0]);
                        hn[1] = kmb_fma2(e1, kmb_f2(hp.z, hp.w), hn[1]);
                    }
                };
                if (fast)
                    carry(std::true_type{});
                else
                    carry(std::false_type{});
                const float2 y2 = kmb_fma2(kmb_f2(C4.z, C4.w), hn[1],
                                           kmb_mul2(kmb_f2(C4.x, C4.y), hn[0]));
                float yv = y2.x + y2.y;
                yv += __shfl_xor_sync(kWFull, yv, 1);
                yv += __shfl_xor_sync(kWFull, yv, 2);
                *reinterpret_cast<float4 *>(hq + (size_t)od * 16) =
                    make_float4(hn[0].x, hn[0].y, hn[1].x, hn[1].y);
                if (q == 0) yq[od] = yv;
                __syncwarp(); /* the slot is refilled next */
            }
        }
        __syncthreads();
    }
}

/* ring depth of k_scannd_fwd_p within 227 KB of shared memory */
template <int ND>
constexpr int fwd_p_stages() {
    return (size_t)kPW * 3 * FwdPSlot<ND>::SIZE * 4 + kPW * 32 * (ND + 1) * 4 <=
                   227 * 1024
               ? 3
               : 2;
}

/* Reduce-scatter of 8 values over the 8 lanes that share q (lane bits
 * 2-4): afterwards lane 4c + q holds the sum of value 4 (c >> 2) + (c & 3). */
__device__ __forceinline__ float rs8_ch(float (&v)[8], int lane) {
#pragma unroll
    for (int o = 16, half = 4; o >= 4; o >>= 1, half >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (k < half) {
                const float send = up ? v[k] : v[k + half];
                const float keep = up ? v[k + half] : v[k];
                v[k] = keep + __shfl_xor_sync(kWFull, send, o);
            }
        }
    }
    return v[0];
}

/* The backward in two passes.  (A) An adjoint sweep (k_scannd_adj_p for
 * M = 16, k_scannd_adj_w otherwise) walks the levels in reverse and only
 * carries the adjoint
 *   G(p) = C dy + sum_axis e_axis(p+e) G(p+e)
 * into the scratch G (few registers, many warps per CTA).  (B) The
 * gradient pass (k_scannd_grad_s, or k_scannd_grad_w) then has no
 * dependency between points and runs over all of them in parallel: per
 * point
 *   dC += dy h,  dB += G dt_bar x  (folded over the 8 channels, one
 *   128-bit atomic per point, state quad and array),
 *   dx = sum_m (G dt_bar) B,  ddelta_axis = sum_m (G h(p-e)) e A_axis
 *   + sum_m (G B) x / ndims,  dA_axis += (G h(p-e)) e delta_axis,
 * with dA folded per CTA in shared memory (the adjoint of the generic
 * backward above, same per-state terms). */
constexpr int kWWarpsA = 32;

template <int ND>
__global__ void __launch_bounds__(kWWarpsA * 32) k_scannd_adj_w(NDDev p) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long b = blockIdx.y;
    const long d = (long)blockIdx.x * kWCh + c;
    const unsigned Du = (unsigned)p.D, Mu = (unsigned)p.M;
    const bool qok = q * 4u < Mu;
    float2 A2[ND][2];
#pragma unroll
    for (int a = 0; a < ND; ++a)
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            const unsigned m = q * 4 + 2 * jp;
            A2[a][jp] = kmb_f2(m < Mu ? p.A[a][d * Mu + m] * KMB_LOG2E : 0.f,
                               m + 1 < Mu ? p.A[a][d * Mu + m + 1] * KMB_LOG2E : 0.f);
        }
    const float *dyq = p.dy + b * p.x_bs + d;
    const float *Cq = p.C + b * p.bc_bs + q * 4;
    float *Gq = p.G + b * p.h_bs + d * Mu + q * 4;
    const float *dq[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) dq[a] = p.delta[a] + b * p.dl_bs + d;
    const int *lvl_off = p.lvl_off, *snext = p.snext, *lvl_start = p.lvl_start;

    for (int l = p.nlevels - 1; l >= 0; --l) {
        const int s0 = lvl_start[l], s1 = lvl_start[l + 1];
        /* indices of 32 of the warp's slots loaded at once and handed out
         * by shuffle (k_scannd_fwd_w hands them out through a shared slot) */
        for (int base = s0 + w; base < s1; base += kWWarpsA * 32) {
            const int sl = base + kWWarpsA * lane;
            int myoff = 0, mynx[ND];
#pragma unroll
            for (int a = 0; a < ND; ++a) mynx[a] = -1;
            if (sl < s1) {
                myoff = lvl_off[sl];
#pragma unroll
                for (int a = 0; a < ND; ++a) mynx[a] = snext[sl * ND + a];
            }
            const int cnt = min(32, (s1 - base + kWWarpsA - 1) / kWWarpsA);
            for (int j = 0; j < cnt; ++j) {
                const unsigned pt = (unsigned)__shfl_sync(kWFull, myoff, j);
                const unsigned od = pt * Du;
                int nx[ND];
#pragma unroll
                for (int a = 0; a < ND; ++a) nx[a] = __shfl_sync(kWFull, mynx[a], j);
                const float gy = dyq[od];
                float4 C4 = make_float4(0.f, 0.f, 0.f, 0.f), gn[ND];
                float dtn[ND];
                if (qok) C4 = *reinterpret_cast<const float4 *>(Cq + (size_t)pt * Mu);
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    const unsigned on = (unsigned)nx[a] * Du;
                    dtn[a] = nx[a] >= 0 ? dq[a][on] : 0.f;
                    if (nx[a] >= 0 && qok)
                        gn[a] = *reinterpret_cast<const float4 *>(Gq + (size_t)on * Mu);
                }
                const float2 gy2 = kmb_f2s(gy);
                float2 gg[2] = {kmb_mul2(kmb_f2(C4.x, C4.y), gy2), kmb_mul2(kmb_f2(C4.z, C4.w), gy2)};
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    if (nx[a] >= 0 && qok) {
                        const float2 dn2 = kmb_f2s(dtn[a]);
                        const float2 e0 = kmb_exp2_decay2(kmb_mul2(dn2, A2[a][0]));
                        const float2 e1 = kmb_exp2_decay2(kmb_mul2(dn2, A2[a][1]));
                        gg[0] = kmb_fma2(e0, kmb_f2(gn[a].x, gn[a].y), gg[0]);
                        gg[1] = kmb_fma2(e1, kmb_f2(gn[a].z, gn[a].w), gg[1]);
                    }
                }
                if (qok)
                    *reinterpret_cast<float4 *>(Gq + (size_t)od * Mu) =
                        make_float4(gg[0].x, gg[0].y, gg[1].x, gg[1].y);
            }
        }
        __syncthreads();
    }
}

/* Gradient terms of one point for the two-pass backward below: lane
 * 4c + q holds channel c and states 4q .. 4q+3 of the point's G, h and B,
 * the predecessor states hp[a] (used where pv[a] >= 0), and the point's
 * x, dy and per-axis delta.  Writes dx (dxp) and ddelta (ddq[a] + od),
 * adds the point's dB / dC (rows dBrow / dCrow, folded over the warp's 8
 * channels: one 128-bit atomic per state quad) and accumulates dA in dAp. */
template <int ND>
__device__ __forceinline__ void grad_point(
    const float4 &B4, const float4 &H4, const float4 &G4, const float4 (&hp)[ND],
    const int (&pv)[ND], float xv, float gy, const float (&dta)[ND],
    const float2 (&A2)[ND][2], const float2 (&Ar)[ND][2], float2 (&dAp)[ND][2], bool qok,
    int lane, int c, int q, float *dxp, float *const (&ddq)[ND], long od, float *dBrow,
    float *dCrow) {
    float dt_bar = 0.f;
#pragma unroll
    for (int a = 0; a < ND; ++a) dt_bar += dta[a];
    dt_bar /= (float)ND;
    const float2 gg[2] = {kmb_f2(G4.x, G4.y), kmb_f2(G4.z, G4.w)};
    const float2 Bp[2] = {kmb_f2(B4.x, B4.y), kmb_f2(B4.z, B4.w)};
    const float2 gy2 = kmb_f2s(gy), dtb2 = kmb_f2s(dt_bar), xv2 = kmb_f2s(xv);
    float2 sx2 = kmb_f2s(0.f), sb2 = kmb_f2s(0.f), sdt2[ND];
    float v8[8];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        sx2 = kmb_fma2(kmb_mul2(gg[jp], dtb2), Bp[jp], sx2);
        sb2 = kmb_fma2(kmb_mul2(gg[jp], Bp[jp]), xv2, sb2);
        const float2 vb = kmb_mul2(kmb_mul2(gg[jp], dtb2), xv2); /* dB */
        const float2 vc = kmb_mul2(gy2, jp ? kmb_f2(H4.z, H4.w) : kmb_f2(H4.x, H4.y));
        v8[2 * jp] = vb.x;
        v8[2 * jp + 1] = vb.y;
        v8[4 + 2 * jp] = vc.x;
        v8[4 + 2 * jp + 1] = vc.y;
    }
#pragma unroll
    for (int a = 0; a < ND; ++a) {
        sdt2[a] = kmb_f2s(0.f);
        if (pv[a] >= 0 && qok) {
            const float2 dv2 = kmb_f2s(dta[a]);
            const float2 hpp[2] = {kmb_f2(hp[a].x, hp[a].y), kmb_f2(hp[a].z, hp[a].w)};
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) {
                const float2 e = kmb_exp2_decay2(kmb_mul2(dv2, A2[a][jp]));
                const float2 gh = kmb_mul2(kmb_mul2(gg[jp], hpp[jp]), e);
                dAp[a][jp] = kmb_fma2(gh, dv2, dAp[a][jp]);
                sdt2[a] = kmb_fma2(gh, Ar[a][jp], sdt2[a]);
            }
        }
    }
    /* sums over the 16 states (the 4 lanes of a channel) */
    float sx = sx2.x + sx2.y, sbv = sb2.x + sb2.y, sdt[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) sdt[a] = sdt2[a].x + sdt2[a].y;
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        sx += __shfl_xor_sync(kWFull, sx, o);
        sbv += __shfl_xor_sync(kWFull, sbv, o);
#pragma unroll
        for (int a = 0; a < ND; ++a) sdt[a] += __shfl_xor_sync(kWFull, sdt[a], o);
    }
    if (q == 0) {
        dxp[0] = sx;
#pragma unroll
        for (int a = 0; a < ND; ++a) ddq[a][od] = sdt[a] + sbv / (float)ND;
    }
    /* dB / dC: sums over the 8 channels, then 4 states into one lane */
    const float r1 = rs8_ch(v8, lane);
    const float r2 = __shfl_down_sync(kWFull, r1, 4);
    const float r3 = __shfl_down_sync(kWFull, r1, 8);
    const float r4 = __shfl_down_sync(kWFull, r1, 12);
    if ((c & 3) == 0 && qok) {
        float *dst = ((c >> 2) ? dCrow : dBrow) + q * 4;
        atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(r1, r2, r3, r4));
    }
}

/* k_scannd_adj_w with each warp's loads pipelined through a ring of S
 * point slots (cp.async), for M = 16: the successors' adjoint rows G(p +
 * e_axis) and deltas delta_axis(p + e_axis), and the point's dy and C, of
 * point j + S - 1 are in flight while point j is computed.  Per channel
 * the successors' deltas and dy sit side by side in the slot. */
template <int ND>
struct AdjPSlot {
    static constexpr int XW = ND + 1 <= 4 ? 4 : 8; /* floats per channel: delta_a, then dy */
    static constexpr int GN = 0;                    /* [ND][128] successor rows */
    static constexpr int DD = ND * kWCh * 16;       /* [8][XW] */
    static constexpr int C = DD + kWCh * XW;        /* [16] */
    static constexpr int SIZE = C + 16;
    static constexpr int NJ = (kWCh * (ND + 1) + 31) / 32;
    static_assert(SIZE % 4 == 0, "slot layout");
};

template <int ND, int S>
__global__ void __launch_bounds__(kPW * 32) k_scannd_adj_p(NDDev p) {
    using L = AdjPSlot<ND>;
    extern __shared__ __align__(16) float asm_[];
    __shared__ __align__(16) int sidx[kPW][32][ND + 1];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long b = blockIdx.y;
    const long d0 = (long)blockIdx.x * kWCh;
    const unsigned Du = (unsigned)p.D;
    float2 A2[ND][2];
#pragma unroll
    for (int a = 0; a < ND; ++a)
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            const float *ap = p.A[a] + (d0 + c) * 16 + q * 4 + 2 * jp;
            A2[a][jp] = kmb_f2(ap[0] * KMB_LOG2E, ap[1] * KMB_LOG2E);
        }
    float amin[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) amin[a] = lane_amin(A2[a]);
    float *wb = asm_ + w * S * L::SIZE;
    const unsigned wbs = (unsigned)__cvta_generic_to_shared(wb);
    const float *gg_src = p.G + b * p.h_bs + d0 * 16 + lane * 4; /* + point * D * 16 */
    float *gq = p.G + b * p.h_bs + d0 * 16 + lane * 4;
    /* this lane's 4-byte copies: value v of channel ch: delta_v of the
     * successor along axis v, or dy of the point (v = ND); vrow indexes
     * the slot's index row (1 + v, or 0 for the point itself) */
    const float *vsrc[L::NJ];
    int vdst[L::NJ], vrow[L::NJ];
    unsigned vmul[L::NJ]; /* D for dy (the slot holds the point index), 1 for the deltas */
    bool vok[L::NJ];
#pragma unroll
    for (int i = 0; i < L::NJ; ++i) {
        const int e = lane + 32 * i, v = e / kWCh, ch = e % kWCh;
        vok[i] = v <= ND;
        const float *src = p.dy + b * p.x_bs;
#pragma unroll
        for (int a = 0; a < ND; ++a)
            if (v == a) src = p.delta[a] + b * p.dl_bs;
        vsrc[i] = src + d0 + ch;
        vdst[i] = L::DD + ch * L::XW + v;
        vrow[i] = v < ND ? 1 + v : 0;
        vmul[i] = v < ND ? 1u : Du;
    }
    const float *csrc = p.C + b * p.bc_bs + (lane & 3) * 4;
    const int cdst = L::C + (lane & 3) * 4;
    const int *lvl_off = p.lvl_off, *snext = p.snext, *lvl_start = p.lvl_start;

    for (int l = p.nlevels - 1; l >= 0; --l) {
        const int s0 = lvl_start[l], s1 = lvl_start[l + 1];
        for (int base = s0 + w; base < s1; base += kPW * 32) {
            const int sl = base + kPW * lane;
            if (sl < s1) { /* the point; successors as element offsets (index x D,
                            * < 2^31) or -1 */
                sidx[w][lane][0] = lvl_off[sl];
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    const int nx = snext[sl * ND + a];
                    sidx[w][lane][1 + a] = nx >= 0 ? nx * (int)Du : -1;
                }
            }
            __syncwarp();
            const int cnt = min(32, (s1 - base + kPW - 1) / kPW);
            auto issue = [&](int j, int slot) {
                const unsigned bs = wbs + slot * (L::SIZE * 4); /* shared address of the slot */
                int ix[ND + 1];
                load_idx<ND>(sidx[w][j], ix);
                /* a missing successor's row and delta are zero-filled: the row adds 0 */
#pragma unroll
                for (int a = 0; a < ND; ++a) {
                    const bool ok = ix[1 + a] >= 0;
                    kmb_cp_async16_s(bs + (L::GN + a * kWCh * 16 + lane * 4) * 4,
                                     gg_src + (size_t)(unsigned)(ok ? ix[1 + a] : 0) * 16,
                                     ok ? 16 : 0);
                }
#pragma unroll
                for (int i = 0; i < L::NJ; ++i) {
                    const int row = sidx[w][j][vrow[i]];
                    const bool ok = row >= 0;
                    if (vok[i])
                        kmb_cp_async4_s(bs + vdst[i] * 4,
                                        vsrc[i] + (unsigned)(ok ? row : 0) * vmul[i], ok ? 4 : 0);
                }
                if (lane < 4) kmb_cp_async16_s(bs + cdst * 4, csrc + (unsigned)ix[0] * 16, 16);
            };
            int si = 0, sc = 0; /* ring slots of the next issue and of the next compute */
#pragma unroll
            for (int j = 0; j < S - 1; ++j) {
                if (j < cnt) {
                    issue(j, si);
                    si = si + 1 == S ? 0 : si + 1;
                }
                kmb_cp_async_commit();
            }
            for (int j = 0; j < cnt; ++j) {
                if (j + S - 1 < cnt) {
                    issue(j + S - 1, si);
                    si = si + 1 == S ? 0 : si + 1;
                }
                kmb_cp_async_commit();
                kmb_cp_async_wait<S - 1>();
                __syncwarp();
                const float *bf = wb + sc * L::SIZE;
                sc = sc + 1 == S ? 0 : sc + 1;
                int ix[ND + 1];
                load_idx<ND>(sidx[w][j], ix);
                float dd[L::XW];
#pragma unroll
                for (int i = 0; i < L::XW; i += 4)
                    *reinterpret_cast<float4 *>(dd + i) =
                        *reinterpret_cast<const float4 *>(bf + L::DD + c * L::XW + i);
                bool weak = false;
#pragma unroll
                for (int a = 0; a < ND; ++a) weak |= fabsf(dd[a]) * amin[a] < KMB_DECAY_POLY_MAX;
                /* MUFU only where no lane of the warp needs the polynomial */
                const bool fast = !__any_sync(kWFull, weak);
                const float4 C4 = *reinterpret_cast<const float4 *>(bf + L::C + q * 4);
                const float2 gy2 = kmb_f2s(dd[ND]);
                float2 gg[2] = {kmb_mul2(kmb_f2(C4.x, C4.y), gy2),
                                kmb_mul2(kmb_f2(C4.z, C4.w), gy2)};
                auto carry = [&](auto fast_tag) {
                    constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
                    for (int a = 0; a < ND; ++a) { /* zero rows for missing successors */
                        const float4 gn = *reinterpret_cast<const float4 *>(
                            bf + L::GN + a * kWCh * 16 + lane * 4);
                        const float2 dn2 = kmb_f2s(dd[a]);
                        const float2 w0 = kmb_mul2(dn2, A2[a][0]);
                        const float2 w1 = kmb_mul2(dn2, A2[a][1]);
                        const float2 e0 = FAST ? kmb_ex2_2(w0) : kmb_exp2_decay2(w0);
                        const float2 e1 = FAST ? kmb_ex2_2(w1) : kmb_exp2_decay2(w1);
                        gg[0] = kmb_fma2(e0, kmb_f2(gn.x, gn.y), gg[0]);
                        gg[1] = kmb_fma2(e1, kmb_f2(gn.z, gn.w), gg[1]);
                    }
                };
                if (fast)
                    carry(std::true_type{});
                else
                    carry(std::false_type{});
                *reinterpret_cast<float4 *>(gq + (size_t)((unsigned)ix[0] * Du) * 16) =
                    make_float4(gg[0].x, gg[0].y, gg[1].x, gg[1].y);
                __syncwarp(); /* the slot is refilled next */
            }
        }
        __syncthreads();
    }
}

template <int ND>
constexpr int adj_p_stages() {
    return (size_t)kPW * 3 * AdjPSlot<ND>::SIZE * 4 + kPW * 32 * (ND + 1) * 4 <=
                   227 * 1024
               ? 3
               : 2;
}

/* k_scannd_grad_w: the gradient pass with per-point loads, for what the
 * staged k_scannd_grad_s below does not take (M != 16, rows not 16-byte
 * aligned) */
constexpr int kGWarps = 8;    /* warps per CTA */
constexpr int kGPts = 2048;   /* points per CTA */

template <int ND>
__global__ void __launch_bounds__(kGWarps * 32) k_scannd_grad_w(NDDev p) {
    __shared__ float sdA[kGWarps][ND][32][4];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long b = blockIdx.z;
    const long d = (long)blockIdx.y * kWCh + c;
    const unsigned Du = (unsigned)p.D, Mu = (unsigned)p.M;
    const bool qok = q * 4u < Mu;
    float2 A2[ND][2], Ar[ND][2], dAp[ND][2];
#pragma unroll
    for (int a = 0; a < ND; ++a)
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            const unsigned m = q * 4 + 2 * jp;
            const float a0 = m < Mu ? p.A[a][d * Mu + m] : 0.f;
            const float a1 = m + 1 < Mu ? p.A[a][d * Mu + m + 1] : 0.f;
            Ar[a][jp] = kmb_f2(a0, a1);
            A2[a][jp] = kmb_f2(a0 * KMB_LOG2E, a1 * KMB_LOG2E);
            dAp[a][jp] = kmb_f2s(0.f);
        }
    const float *xq = p.x + b * p.x_bs + d;
    const float *dyq = p.dy + b * p.x_bs + d;
    const float *Bq = p.B + b * p.bc_bs + q * 4;
    const float *hq = p.h + b * p.h_bs + d * Mu + q * 4;
    const float *Gq = p.G + b * p.h_bs + d * Mu + q * 4;
    float *dxq = p.dx + b * p.x_bs + d;
    float *dBb = p.dB + b * p.bc_bs;
    float *dCb = p.dC + b * p.bc_bs;
    const float *dq[ND];
    float *ddq[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) {
        dq[a] = p.delta[a] + b * p.dl_bs + d;
        ddq[a] = p.ddelta[a] + b * p.dl_bs + d;
    }
    const long p0 = (long)blockIdx.x * kGPts;
    const long p1 = min(p.P, p0 + kGPts);
    for (long pl = p0 + w; pl < p1; pl += kGWarps) {
        const unsigned pt = (unsigned)pl;
        const unsigned od = pt * Du;
        int pv[ND];
#pragma unroll
        for (int a = 0; a < ND; ++a) pv[a] = p.prev[(size_t)pt * ND + a];
        const float xv = xq[od], gy = dyq[od];
        float dta[ND];
#pragma unroll
        for (int a = 0; a < ND; ++a) dta[a] = dq[a][od];
        float4 B4 = make_float4(0.f, 0.f, 0.f, 0.f), H4 = B4, G4 = B4, hp[ND];
        if (qok) {
            B4 = *reinterpret_cast<const float4 *>(Bq + (size_t)pt * Mu);
            H4 = *reinterpret_cast<const float4 *>(hq + (size_t)od * Mu);
            G4 = *reinterpret_cast<const float4 *>(Gq + (size_t)od * Mu);
        }
#pragma unroll
        for (int a = 0; a < ND; ++a)
            if (pv[a] >= 0 && qok)
                hp[a] = *reinterpret_cast<const float4 *>(hq + (size_t)((unsigned)pv[a] * Du) * Mu);
        grad_point<ND>(B4, H4, G4, hp, pv, xv, gy, dta, A2, Ar, dAp, qok, lane, c, q,
                       dxq + od, ddq, od, dBb + (size_t)pt * Mu, dCb + (size_t)pt * Mu);
    }
    /* dA: fold the CTA's warps, one atomic per (axis, channel, state) */
#pragma unroll
    for (int a = 0; a < ND; ++a) {
        sdA[w][a][lane][0] = dAp[a][0].x;
        sdA[w][a][lane][1] = dAp[a][0].y;
        sdA[w][a][lane][2] = dAp[a][1].x;
        sdA[w][a][lane][3] = dAp[a][1].y;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ND * 32 * 4; i += kGWarps * 32) {
        const int a = i / 128, ln = (i / 4) % 32, j = i % 4;
        float t = 0.f;
        for (int ww = 0; ww < kGWarps; ++ww) t += sdA[ww][a][ln][j];
        const int cc = ln >> 2, qq = ln & 3;
        const unsigned m = qq * 4 + j;
        if (m < Mu) atomicAdd(p.dA[a] + ((long)blockIdx.y * kWCh + cc) * Mu + m, t);
    }
}

/* Staged gradient pass: the per-point terms of k_scannd_grad_w with the
 * loads batched, for M = 16.  A CTA of kSW warps takes the 8 channels of
 * one channel group over a range of PR consecutive points (a multiple of
 * kST; a z-slice of a 64^3 grid) and streams it in stages of kST points
 * through a cp.async pipeline SS stages deep: per stage the G rows of its
 * points (128 floats: 8 channels x 16 states), the h rows of their
 * predecessors along the NF far axes (stride > kNR; the leading axes of
 * the row-major grid), and their x, dy, delta, B and predecessor-table
 * entries.  The points' own h rows go to a ring of R rows, from which the
 * predecessors along the near axes (stride <= kNR) are read: kNR rows
 * before the range are staged first.  Each warp then computes kST / kSW
 * points of the stage from shared memory, so all global loads of a stage
 * are in flight together.  The layout is fixed at compile time (shared
 * memory offsets are immediates). */
constexpr int kSW = 16; /* warps per CTA */
constexpr int kST = 32; /* points per stage */
constexpr int kNR = 64; /* largest axis stride read from the ring */

template <int ND, int NF>
struct GSLayout {
    static constexpr int ROW = kWCh * 16;                    /* floats per state row */
    static constexpr int O_G = 0;                            /* [kST][ROW] */
    static constexpr int O_FAR = O_G + kST * ROW;            /* [NF][kST][ROW] */
    static constexpr int O_X = O_FAR + NF * kST * ROW;       /* [2 + ND][kST][kWCh] */
    static constexpr int O_B = O_X + (2 + ND) * kST * kWCh;  /* [kST][16] */
    static constexpr int PVW = ND == 3 ? 4 : ND;              /* ints per point (3 axes: padded) */
    static constexpr int O_PV = O_B + kST * 16;              /* [kST][PVW] ints */
    static constexpr int STAGE = (O_PV + kST * PVW + 3) & ~3;
    static constexpr size_t bytes(int ss) {
        return sizeof(float) * ((size_t)(ss * kST + kNR) * ROW + (size_t)ss * STAGE);
    }
    static constexpr int SS = bytes(3) <= 227 * 1024 ? 3 : 2; /* stages in flight */
    /* ring rows: stage k + SS - 1 is loaded while stage k reads kNR rows back */
    static constexpr int R = SS * kST + kNR;
    static constexpr size_t SMEM = bytes(SS);
    static_assert(bytes(SS) <= 227 * 1024, "staged gradient layout");
    static_assert((2 + ND) * 2 * kST + 4 * kST <= kSW * 32, "stage copy threads");
};

struct GradS {
    int stride[kMaxAxes]; /* point stride of each axis (row-major) */
    int PR;               /* points per CTA, a multiple of kST */
};

/* grad_point's terms with the sums over a channel's 4 lanes reduce-
 * scattered: lane q stores dx (q 0) or ddelta_{q-1}; a fifth value
 * (ddelta_3 of 4 axes) is summed by butterfly and stored by lane 0.
 * FAST: no decay exponent of the point is in the polynomial range, so
 * kmb_exp2_decay2 would return the MUFU values, which are used directly. */
template <int ND, bool FAST>
__device__ __forceinline__ void grad_point16(
    const float4 &B4, const float4 &H4, const float4 &G4, const float4 (&hp)[ND],
    const int (&pv)[ND], float xv, float gy, const float (&dta)[ND],
    const float2 (&A2)[ND][2], float2 (&dAp)[ND][2], int lane,
    int c, int q, float *out0, float *out4, float *dBrow, float *dCrow) {
    constexpr float kInvND = 1.0f / ND; /* the mean within 1 ulp of a division */
    float dt_bar = 0.f;
#pragma unroll
    for (int a = 0; a < ND; ++a) dt_bar += dta[a];
    dt_bar *= kInvND;
    const float2 gg[2] = {kmb_f2(G4.x, G4.y), kmb_f2(G4.z, G4.w)};
    const float2 Bp[2] = {kmb_f2(B4.x, B4.y), kmb_f2(B4.z, B4.w)};
    const float2 gy2 = kmb_f2s(gy), dtb2 = kmb_f2s(dt_bar), xv2 = kmb_f2s(xv);
    float2 sx2 = kmb_f2s(0.f), sb2 = kmb_f2s(0.f), sdt2[ND];
    float v8[8];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        const float2 gd = kmb_mul2(gg[jp], dtb2);
        sx2 = kmb_fma2(gd, Bp[jp], sx2);
        sb2 = kmb_fma2(kmb_mul2(gg[jp], Bp[jp]), xv2, sb2);
        const float2 vb = kmb_mul2(gd, xv2); /* dB */
        const float2 vc = kmb_mul2(gy2, jp ? kmb_f2(H4.z, H4.w) : kmb_f2(H4.x, H4.y));
        v8[2 * jp] = vb.x;
        v8[2 * jp + 1] = vb.y;
        v8[4 + 2 * jp] = vc.x;
        v8[4 + 2 * jp + 1] = vc.y;
    }
#pragma unroll
    for (int a = 0; a < ND; ++a) {
        sdt2[a] = kmb_f2s(0.f);
        if (pv[a] >= 0) {
            const float2 dv2 = kmb_f2s(dta[a]);
            const float2 hpp[2] = {kmb_f2(hp[a].x, hp[a].y), kmb_f2(hp[a].z, hp[a].w)};
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) {
                const float2 wv = kmb_mul2(dv2, A2[a][jp]);
                const float2 e = FAST ? kmb_ex2_2(wv) : kmb_exp2_decay2(wv);
                const float2 gh = kmb_mul2(kmb_mul2(gg[jp], hpp[jp]), e);
                dAp[a][jp] = kmb_fma2(gh, dv2, dAp[a][jp]);
                sdt2[a] = kmb_fma2(gh, A2[a][jp], sdt2[a]); /* A log2 e: times ln 2 below */
            }
        }
    }
    /* per-lane partial sums: dx, then ddelta_a = sum G h(p-e) e A_a + (sum G B x) / ND */
    const float sbn = (sb2.x + sb2.y) * kInvND;
    float v[4] = {sx2.x + sx2.y, 0.f, 0.f, 0.f};
#pragma unroll
    for (int a = 0; a < ND && a < 3; ++a) v[1 + a] = (sdt2[a].x + sdt2[a].y) * KMB_LN2 + sbn;
    /* reduce-scatter over the channel's 4 lanes (q = lane bits 0-1) */
    const bool hi = q & 2, lo = q & 1;
    float k0 = hi ? v[2] : v[0], k1 = hi ? v[3] : v[1];
    const float s0 = hi ? v[0] : v[2], s1 = hi ? v[1] : v[3];
    k0 += __shfl_xor_sync(kWFull, s0, 2);
    k1 += __shfl_xor_sync(kWFull, s1, 2);
    const float keep = lo ? k1 : k0, send = lo ? k0 : k1;
    const float mine = keep + __shfl_xor_sync(kWFull, send, 1);
    if (q <= ND) *out0 = mine;
    if constexpr (ND == 4) {
        float v4 = (sdt2[3].x + sdt2[3].y) * KMB_LN2 + sbn;
        v4 += __shfl_xor_sync(kWFull, v4, 1);
        v4 += __shfl_xor_sync(kWFull, v4, 2);
        if (q == 0) *out4 = v4;
    }
    /* dB / dC: sums over the 8 channels, then 4 states into one lane */
    const float r1 = rs8_ch(v8, lane);
    const float r2 = __shfl_down_sync(kWFull, r1, 4);
    const float r3 = __shfl_down_sync(kWFull, r1, 8);
    const float r4 = __shfl_down_sync(kWFull, r1, 12);
    if ((c & 3) == 0) {
        float *dst = ((c >> 2) ? dCrow : dBrow) + q * 4;
        atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(r1, r2, r3, r4));
    }
}

template <int ND, int NF>
__global__ void __launch_bounds__(kSW * 32, 1) k_scannd_grad_s(NDDev p, GradS g) {
    using L = GSLayout<ND, NF>;
    constexpr int ROW = L::ROW, SS = L::SS, R = L::R;
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long b = blockIdx.z;
    const long d0 = (long)blockIdx.y * kWCh;
    const long d = d0 + c;
    float2 A2[ND][2], dAp[ND][2];
#pragma unroll
    for (int a = 0; a < ND; ++a)
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            const float *ap = p.A[a] + d * 16 + q * 4 + 2 * jp;
            const float2 av = kmb_f2(ap[0], ap[1]);
            A2[a][jp] = kmb_f2(av.x * KMB_LOG2E, av.y * KMB_LOG2E);
            dAp[a][jp] = kmb_f2s(0.f);
        }
    float amin[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) amin[a] = lane_amin(A2[a]);
    const long D = p.D;
    const size_t hrow = (size_t)D * 16; /* floats between two points' state rows */
    const float *hg = p.h + b * p.h_bs + d0 * 16 + lane * 4;
    const float *Gg = p.G + b * p.h_bs + d0 * 16 + lane * 4;
    const float *dlg[ND];
#pragma unroll
    for (int a = 0; a < ND; ++a) dlg[a] = p.delta[a] + b * p.dl_bs + d0;
    /* this lane's output of the dx / ddelta reduce-scatter */
    float *ob = p.dx + b * p.x_bs + d;
#pragma unroll
    for (int a = 0; a < ND && a < 3; ++a)
        if (q == a + 1) ob = p.ddelta[a] + b * p.dl_bs + d;
    float *ob4 = p.ddelta[ND - 1] + b * p.dl_bs + d; /* 4 axes: ddelta_3 */
    float *dBb = p.dB + b * p.bc_bs, *dCb = p.dC + b * p.bc_bs;

    const long pb = (long)blockIdx.x * g.PR;     /* first point computed */
    const long pe = min(p.P, pb + (long)g.PR);   /* end of the range */
    const long ps = pb > kNR ? pb - kNR : 0;     /* first point staged */
    const int nst = (int)((pe - ps + kST - 1) / kST);
    float *ring = sm;
    float *stages = sm + R * ROW;

    /* copy jobs of this thread that do not change between stages */
    constexpr int NA = (2 + ND) * 2 * kST; /* x, dy, delta rows: 2 chunks a point */
    const bool j_arr = tid < NA;
    const int arr = tid / (2 * kST), aj = tid % (2 * kST);
    const float *abase = p.x + b * p.x_bs + d0;
    if (arr == 1) abase = p.dy + b * p.x_bs + d0;
#pragma unroll
    for (int a = 0; a < ND; ++a)
        if (arr == 2 + a) abase = dlg[a];
    const long aoff = (long)(aj >> 1) * D + (aj & 1) * 4;
    const int adst = L::O_X + (arr * kST + (aj >> 1)) * kWCh + (aj & 1) * 4;
    const bool j_b = tid >= NA && tid < NA + 4 * kST;
    const int bj = tid - NA;
    const float *bbase = p.B + b * p.bc_bs;
    const int boff = (bj >> 2) * 16 + (bj & 3) * 4;
    const bool j_pv = tid < ND * kST;

    auto load = [&](int k) {
        const long s0 = ps + (long)k * kST;
        float *rs = ring + (k % (R / kST)) * kST * ROW + lane * 4;
        float *st = stages + (k % SS) * L::STAGE;
#pragma unroll
        for (int u = 0; u < kST / kSW; ++u) {
            const int r = w + u * kSW;
            const long pt = s0 + r;
            const bool ok = pt < pe;
            kmb_cp_async16(rs + r * ROW, hg + (ok ? pt * hrow : 0), ok ? 16 : 0);
        }
        if (s0 < pb) return; /* rows before the range: the ring only */
#pragma unroll
        for (int u = 0; u < kST / kSW; ++u) {
            const int r = w + u * kSW;
            const long pt = s0 + r;
            const bool ok = pt < pe;
            kmb_cp_async16(st + L::O_G + r * ROW + lane * 4, Gg + (ok ? pt * hrow : 0),
                           ok ? 16 : 0);
#pragma unroll
            for (int f = 0; f < NF; ++f) {
                const long pp = pt - g.stride[f];
                const bool okf = ok && pp >= 0;
                kmb_cp_async16(st + L::O_FAR + (f * kST + r) * ROW + lane * 4,
                               hg + (okf ? pp * hrow : 0), okf ? 16 : 0);
            }
        }
        if (j_arr) {
            const bool ok = s0 + (aj >> 1) < pe;
            kmb_cp_async16(st + adst, abase + (ok ? s0 * D + aoff : 0), ok ? 16 : 0);
        }
        if (j_b) {
            const bool ok = s0 + (bj >> 2) < pe;
            kmb_cp_async16(st + L::O_B + boff, bbase + (ok ? s0 * 16 + boff : 0), ok ? 16 : 0);
        }
        if (j_pv) {
            const int r = tid / ND, a = tid % ND;
            const bool ok = s0 + r < pe;
            kmb_cp_async4(st + L::O_PV + r * L::PVW + a, p.prev + (ok ? s0 * ND + tid : 0), ok);
        }
    };

#pragma unroll 1
    for (int k = 0; k < SS - 1; ++k) {
        if (k < nst) load(k);
        kmb_cp_async_commit();
    }
#pragma unroll 1
    for (int k = 0; k < nst; ++k) {
        kmb_cp_async_wait<SS - 2>();
        __syncthreads();
        if (k + SS - 1 < nst) load(k + SS - 1);
        kmb_cp_async_commit();
        const long s0 = ps + (long)k * kST;
        if (s0 < pb) continue;
        const float *st = stages + (k % SS) * L::STAGE;
        const int *spv = reinterpret_cast<const int *>(st + L::O_PV);
        const int sb = (k % (R / kST)) * kST; /* ring row of the stage's first point */
        /* MUFU only where no lane needs the polynomial for the warp's points
         * (missing predecessors are included: conservative) */
        bool weak = false;
#pragma unroll
        for (int u = 0; u < kST / kSW; ++u) {
            const int r = w + u * kSW;
#pragma unroll
            for (int a = 0; a < ND; ++a)
                weak |= fabsf(st[L::O_X + ((2 + a) * kST + r) * kWCh + c]) * amin[a] <
                        KMB_DECAY_POLY_MAX;
        }
        auto points = [&](auto fast_tag) {
        constexpr bool FAST = decltype(fast_tag)::value;
        /* a warp's points interleaved (3 axes; 4 would spill) */
        constexpr int kUnroll = ND == 3 ? kST / kSW : 1;
#pragma unroll kUnroll
        for (int u = 0; u < kST / kSW; ++u) {
            const int r = w + u * kSW;
            const long pt = s0 + r;
            if (pt >= pe) break;
            int pv[ND];
            float dta[ND];
            float4 hp[ND];
            if constexpr (L::PVW == 4) {
                const int4 t = *reinterpret_cast<const int4 *>(spv + r * 4);
                pv[0] = t.x;
                pv[1] = t.y;
                pv[2] = t.z;
                if constexpr (ND == 4) pv[ND - 1] = t.w;
            } else {
#pragma unroll
                for (int a = 0; a < ND; ++a) pv[a] = spv[r * L::PVW + a];
            }
#pragma unroll
            for (int a = 0; a < ND; ++a) dta[a] = st[L::O_X + ((2 + a) * kST + r) * kWCh + c];
            const float xv = st[L::O_X + r * kWCh + c];
            const float gy = st[L::O_X + (kST + r) * kWCh + c];
            const float4 B4 = *reinterpret_cast<const float4 *>(st + L::O_B + r * 16 + q * 4);
            const float4 G4 = *reinterpret_cast<const float4 *>(st + L::O_G + r * ROW + lane * 4);
            const float4 H4 = *reinterpret_cast<const float4 *>(ring + (sb + r) * ROW + lane * 4);
#pragma unroll
            for (int a = 0; a < ND; ++a)
                if (pv[a] >= 0) {
                    const float *src;
                    if (a < NF) {
                        src = st + L::O_FAR + (a * kST + r) * ROW;
                    } else {
                        int sl = sb + r - g.stride[a];
                        if (sl < 0) sl += R;
                        src = ring + sl * ROW;
                    }
                    hp[a] = *reinterpret_cast<const float4 *>(src + lane * 4);
                }
            const long od = pt * D;
            grad_point16<ND, FAST>(B4, H4, G4, hp, pv, xv, gy, dta, A2, dAp, lane, c, q,
                                   ob + od, ob4 + od, dBb + pt * 16, dCb + pt * 16);
        }
        };
        if (__any_sync(kWFull, weak))
            points(std::false_type{});
        else
            points(std::true_type{});
    }
    kmb_cp_async_wait<0>();
    __syncthreads();
    /* dA: fold the CTA's warps, one atomic per (axis, channel, state) */
    float *sdA = sm; /* [kSW][ND][32][4] */
#pragma unroll
    for (int a = 0; a < ND; ++a)
        *reinterpret_cast<float4 *>(sdA + ((w * ND + a) * 32 + lane) * 4) =
            make_float4(dAp[a][0].x, dAp[a][0].y, dAp[a][1].x, dAp[a][1].y);
    __syncthreads();
    for (int i = tid; i < ND * 32 * 4; i += kSW * 32) {
        const int a = i / 128, ln = (i / 4) % 32, j = i % 4;
        float t = 0.f;
        for (int ww = 0; ww < kSW; ++ww) t += sdA[((ww * ND + a) * 32 + ln) * 4 + j];
        atomicAdd(p.dA[a] + (d0 + (ln >> 2)) * 16 + (ln & 3) * 4 + j, t);
    }
}

/* Channel tile of a CTA: a power of two dividing 256, small enough that
 * the grid has >= 2 CTAs per SM (every CTA walks all levels, so CTAs are
 * the only parallelism across chains), and within the backward's shared
 * dA budget. */
int pick_dtile(long D, int nd, long M, bool bwd, long batch) {
    int t = 64;
    while (t > 1 && t / 2 >= D) t >>= 1;
    while (t > 4 && batch * ((D + t - 1) / t) < 2 * 148) t >>= 1;
    if (bwd)
        while (t > 1 && (long)nd * t * M * 4 > 96 * 1024) t >>= 1;
    return t;
}

void fill_dev(const KmbNDLaunch *a, NDDev *p) {
    memset(p, 0, sizeof *p);
    p->x = a->x; p->B = a->B; p->C = a->C; p->dy = a->dy;
    p->h = a->h; p->y = a->y; p->G = a->G;
    p->dx = a->dx; p->dB = a->dB; p->dC = a->dC;
    for (int i = 0; i < a->nd; ++i) {
        p->delta[i] = a->delta[i];
        p->A[i] = a->A[i];
        p->dA[i] = a->dA[i];
        p->ddelta[i] = a->ddelta[i];
    }
    p->lvl_start = a->lvl_start; p->lvl_off = a->lvl_off; p->prev = a->prev; p->next = a->next;
    p->sprev = a->sprev; p->snext = a->snext;
    p->P = a->P; p->D = a->D; p->M = a->M; p->nd = a->nd; p->nlevels = a->nlevels;
    p->x_bs = a->P * a->D;
    p->dl_bs = a->delta_bstride;
    p->bc_ds = a->bc_shared ? 0 : a->M;
    p->bc_ps = a->bc_shared ? a->M : a->D * a->M;
    p->bc_bs = a->P * p->bc_ps;
    p->h_bs = a->P * a->D * a->M;
}

} // namespace

/* the warp-per-point kernels: channel-shared B/C with 16-byte rows,
 * M % 4 == 0 <= 16, D % 8 == 0, 3 or 4 axes */
static bool use_w(const KmbNDLaunch *a) {
    auto al = [](const void *q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
    return (a->nd == 3 || a->nd == 4) && a->bc_shared && a->M % 4 == 0 && a->M <= 16 &&
           a->D % kWCh == 0 && a->P * a->D < (1L << 31) && al(a->B) && al(a->C) && al(a->h) &&
           al(a->G) && al(a->dB) && al(a->dC);
}

/* Far-axis count and range size of k_scannd_grad_s for this launch; -1
 * when it does not apply (M != 16 or rows not 16-byte aligned:
 * k_scannd_grad_w then runs).  Strides do not grow with the axis index,
 * so the far axes (stride > kNR) are the leading ones. */
static int grad_s_cfg(const KmbNDLaunch *a, GradS *g) {
    auto al = [](const void *q) { return ((uintptr_t)q & 15u) == 0; };
    if (a->M != 16 || !al(a->x) || !al(a->dy) || a->delta_bstride % 4 != 0) return -1;
    for (int i = 0; i < a->nd; ++i)
        if (!al(a->delta[i])) return -1;
    memset(g, 0, sizeof *g);
    long st = 1;
    int nf = 0;
    for (int i = a->nd - 1; i >= 0; --i) {
        if (st > (1L << 30)) return -1;
        g->stride[i] = (int)st;
        st *= a->dims[i];
    }
    for (int i = 0; i < a->nd; ++i) nf += g->stride[i] > kNR;
    /* points per CTA: 4096-point ranges unless the grid gets thin */
    const long groups = a->batch * (a->D / kWCh);
    int pr = 4096;
    while (pr > 4 * kST && ((a->P + pr - 1) / pr) * groups < 2 * 148) pr >>= 1;
    g->PR = pr;
    return nf;
}

template <int ND, int NF>
static cudaError_t launch_grad_s(const NDDev &p, const KmbNDLaunch *a, const GradS &g,
                                 cudaStream_t s) {
    constexpr size_t smem = GSLayout<ND, NF>::SMEM;
    cudaError_t e = cudaFuncSetAttribute(k_scannd_grad_s<ND, NF>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((a->P + g.PR - 1) / g.PR), (unsigned)(a->D / kWCh), (unsigned)a->batch);
    k_scannd_grad_s<ND, NF><<<grid, kSW * 32, smem, s>>>(p, g);
    return cudaGetLastError();
}

/* the pipelined warp kernels copy 16-byte chunks of the M = 16 state
 * rows and of the per-point rows of x or dy (xdy) and delta */
static bool staged_rows(const KmbNDLaunch *a, const void *xdy) {
    auto al = [](const void *q) { return ((uintptr_t)q & 15u) == 0; };
    bool ok = a->M == 16 && al(xdy) && a->delta_bstride % 4 == 0;
    for (int i = 0; i < a->nd; ++i) ok = ok && al(a->delta[i]);
    return ok;
}

template <int ND>
static cudaError_t launch_w(const NDDev &p, const KmbNDLaunch *a, bool bwd, cudaStream_t s) {
    dim3 grid((unsigned)(a->D / kWCh), (unsigned)a->batch);
    if (!bwd) {
        if (staged_rows(a, a->x)) {
            constexpr int S = fwd_p_stages<ND>();
            constexpr size_t smem = (size_t)kPW * S * FwdPSlot<ND>::SIZE * sizeof(float);
            cudaError_t e = cudaFuncSetAttribute(
                k_scannd_fwd_p<ND, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            k_scannd_fwd_p<ND, S><<<grid, kPW * 32, smem, s>>>(p);
            return cudaGetLastError();
        }
        k_scannd_fwd_w<ND><<<grid, kWWarpsF * 32, 0, s>>>(p);
        return cudaGetLastError();
    }
    cudaError_t e;
    if (staged_rows(a, a->dy)) {
        constexpr int S = adj_p_stages<ND>();
        constexpr size_t smem = (size_t)kPW * S * AdjPSlot<ND>::SIZE * sizeof(float);
        e = cudaFuncSetAttribute(k_scannd_adj_p<ND, S>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k_scannd_adj_p<ND, S><<<grid, kPW * 32, smem, s>>>(p);
    } else {
        k_scannd_adj_w<ND><<<grid, kWWarpsA * 32, 0, s>>>(p);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    GradS g;
    switch (grad_s_cfg(a, &g)) {
    case 0: return launch_grad_s<ND, 0>(p, a, g, s);
    case 1: return launch_grad_s<ND, 1>(p, a, g, s);
    case 2: return launch_grad_s<ND, 2>(p, a, g, s);
    case 3:
        if constexpr (ND == 4) return launch_grad_s<ND, 3>(p, a, g, s);
        break;
    default: break;
    }
    dim3 gg((unsigned)((a->P + kGPts - 1) / kGPts), (unsigned)(a->D / kWCh), (unsigned)a->batch);
    k_scannd_grad_w<ND><<<gg, kGWarps * 32, 0, s>>>(p);
    return cudaGetLastError();
}

extern "C" int kmb_launch_scannd_fwd(const KmbNDLaunch *a, cudaStream_t s) {
    NDDev p;
    fill_dev(a, &p);
    if (use_w(a)) {
        const cudaError_t e = a->nd == 3 ? launch_w<3>(p, a, false, s) : launch_w<4>(p, a, false, s);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "scannd forward launch");
        return KMB_OK;
    }
    p.dtile = pick_dtile(a->D, a->nd, a->M, false, a->batch);
    dim3 grid((unsigned)((a->D + p.dtile - 1) / p.dtile), (unsigned)a->batch);
    k_scannd_fwd<<<grid, kThreads, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scannd forward launch");
    return KMB_OK;
}

extern "C" int kmb_launch_scannd_bwd(const KmbNDLaunch *a, cudaStream_t s) {
    NDDev p;
    fill_dev(a, &p);
    p.dtile = pick_dtile(a->D, a->nd, a->M, true, a->batch);
    if ((long)a->nd * p.dtile * a->M * 4 > 96 * 1024)
        return kmb_fail(KMB_EUNSUPPORTED, "scannd backward: ndims*M too large (M=%ld)", a->M);
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < a->nd && e == cudaSuccess; ++i)
        e = cudaMemsetAsync(a->dA[i], 0, sizeof(float) * a->D * a->M, s);
    if (e == cudaSuccess && a->bc_shared) {
        const size_t nb = sizeof(float) * a->batch * a->P * a->M;
        e = cudaMemsetAsync(a->dB, 0, nb, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(a->dC, 0, nb, s);
    }
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scannd backward memset");
    if (use_w(a)) {
        e = a->nd == 3 ? launch_w<3>(p, a, true, s) : launch_w<4>(p, a, true, s);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "scannd backward launch");
        return KMB_OK;
    }
    const size_t smem = sizeof(float) * a->nd * p.dtile * a->M;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(k_scannd_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "scannd backward smem attribute");
    }
    dim3 grid((unsigned)((a->D + p.dtile - 1) / p.dtile), (unsigned)a->batch);
    k_scannd_bwd<<<grid, kThreads, smem, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scannd backward launch");
    return KMB_OK;
}
