/*
 * 2D selective scan over an H x W grid (ND scan with ndims = 2), forward
 * and backward, for channel-shared B/C (the config-4 shape).  Semantics of
 * the reference src/scan_nd.c:86-230 with theta = lambda = NULL, axis 0 the
 * rows (predecessor p - W) and axis 1 the columns (p - 1):
 *
 *   dt_bar(p,d) = (delta_0(p,d) + delta_1(p,d)) / 2
 *   h(p,d,m)    = dt_bar (B(p,m) x(p,d))
 *               + exp(delta_0 A_0(d,m)) h(p-W,d,m) + exp(delta_1 A_1(d,m)) h(p-1,d,m)
 *   y(p,d)      = sum_m C(p,m) h(p,d,m)
 *
 * and the full state history h [P, D, M] written, as the reference API
 * requires (the backward reads it).
 *
 * Decomposition.  A CTA owns one batch item and 8 channels (a warp's lanes
 * are 8 channels x 4 groups of 4 states, two FFMA2 pairs each) and sweeps
 * the grid in strips of 64 columns.  Warp w of a strip owns 8 adjacent
 * columns and runs one row behind warp w-1: at step t it computes row
 * t - w, left to right, with the vertical carry h(i-1, .) of its columns
 * in registers and the state of the column to its left taken from warp
 * w-1's previous step (double-buffered shared slot; the first warp of a
 * strip reads the previous strip's last column from an L2 scratch column).
 * One CTA barrier per step.  Inputs are staged per warp by cp.async a few
 * rows ahead.
 *
 * The backward walks the same strips right to left and bottom to top with
 * the adjoint
 *   G(p) = C(p) dy(p) + exp(delta_0(p+W) A_0) G(p+W) + exp(delta_1(p+1) A_1) G(p+1)
 * carried the same way (vertical carry in registers, right neighbour from
 * warp w+1), and per point
 *   dx = dt_bar sum_m G B,   ddelta_a = (sum_m G B x) / 2 + sum_m G h(p-e_a) A_a e_a(p),
 *   dA_a += G h(p-e_a) delta_a e_a(p),   dB(p,m) += G dt_bar x,  dC(p,m) += dy h
 * with e_a(p) = exp(delta_a(p) A_a); dB / dC are folded over the CTA's 8
 * channels by shuffles and added to global memory with one atomic per
 * (point, state) and CTA.
 */
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include <cuda_bf16.h>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kWarps = 8;                 /* warps per CTA */
constexpr int kCPW = 8;                   /* columns per warp */
constexpr int kStrip = kWarps * kCPW;     /* columns per strip */
constexpr int kCh = 8;                    /* channels per CTA */
constexpr int kRing = 4;                  /* input rows staged ahead per warp */
constexpr unsigned kFull = 0xffffffffu;

/* floats of one staged row of a warp: x, delta_0, delta_1 as [col][ch],
 * B and C as [col][16], and the left edge column (32 lanes x 4 states,
 * used by the first warp of a strip) */
constexpr int kSlotX = kCPW * kCh;
constexpr int kSlotB = kCPW * 16;
constexpr int kSlotE = 128;
constexpr int kSlot = 3 * kSlotX + 2 * kSlotB + kSlotE;

/* The same slot with inputs of element type T (fp32, or bf16 for the
 * bf16-I/O entry points), offsets in floats: x / delta_0 / delta_1 regions
 * of X floats, B / C regions of Bn floats, then the fp32 edge column. */
template <typename T> struct FL {
    static constexpr int X = kSlotX * (int)sizeof(T) / 4;
    static constexpr int Bn = kSlotB * (int)sizeof(T) / 4;
    static constexpr int E0 = 3 * X + 2 * Bn;
    static constexpr int SLOT = E0 + kSlotE;
};
static_assert(FL<float>::SLOT == kSlot, "fp32 forward slot layout");

/* Element idx of a staged region of T, as float. */
template <typename T> __device__ __forceinline__ float ldT(const float *region, int idx) {
    if constexpr (sizeof(T) == 4) return region[idx];
    else return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(region)[idx]);
}

/* Elements idx .. idx + 3 (idx a multiple of 4) of a staged region of T. */
template <typename T> __device__ __forceinline__ float4 ld4T(const float *region, int idx) {
    if constexpr (sizeof(T) == 4) {
        return *reinterpret_cast<const float4 *>(region + idx);
    } else {
        const uint2 u = *reinterpret_cast<const uint2 *>(
            reinterpret_cast<const __nv_bfloat16 *>(region) + idx);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
}

template <typename T> __device__ __forceinline__ void stT(T *dst, float v) {
    if constexpr (sizeof(T) == 4) *dst = v;
    else *dst = __float2bfloat16_rn(v);
}

struct S2D {
    const float *x, *d0, *d1, *A0, *A1, *B, *C, *dy, *h;
    float *hout, *y, *edge;
    float *dx, *dd0, *dd1, *dA0, *dA1, *dB, *dC;
    long H, W, D, M;
    long dl_bs; /* floats between batch items of each delta axis */
    long batch;
    /* strip split: every (item, channel group, strip) is a work item taken
     * in order from *work by persistent CTAs; prog[(strip * batch + b) *
     * groups + g] counts the rows whose edge column that strip has
     * published */
    int split;
    int *work, *prog;
};

/* set when a wait on another CTA's progress gave up (kmb_scan2d_check_error) */
__device__ int g_scan2d_error;

/* Warp-wide wait until *prog >= need (lane 0 polls with acquire loads,
 * bounded by about 2^31 clock cycles; on expiry the error word is set and
 * later waits return at once). */
__device__ __forceinline__ void wait_progress(const int *prog, int need, int lane) {
    if (lane == 0) {
        const long long t0 = clock64();
        for (;;) {
            int v;
            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(prog) : "memory");
            if (v >= need) break;
            if (*reinterpret_cast<volatile int *>(&g_scan2d_error)) break;
            if (clock64() - t0 > (1ll << 31)) {
                atomicExch(&g_scan2d_error, 1);
                break;
            }
            __nanosleep(64);
        }
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
    __syncwarp();
}

/* Publishes `value` rows of this warp's edge writes (all lanes call it). */
__device__ __forceinline__ void publish_progress(int *prog, int value, int lane) {
    __threadfence();
    __syncwarp();
    if (lane == 0)
        asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(prog), "r"(value) : "memory");
}

/* The next work item of a CTA: (b, g, first strip, end strip).  Strip-split
 * items come strip by strip in the order `order` (forward: ascending,
 * backward: descending), so the producer of an item's edge column was
 * taken earlier by a CTA already running; without the split a CTA has one
 * item, all strips of its (blockIdx.y, blockIdx.x). */
__device__ __forceinline__ bool next_item(const S2D &p, long iter, long nstrips, bool descending,
                                          long *sh, long &b, long &g, long &s0, long &s1) {
    const long groups = p.D / kCh;
    if (!p.split) {
        if (iter > 0) return false;
        b = blockIdx.y;
        g = blockIdx.x;
        s0 = 0;
        s1 = nstrips;
        return true;
    }
    if (threadIdx.x == 0) *sh = atomicAdd(p.work, 1);
    __syncthreads();
    const long it = *sh;
    __syncthreads();
    const long per = p.batch * groups;
    if (it >= nstrips * per) return false;
    const long s = descending ? nstrips - 1 - it / per : it / per, r = it % per;
    b = r / groups;
    g = r % groups;
    s0 = s;
    s1 = s + 1;
    return true;
}

/* min over the lane's four states of |log2(e) A| */
__device__ __forceinline__ float abs_min4(const float2 (&a)[2]) {
    return fminf(fminf(fabsf(a[0].x), fabsf(a[0].y)), fminf(fabsf(a[1].x), fabsf(a[1].y)));
}

/* False only when every |w| = |delta A log2(e)| of the lane's states is at
 * least KMB_DECAY_POLY_MAX, i.e. no element takes the weak-decay polynomial:
 * rounding is monotonic, so |delta| amin >= that bound implies
 * fl(|delta| |A_m|) >= it for
 * every state m.  Lanes past the last state (`live` false) never count. */
__device__ __forceinline__ bool weak_possible(float dv0, float dv1, float amin0, float amin1,
                                              bool live) {
    return live && (fabsf(dv0) * amin0 < KMB_DECAY_POLY_MAX ||
                    fabsf(dv1) * amin1 < KMB_DECAY_POLY_MAX);
}

/* e = 2^w for the four state pairs of one point (both axes, two pairs
 * each), elementwise equal to kmb_exp2_decay2: the MUFU ex2 for all, and
 * the polynomial path only when some lane of the warp may need it.  All 32
 * lanes must run it. */
__device__ __forceinline__ void exp2_decay_point(const float2 (&w)[4], float2 (&e)[4], bool weak) {
#pragma unroll
    for (int u = 0; u < 4; ++u) e[u] = kmb_f2(kmb_ex2(w[u].x), kmb_ex2(w[u].y));
    if (__any_sync(kFull, weak)) {
#pragma unroll
        for (int u = 0; u < 4; ++u) e[u] = kmb_exp2_decay2(w[u]);
    }
}

/* The forward's copies of one staged row, per lane: chunk u of the lane
 * is element lane + 32u of the slot's 112 16-byte chunks (x / delta_0 /
 * delta_1: 16 each, B / C: 32 each).  Only the row changes between rows,
 * so the source pointer at row 0, the row stride and the column validity
 * are fixed for a strip. */
struct FwdCopies {
    const char *src[4]; /* source of the next row staged */
    long rs[4];         /* row stride in bytes (x / delta rows: W*D; B / C rows: W*M elements) */
    int dst[4];         /* destination in floats from the slot start */
    bool ok[4];
};

/* fp32: x / delta_0 / delta_1 rows are 8 columns x 8 channels = 16 chunks
 * of 16 bytes each, B / C rows 8 columns x 16 states = 32 chunks each (112
 * in all); bf16: 8 and 16 chunks (56 in all).  Chunk e goes to lane e % 32. */
template <typename T>
__device__ __forceinline__ void fwd_copies(const S2D &p, long b, long j0, long dch0, int lane,
                                           FwdCopies &f) {
    using L = FL<T>;
    constexpr int ES = (int)sizeof(T), EPC = 16 / ES;       /* elements per chunk */
    constexpr int XC = kCh / EPC;                            /* chunks per column of x */
    constexpr int BC = 16 / EPC;                             /* chunks per column of B */
    constexpr int NX = 3 * kCPW * XC, NB = 2 * kCPW * BC;
    const long W = p.W, D = p.D, M = p.M;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int e = lane + 32 * u;
        if (e < NX) {
            const int t = e / (kCPW * XC), r = e % (kCPW * XC), col = r / XC, part = r % XC;
            const long j = j0 + col;
            const T *base = t == 0 ? reinterpret_cast<const T *>(p.x) + b * p.H * W * D
                                   : reinterpret_cast<const T *>(t == 1 ? p.d0 : p.d1) + b * p.dl_bs;
            f.src[u] = reinterpret_cast<const char *>(base + j * D + dch0 + part * EPC);
            f.rs[u] = W * D * ES;
            f.dst[u] = t * L::X + (col * kCh + part * EPC) * ES / 4;
            f.ok[u] = j < W;
        } else if (e < NX + NB) {
            const int e2 = e - NX, t = e2 / (kCPW * BC), r = e2 % (kCPW * BC);
            const int col = r / BC, q = r % BC;
            const long j = j0 + col;
            const T *base = reinterpret_cast<const T *>(t == 0 ? p.B : p.C) + b * p.H * W * M;
            f.src[u] = reinterpret_cast<const char *>(base + j * M + q * EPC);
            f.rs[u] = W * M * ES;
            f.dst[u] = 3 * L::X + t * L::Bn + (col * 16 + q * EPC) * ES / 4;
            f.ok[u] = j < W && q * EPC < M;
        } else {
            f.src[u] = reinterpret_cast<const char *>(p.x);
            f.rs[u] = 0;
            f.dst[u] = -1;
            f.ok[u] = false;
        }
    }
}

/* stages row i (rows are staged in order 0, 1, 2, ... once each: the
 * sources then move one row down) */
template <typename T>
__device__ __forceinline__ void stage_row_fast(const S2D &p, FwdCopies &f, long i, float *s,
                                               int lane, const float *edge_row) {
    const bool rok = i >= 0 && i < p.H;
    if (edge_row)
        kmb_cp_async16(s + FL<T>::E0 + lane * 4, rok ? edge_row + lane * 4 : p.x,
                       rok ? 16 : 0);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        if (f.dst[u] >= 0) {
            const bool ok = rok && f.ok[u];
            kmb_cp_async16(s + f.dst[u], ok ? (const void *)f.src[u] : (const void *)p.x,
                           ok ? 16 : 0);
            f.src[u] += f.rs[u];
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32, 2) k_scan2d_fwd(S2D p) {
    using L = FL<T>;
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long H = p.H, W = p.W, D = p.D, M = p.M;
    const bool qok = q * 4 < M;
    float *ring = sm + w * kRing * L::SLOT;                    /* this warp's rows */
    float *xbuf = sm + kWarps * kRing * L::SLOT;               /* [warp][2][32][4] */
    const long nstrips = (W + kStrip - 1) / kStrip;
    const long groups = D / kCh;
    __shared__ long item_sh;
    long b, g, s0, s1;
    for (long iter = 0; next_item(p, iter, nstrips, false, &item_sh, b, g, s0, s1); ++iter) {
    const long dch0 = g * kCh;
    const long d = dch0 + c;
    /* edge columns: one per (item, group), two alternating by strip
     * parity when strips are split over CTAs */
    float *const edge_base = p.edge + (b * groups + g) * (p.split ? 2 : 1) * H * 128;

    float2 A0p[2], A1p[2];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        const int m = q * 4 + 2 * jp;
        const float a0 = m < M ? p.A0[d * M + m] : 0.f, a1 = m + 1 < M ? p.A0[d * M + m + 1] : 0.f;
        const float e0 = m < M ? p.A1[d * M + m] : 0.f, e1 = m + 1 < M ? p.A1[d * M + m + 1] : 0.f;
        A0p[jp] = kmb_f2(a0 * KMB_LOG2E, a1 * KMB_LOG2E);
        A1p[jp] = kmb_f2(e0 * KMB_LOG2E, e1 * KMB_LOG2E);
    }
    const float amin0 = abs_min4(A0p), amin1 = abs_min4(A1p);
    const long nsteps = H + kWarps - 1;
    float *hb = p.hout + b * H * W * D * M;
    T *yb = reinterpret_cast<T *>(p.y) + b * H * W * D;

    for (long sidx = s0; sidx < s1; ++sidx) {
        float *const edge_rd = edge_base + (p.split ? ((sidx - 1) & 1) * H * 128 : 0);
        float *const edge_wr = edge_base + (p.split ? (sidx & 1) * H * 128 : 0);
        const int *prog_rd = p.split && sidx > 0 ? p.prog + ((sidx - 1) * p.batch + b) * groups + g
                                                 : nullptr;
        int *prog_wr = p.split ? p.prog + (sidx * p.batch + b) * groups + g : nullptr;
        const long j0 = sidx * kStrip + w * kCPW; /* this warp's first column */
        float2 hv[kCPW][2];                       /* h(i-1, j0 + k) */
#pragma unroll
        for (int k = 0; k < kCPW; ++k) hv[k][0] = hv[k][1] = kmb_f2s(0.f);
        /* the first warp of a strip also stages the previous strip's last
         * column, written by that strip's last warp (CTA barriers since) */
        const bool use_edge = w == 0 && sidx > 0;
        /* the edge row r of the previous strip; with the split, once its
         * CTA has published it */
        auto edge_row = [&](long r) -> const float * {
            if (!use_edge) return nullptr;
            if (prog_rd && r < H) wait_progress(prog_rd, (int)r + 1, lane);
            return edge_rd + r * 128;
        };
        FwdCopies fc;
        fwd_copies<T>(p, b, j0, dch0, lane, fc);
        /* h and y of this warp's first column at row 0; a row is W*D*M
         * (W*D) floats further */
        float *hcol = hb + (j0 * D + d) * M + q * 4;
        T *ycol = yb + j0 * D + d;
        const long hrow = W * D * M, yrow = W * D;
        const int hcolst = (int)(D * M), ycolst = (int)D; /* one column further */
        /* every column of this warp inside the grid and every lane's states
         * inside M: the per-point guards are all true */
        const bool full = j0 + kCPW <= W && M == 16;
        /* prologue: rows 0 .. kRing-2 of this warp */
#pragma unroll
        for (int r = 0; r < kRing - 1; ++r) {
            stage_row_fast<T>(p, fc, r, ring + r * L::SLOT, lane, edge_row(r));
            kmb_cp_async_commit();
        }
        int slot = 0; /* i % kRing once i >= 0 */
        for (long t = 0; t < nsteps; ++t) {
            const long i = t - w; /* this warp's row */
            /* row i + kRing - 1 goes into the slot row i - 1 used; rows below
             * kRing - 1 came with the prologue.  One commit per step keeps
             * the group count uniform. */
            if (i >= 0)
                stage_row_fast<T>(p, fc, i + kRing - 1,
                                  ring + (slot == 0 ? kRing - 1 : slot - 1) * L::SLOT, lane,
                                  edge_row(i + kRing - 1));
            kmb_cp_async_commit();
            kmb_cp_async_wait<kRing - 1>();
            __syncwarp();
            if (i >= 0 && i < H) {
                const float *s = ring + slot * L::SLOT;
                /* left neighbour of column j0 at row i */
                float2 hl[2];
                if (w > 0) {
                    const float4 v = *reinterpret_cast<const float4 *>(
                        xbuf + (((w - 1) * 2 + ((t - 1) & 1)) * 32 + lane) * 4);
                    hl[0] = kmb_f2(v.x, v.y);
                    hl[1] = kmb_f2(v.z, v.w);
                } else if (use_edge) {
                    const float4 v = *reinterpret_cast<const float4 *>(s + L::E0 + lane * 4);
                    hl[0] = kmb_f2(v.x, v.y);
                    hl[1] = kmb_f2(v.z, v.w);
                } else {
                    hl[0] = hl[1] = kmb_f2s(0.f);
                }
                /* this step's row of h / y (32-bit column offsets below) */
                float *const hrowp = hcol + i * hrow;
                T *const yrowp = ycol + i * yrow;
                auto points = [&](auto full_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
                float yq[4];
#pragma unroll
                for (int k = 0; k < kCPW; ++k) {
                    const long j = j0 + k;
                    const float xv = ldT<T>(s, k * kCh + c);
                    const float dv0 = ldT<T>(s + L::X, k * kCh + c);
                    const float dv1 = ldT<T>(s + 2 * L::X, k * kCh + c);
                    const float4 B4 = ld4T<T>(s + 3 * L::X, k * 16 + q * 4);
                    const float4 C4 = ld4T<T>(s + 3 * L::X + L::Bn, k * 16 + q * 4);
                    const float2 dtx2 = kmb_f2s((dv0 + dv1) / 2.0f * xv); /* dt_bar x */
                    const float2 dv02 = kmb_f2s(dv0), dv12 = kmb_f2s(dv1);
                    const float2 Bp[2] = {kmb_f2(B4.x, B4.y), kmb_f2(B4.z, B4.w)};
                    const float2 Cp[2] = {kmb_f2(C4.x, C4.y), kmb_f2(C4.z, C4.w)};
                    float2 y2 = kmb_f2s(0.f);
                    const float2 wv[4] = {kmb_mul2(dv02, A0p[0]), kmb_mul2(dv02, A0p[1]),
                                          kmb_mul2(dv12, A1p[0]), kmb_mul2(dv12, A1p[1])};
                    float2 ev[4];
                    exp2_decay_point(wv, ev, weak_possible(dv0, dv1, amin0, amin1, qok));
#pragma unroll
                    for (int jp = 0; jp < 2; ++jp) {
                        float2 hn = kmb_mul2(Bp[jp], dtx2);
                        const float2 e0 = ev[jp], e1 = ev[2 + jp];
                        hn = kmb_fma2(e0, hv[k][jp], hn);
                        hn = kmb_fma2(e1, hl[jp], hn);
                        hv[k][jp] = hn;
                        hl[jp] = hn;
                        y2 = kmb_fma2(Cp[jp], hn, y2);
                    }
                    if (FULL || (j < W && qok))
                        *reinterpret_cast<float4 *>(hrowp + k * hcolst) =
                            make_float4(hv[k][0].x, hv[k][0].y, hv[k][1].x, hv[k][1].y);
                    /* y: sum over the 4 state groups, 4 columns per fold */
                    yq[k & 3] = y2.x + y2.y;
                    if ((k & 3) == 3) {
#pragma unroll
                        for (int hh = 2; hh > 0; hh >>= 1) {
                            const bool up = (q & hh) != 0;
#pragma unroll
                            for (int u = 0; u < hh; ++u) {
                                const float send = up ? yq[u] : yq[u + hh];
                                const float keep = up ? yq[u + hh] : yq[u];
                                yq[u] = keep + __shfl_xor_sync(kFull, send, hh);
                            }
                        }
                        const long jy = j0 + (k - 3) + q;
                        if (FULL || jy < W) stT<T>(yrowp + ((k - 3) + q) * ycolst, yq[0]);
                    }
                }
                };
                if (full) points(std::true_type{});
                else points(std::false_type{});
                /* the last column's states go to the next warp (and, from
                 * the last warp, to the next strip) */
                const float4 last = make_float4(hl[0].x, hl[0].y, hl[1].x, hl[1].y);
                *reinterpret_cast<float4 *>(xbuf + ((w * 2 + (t & 1)) * 32 + lane) * 4) = last;
                if (w == kWarps - 1) {
                    *reinterpret_cast<float4 *>(edge_wr + i * 128 + lane * 4) = last;
                    if (prog_wr) publish_progress(prog_wr, (int)i + 1, lane);
                }
            }
            if (i >= 0) slot = slot == kRing - 1 ? 0 : slot + 1;
            __syncthreads();
        }
        kmb_cp_async_wait<0>();
        __syncthreads();
    }
    } /* work items */
}

/* ------------------------------------------------------------------ */
/* backward                                                            */
/* ------------------------------------------------------------------ */

constexpr int kBCPW = 4;                 /* columns per warp */
constexpr int kBStrip = kWarps * kBCPW;  /* columns per strip */
constexpr int kBRing = 3;                /* rows staged ahead per warp */
/* one staged row of a warp (floats): x, delta_0, delta_1, dy as [col][ch];
 * B, C as [col][16]; h of the row above [col][ch][16]; h of the column
 * left of the warp [ch][16]; the right-edge carry [32 lanes][4] */
constexpr int kBX = kBCPW * kCh;
constexpr int kBB = kBCPW * 16;
constexpr int kBH = kBCPW * kCh * 16;
constexpr int kBL = kCh * 16;
constexpr int kBE = 128;
constexpr int kBSlot = 4 * kBX + 2 * kBB + kBH + kBL + kBE;

/* The backward slot with inputs of element type T, offsets in floats:
 * x / delta_0 / delta_1 / dy regions of X floats, B / C regions of Bn,
 * then the fp32 h rows (H0), left h column (L0) and edge carry (E0). */
template <typename T> struct BL {
    static constexpr int X = kBX * (int)sizeof(T) / 4;
    static constexpr int Bn = kBB * (int)sizeof(T) / 4;
    static constexpr int H0 = 4 * X + 2 * Bn;
    static constexpr int L0 = H0 + kBH;
    static constexpr int E0 = L0 + kBL;
    static constexpr int SLOT = E0 + kBE;
};
static_assert(BL<float>::SLOT == kBSlot, "fp32 backward slot layout");

/* The backward's copies of one staged row, per lane, fixed for a strip:
 * one chunk of x / delta_0 / delta_1 / dy (lane / 8 picks the tensor), one
 * of B / C (lane / 16), and five of h: h(i-1, j0 + u) for u < 4 and
 * h(i, j0-1) for u = 4, all for channel lane / 4 and states 4 (lane % 4).
 * Sources are kept at row 0; a row further is W*D (inputs), W*M (B, C)
 * or W*D*M (h) floats. */
struct BwdCopies {
    const char *in, *bc;      /* sources at the next row staged */
    const float *h;
    long in_rs, bc_rs;        /* row strides in bytes: W*D, W*M elements */
    int h_rs;                 /* W*D*M floats */
    int h_col;                /* one column of h: D*M floats */
    int in_dst, bc_dst;       /* floats from the slot start; -1: no chunk */
    bool in_ok, bc_ok;
    unsigned h_ok; /* bit u: column of h chunk u inside the grid and q*4 < M */
};

/* Per lane one 16-byte chunk of the x / delta / dy rows (fp32: 4 tensors x
 * 4 columns x 2 chunks; bf16: 4 x 4 x 1, lanes 0-15), one of the B / C rows
 * (fp32: 2 x 4 columns x 4 chunks; bf16: 2 x 4 x 2, lanes 0-15) and five of
 * h (fp32 always). */
template <typename T>
__device__ __forceinline__ void bwd_copies(const S2D &p, long b, long j0, long dch0, int lane,
                                           BwdCopies &f) {
    using L = BL<T>;
    constexpr int ES = (int)sizeof(T), EPC = 16 / ES;
    constexpr int XC = kCh / EPC, BC = 16 / EPC;
    const long H = p.H, W = p.W, D = p.D, M = p.M;
    {
        const int t = lane / (kBCPW * XC), r = lane % (kBCPW * XC), col = r / XC, part = r % XC;
        const long j = j0 + col;
        const T *base = t == 0   ? reinterpret_cast<const T *>(p.x) + b * H * W * D
                        : t == 1 ? reinterpret_cast<const T *>(p.d0) + b * p.dl_bs
                        : t == 2 ? reinterpret_cast<const T *>(p.d1) + b * p.dl_bs
                                 : reinterpret_cast<const T *>(p.dy) + b * H * W * D;
        const bool live = lane < 4 * kBCPW * XC;
        f.in = reinterpret_cast<const char *>(base + j * D + dch0 + part * EPC);
        f.in_dst = live ? t * L::X + (col * kCh + part * EPC) * ES / 4 : -1;
        f.in_ok = live && j < W;
    }
    {
        const int t = lane / (kBCPW * BC), r = lane % (kBCPW * BC), col = r / BC, q = r % BC;
        const long j = j0 + col;
        const bool live = lane < 2 * kBCPW * BC;
        f.bc = reinterpret_cast<const char *>(reinterpret_cast<const T *>(t == 0 ? p.B : p.C) +
                                              b * H * W * M + j * M + q * EPC);
        f.bc_dst = live ? 4 * L::X + t * L::Bn + (col * 16 + q * EPC) * ES / 4 : -1;
        f.bc_ok = live && j < W && q * EPC < M;
    }
    const int ch = lane / 4, q = lane % 4;
    f.h = p.h + b * H * W * D * M + (j0 * D + dch0 + ch) * M + q * 4;
    f.in_rs = W * D * ES;
    f.bc_rs = W * M * ES;
    f.h_rs = (int)(W * D * M);
    f.h_col = (int)(D * M);
    /* rows are staged from the last one up */
    f.in += (H - 1) * f.in_rs;
    f.bc += (H - 1) * f.bc_rs;
    f.h += (H - 1) * W * D * M;
    f.h_ok = 0;
#pragma unroll
    for (int u = 0; u < kBCPW + 1; ++u) {
        const long j = u < kBCPW ? j0 + u : j0 - 1;
        if (j >= 0 && j < W && q * 4 < M) f.h_ok |= 1u << u;
    }
}

/* stages row i of this warp (columns j0 .. j0+3): inputs of row i, h of
 * row i-1 for the same columns and h(i, j0-1); zero outside the grid.
 * Rows are staged in order H-1, H-2, ... once each: the sources then move
 * one row up. */
template <typename T>
__device__ __forceinline__ void stage_row_bwd_fast(const S2D &p, BwdCopies &f, long i, float *s,
                                                   int lane, const float *edge_row) {
    using L = BL<T>;
    const bool rok = i >= 0 && i < p.H;
    if (edge_row)
        kmb_cp_async16(s + L::E0 + lane * 4, rok ? edge_row + lane * 4 : p.x, rok ? 16 : 0);
    if (sizeof(T) == 4 || f.in_dst >= 0) {
        const bool ok = rok && f.in_ok;
        kmb_cp_async16(s + f.in_dst, ok ? (const void *)f.in : (const void *)p.x, ok ? 16 : 0);
    }
    if (sizeof(T) == 4 || f.bc_dst >= 0) {
        const bool ok = rok && f.bc_ok;
        kmb_cp_async16(s + f.bc_dst, ok ? (const void *)f.bc : (const void *)p.x, ok ? 16 : 0);
    }
    const int ch = lane / 4, q = lane % 4;
    const float *hup = f.h - f.h_rs;
#pragma unroll
    for (int u = 0; u < kBCPW; ++u) {
        const bool ok = rok && i >= 1 && ((f.h_ok >> u) & 1);
        kmb_cp_async16(s + L::H0 + (u * kCh + ch) * 16 + q * 4,
                       ok ? hup + u * f.h_col : p.x, ok ? 16 : 0);
    }
    {
        const bool ok = rok && ((f.h_ok >> kBCPW) & 1);
        kmb_cp_async16(s + L::L0 + ch * 16 + q * 4,
                       ok ? f.h - f.h_col : p.x, ok ? 16 : 0);
    }
    f.in -= f.in_rs;
    f.bc -= f.bc_rs;
    f.h -= f.h_rs;
}

/* Reduce-scatter of 8 values over the 8 lanes that share q (lane bits 2-4):
 * afterwards lane 4c + q holds the sum of value 4 (c >> 2) + (c & 3). */
__device__ __forceinline__ float rs8_channels(float (&v)[8], int lane) {
#pragma unroll
    for (int o = 16, half = 4; o >= 4; o >>= 1, half >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (k < half) {
                const float send = up ? v[k] : v[k + half];
                const float keep = up ? v[k + half] : v[k];
                v[k] = keep + __shfl_xor_sync(kFull, send, o);
            }
        }
    }
    return v[0];
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32, 2) k_scan2d_bwd(S2D p) {
    using L = BL<T>;
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int c = lane >> 2, q = lane & 3;
    const long H = p.H, W = p.W, D = p.D, M = p.M;
    const bool qok = q * 4 < M;
    float *ring = sm + w * kBRing * L::SLOT;
    float *xbuf = sm + kWarps * kBRing * L::SLOT; /* [warp][2][32][4] */
    const long nstrips = (W + kBStrip - 1) / kBStrip;
    const long groups = D / kCh;
    __shared__ long item_sh;
    long b, g, s0, s1;
    for (long iter = 0; next_item(p, iter, nstrips, true, &item_sh, b, g, s0, s1); ++iter) {
    const long dch0 = g * kCh;
    const long d = dch0 + c;
    float *const edge_base = p.edge + (b * groups + g) * (p.split ? 2 : 1) * H * 128;

    float2 A0p[2], A1p[2], dA0[2], dA1[2];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        const int m = q * 4 + 2 * jp;
        const float a0 = m < M ? p.A0[d * M + m] : 0.f, a1 = m + 1 < M ? p.A0[d * M + m + 1] : 0.f;
        const float e0 = m < M ? p.A1[d * M + m] : 0.f, e1 = m + 1 < M ? p.A1[d * M + m + 1] : 0.f;
        A0p[jp] = kmb_f2(a0 * KMB_LOG2E, a1 * KMB_LOG2E);
        A1p[jp] = kmb_f2(e0 * KMB_LOG2E, e1 * KMB_LOG2E);
        dA0[jp] = dA1[jp] = kmb_f2s(0.f);
    }
    const float amin0 = abs_min4(A0p), amin1 = abs_min4(A1p);
    const long nsteps = H + kWarps - 1;
    const float *hb = p.h + b * H * W * D * M;
    T *dxb = reinterpret_cast<T *>(p.dx) + b * H * W * D;
    T *dd0b = reinterpret_cast<T *>(p.dd0) + b * p.dl_bs;
    T *dd1b = reinterpret_cast<T *>(p.dd1) + b * p.dl_bs;
    float *dBb = p.dB + b * H * W * M;
    float *dCb = p.dC + b * H * W * M;
    const int lead = kWarps - 1 - w; /* steps this warp runs behind the leader */

    for (long sidx = s1 - 1; sidx >= s0; --sidx) {
        /* the carry column comes from strip sidx + 1 (to the right) */
        float *const edge_rd = edge_base + (p.split ? ((sidx + 1) & 1) * H * 128 : 0);
        float *const edge_wr = edge_base + (p.split ? (sidx & 1) * H * 128 : 0);
        const int *prog_rd = p.split && sidx + 1 < nstrips
                                 ? p.prog + ((sidx + 1) * p.batch + b) * groups + g : nullptr;
        int *prog_wr = p.split ? p.prog + (sidx * p.batch + b) * groups + g : nullptr;
        const long j0 = sidx * kBStrip + w * kBCPW;
        /* step t handles row r(t) = H-1 - (t - lead) */
        auto row_of = [&](long t) { return H - 1 - (t - lead); };
        float2 qv[kBCPW][2];   /* e0(p) G(p) of the row below, per column */
        float2 hc[kBCPW][2];   /* h(i, j0 + k) of the current row */
#pragma unroll
        for (int k = 0; k < kBCPW; ++k) {
            qv[k][0] = qv[k][1] = kmb_f2s(0.f);
            const long j = j0 + k;
            if (j < W && qok) {
                const float4 v = *reinterpret_cast<const float4 *>(
                    hb + (((H - 1) * W + j) * D + d) * M + q * 4);
                hc[k][0] = kmb_f2(v.x, v.y);
                hc[k][1] = kmb_f2(v.z, v.w);
            } else {
                hc[k][0] = hc[k][1] = kmb_f2s(0.f);
            }
        }
        const bool use_edge = w == kWarps - 1 && sidx + 1 < nstrips;
        /* rows run bottom-up: row r is published once H - r rows are done */
        auto edge_row = [&](long r) -> const float * {
            if (!use_edge) return nullptr;
            if (prog_rd && r >= 0 && r < H) wait_progress(prog_rd, (int)(H - r), lane);
            return edge_rd + r * 128;
        };
        /* every column of this warp inside the grid and every lane's states
         * inside M: the per-point guards are all true */
        const bool full = j0 + kBCPW <= W && M == 16;
        BwdCopies bc;
        bwd_copies<T>(p, b, j0, dch0, lane, bc);
        /* prologue: the first kBRing-1 rows this warp will run (H-1, H-2, ..) */
#pragma unroll
        for (int r = 0; r < kBRing - 1; ++r) {
            stage_row_bwd_fast<T>(p, bc, H - 1 - r, ring + r * L::SLOT, lane, edge_row(H - 1 - r));
            kmb_cp_async_commit();
        }
        int slot = 0; /* n % kBRing once n >= 0 */
        for (long t = 0; t < nsteps; ++t) {
            const long n = t - lead; /* rows this warp has done before this step */
            if (n >= 0) {
                const long nr = n + kBRing - 1;
                stage_row_bwd_fast<T>(p, bc, H - 1 - nr,
                                      ring + (slot == 0 ? kBRing - 1 : slot - 1) * L::SLOT, lane,
                                      edge_row(H - 1 - nr));
            }
            kmb_cp_async_commit();
            kmb_cp_async_wait<kBRing - 1>();
            __syncwarp();
            const long i = row_of(t);
            if (n >= 0 && i >= 0) {
                const float *s = ring + slot * L::SLOT;
                /* carry from the right neighbour column: e1(p+1) G(p+1) */
                float2 qh[2];
                if (w < kWarps - 1) {
                    const float4 v = *reinterpret_cast<const float4 *>(
                        xbuf + (((w + 1) * 2 + ((t - 1) & 1)) * 32 + lane) * 4);
                    qh[0] = kmb_f2(v.x, v.y);
                    qh[1] = kmb_f2(v.z, v.w);
                } else if (use_edge) {
                    const float4 v = *reinterpret_cast<const float4 *>(s + L::E0 + lane * 4);
                    qh[0] = kmb_f2(v.x, v.y);
                    qh[1] = kmb_f2(v.z, v.w);
                } else {
                    qh[0] = qh[1] = kmb_f2s(0.f);
                }
                /* offsets of (i, j0): channel d in [P, D] tensors, states
                 * 4q.. in [P, M] ones */
                const long ox = (i * W + j0) * D + d, obc = (i * W + j0) * M + q * 4;
                T *const dxr = dxb + ox, *const dd0r = dd0b + ox, *const dd1r = dd1b + ox;
                auto points = [&](auto full_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
                for (int k = kBCPW - 1; k >= 0; --k) {
                    const long j = j0 + k;
                    const float xv = ldT<T>(s, k * kCh + c);
                    const float dv0 = ldT<T>(s + L::X, k * kCh + c);
                    const float dv1 = ldT<T>(s + 2 * L::X, k * kCh + c);
                    const float gy = ldT<T>(s + 3 * L::X, k * kCh + c);
                    const float4 B4 = ld4T<T>(s + 4 * L::X, k * 16 + q * 4);
                    const float4 C4 = ld4T<T>(s + 4 * L::X + L::Bn, k * 16 + q * 4);
                    const float4 H0 = *reinterpret_cast<const float4 *>(
                        s + L::H0 + (k * kCh + c) * 16 + q * 4); /* h(i-1, j) */
                    float2 hl[2]; /* h(i, j-1) */
                    if (k > 0) {
                        hl[0] = hc[k > 0 ? k - 1 : 0][0];
                        hl[1] = hc[k > 0 ? k - 1 : 0][1];
                    } else {
                        const float4 v = *reinterpret_cast<const float4 *>(
                            s + L::L0 + c * 16 + q * 4);
                        hl[0] = kmb_f2(v.x, v.y);
                        hl[1] = kmb_f2(v.z, v.w);
                    }
                    const float2 hu[2] = {kmb_f2(H0.x, H0.y), kmb_f2(H0.z, H0.w)};
                    const float2 Bp[2] = {kmb_f2(B4.x, B4.y), kmb_f2(B4.z, B4.w)};
                    const float2 Cp[2] = {kmb_f2(C4.x, C4.y), kmb_f2(C4.z, C4.w)};
                    const float dtb = (dv0 + dv1) / 2.0f;
                    /* dB(p, m) gets G dt_bar x: one product per point */
                    const float2 dtx2 = kmb_f2s(dtb * xv), gy2 = kmb_f2s(gy);
                    const float2 dv02 = kmb_f2s(dv0), dv12 = kmb_f2s(dv1);
                    float2 gb2 = kmb_f2s(0.f), s02 = kmb_f2s(0.f), s12 = kmb_f2s(0.f);
                    float vbc[8];
                    const float2 wv[4] = {kmb_mul2(dv02, A0p[0]), kmb_mul2(dv02, A0p[1]),
                                          kmb_mul2(dv12, A1p[0]), kmb_mul2(dv12, A1p[1])};
                    float2 ev[4];
                    exp2_decay_point(wv, ev, weak_possible(dv0, dv1, amin0, amin1, qok));
#pragma unroll
                    for (int jp = 0; jp < 2; ++jp) {
                        const float2 e0 = ev[jp], e1 = ev[2 + jp];
                        const float2 G = kmb_add2(kmb_fma2(Cp[jp], gy2, qv[k][jp]), qh[jp]);
                        gb2 = kmb_fma2(G, Bp[jp], gb2); /* sum_m G B */
                        /* carries to the point above and to the left; the
                         * h-weighted terms reuse them: G h e = (e G) h */
                        qv[k][jp] = kmb_mul2(e0, G);
                        qh[jp] = kmb_mul2(e1, G);
                        const float2 gh0 = kmb_mul2(qv[k][jp], hu[jp]);
                        const float2 gh1 = kmb_mul2(qh[jp], hl[jp]);
                        dA0[jp] = kmb_fma2(gh0, dv02, dA0[jp]);
                        dA1[jp] = kmb_fma2(gh1, dv12, dA1[jp]);
                        s02 = kmb_fma2(gh0, A0p[jp], s02); /* log2(e) A_0: scaled by ln 2 below */
                        s12 = kmb_fma2(gh1, A1p[jp], s12);
                        const float2 vb = kmb_mul2(G, dtx2);        /* dB */
                        const float2 vc = kmb_mul2(gy2, hc[k][jp]); /* dC */
                        vbc[2 * jp] = vb.x;
                        vbc[2 * jp + 1] = vb.y;
                        vbc[4 + 2 * jp] = vc.x;
                        vbc[4 + 2 * jp + 1] = vc.y;
                    }
                    /* sums over the 16 states (4 lanes): dx = dt_bar sum G B,
                     * the x-term of ddelta = x sum G B / 2 */
                    float gb = gb2.x + gb2.y;
                    float s0 = s02.x + s02.y, s1 = s12.x + s12.y;
#pragma unroll
                    for (int o = 1; o <= 2; o <<= 1) {
                        gb += __shfl_xor_sync(kFull, gb, o);
                        s0 += __shfl_xor_sync(kFull, s0, o);
                        s1 += __shfl_xor_sync(kFull, s1, o);
                    }
                    const float sx = dtb * gb, sb = xv * gb;
                    /* dB / dC: sums over the 8 channels, then 4 states into
                     * one lane for a 128-bit atomic */
                    float v8[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) v8[u] = vbc[u];
                    const float r1 = rs8_channels(v8, lane);
                    /* lane 16 arr + 4 st + q holds state 4q + st of array arr */
                    const float r2 = __shfl_down_sync(kFull, r1, 4);
                    const float r3 = __shfl_down_sync(kFull, r1, 8);
                    const float r4 = __shfl_down_sync(kFull, r1, 12);
                    if (FULL || j < W) {
                        if (q == 0) {
                            stT<T>(dxr + k * D, sx);
                            stT<T>(dd0r + k * D, s0 * KMB_LN2 + sb / 2.0f);
                            stT<T>(dd1r + k * D, s1 * KMB_LN2 + sb / 2.0f);
                        }
                        if ((c & 3) == 0 && (FULL || qok)) {
                            float *dst = ((c >> 2) ? dCb : dBb) + obc + k * M;
                            atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(r1, r2, r3, r4));
                        }
                    }
                }
                };
                if (full) points(std::true_type{});
                else points(std::false_type{});
                /* hand the carries on: the left neighbour warp (next step) and
                 * the next strip (its last warp) get e1 G of column j0 */
                const float4 outq = make_float4(qh[0].x, qh[0].y, qh[1].x, qh[1].y);
                *reinterpret_cast<float4 *>(xbuf + ((w * 2 + (t & 1)) * 32 + lane) * 4) = outq;
                if (w == 0) {
                    *reinterpret_cast<float4 *>(edge_wr + i * 128 + lane * 4) = outq;
                    if (prog_wr) publish_progress(prog_wr, (int)(H - i), lane);
                }
                /* h of row i-1 becomes the current row */
#pragma unroll
                for (int k = 0; k < kBCPW; ++k) {
                    const float4 v = *reinterpret_cast<const float4 *>(
                        s + L::H0 + (k * kCh + c) * 16 + q * 4);
                    hc[k][0] = kmb_f2(v.x, v.y);
                    hc[k][1] = kmb_f2(v.z, v.w);
                }
            }
            if (n >= 0) slot = slot == kBRing - 1 ? 0 : slot + 1;
            __syncthreads();
        }
        kmb_cp_async_wait<0>();
        __syncthreads();
    }
    const float dAs0[4] = {dA0[0].x, dA0[0].y, dA0[1].x, dA0[1].y};
    const float dAs1[4] = {dA1[0].x, dA1[0].y, dA1[1].x, dA1[1].y};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        if (q * 4 + u < M) {
            atomicAdd(p.dA0 + d * M + q * 4 + u, dAs0[u]);
            atomicAdd(p.dA1 + d * M + q * 4 + u, dAs1[u]);
        }
    }
    } /* work items */
}

} // namespace

extern "C" int kmb_scan2d_supported(const KmbNDLaunch *a) {
    return a->nd == 2 && a->bc_shared && a->M % 4 == 0 && a->M <= 16 && a->D % kCh == 0 &&
           a->dims[0] > 0 && a->dims[1] > 0 && a->D * a->M < (1L << 24);
}

static S2D make_s2d(const KmbNDLaunch *a) {
    S2D p;
    memset(&p, 0, sizeof p);
    p.x = a->x;
    p.d0 = a->delta[0];
    p.d1 = a->delta[1];
    p.A0 = a->A[0];
    p.A1 = a->A[1];
    p.B = a->B;
    p.C = a->C;
    p.dy = a->dy;
    p.H = a->dims[0];
    p.W = a->dims[1];
    p.D = a->D;
    p.M = a->M;
    p.dl_bs = a->delta_bstride;
    return p;
}

/* Scratch layout (floats): two edge columns (H rows x 32 lanes x 4 states)
 * per (item, channel group), then the strip-split progress counters (one
 * int per (strip, item, group), backward strips being the narrower) and the
 * work counter. */
static size_t edge_elems(const KmbNDLaunch *a) {
    return (size_t)a->batch * (a->D / kCh) * a->dims[0] * 128 * 2;
}
static size_t prog_ints(const KmbNDLaunch *a) {
    return (size_t)a->batch * (a->D / kCh) * ((a->dims[1] + kBStrip - 1) / kBStrip) + 1;
}

extern "C" size_t kmb_scan2d_scratch_elems(const KmbNDLaunch *a) {
    return edge_elems(a) + prog_ints(a) + 4;
}

namespace {

/* Strips split over CTAs (persistent CTAs taking (item, group, strip) work
 * items) when the items and channel groups alone leave SMs idle.  Config 4
 * (256 x 256, 32 groups per item), forward / backward ms whole -> split:
 * batch 1 1.95 / 5.23 -> 0.89 / 1.79, batch 2 1.94 / 5.33 -> 1.60 / 2.74,
 * batch 4 1.95 / 5.40 -> 2.19 / 4.46, batch 8 2.76 / 7.26 -> 3.61 / 7.60;
 * hence the forward splits up to half an SM's worth of groups, the
 * backward up to one per SM (`max_per_sm` x SMs).  KMB_SCAN2D_SPLIT=0 / 1
 * forces it off / on. */
bool split_wanted(long item_groups, long nstrips, int sms, double max_per_sm) {
    const char *e = getenv("KMB_SCAN2D_SPLIT");
    if (e && e[0] == '0' && e[1] == 0) return false;
    if (e && e[0] == '1' && e[1] == 0) return nstrips > 1;
    return nstrips > 1 && (double)item_groups <= max_per_sm * sms;
}

int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 148;
    }
    return n;
}

/* Grid of a launch: (groups, batch) CTAs, or with the split as many
 * persistent CTAs as fit (at most one per work item). */
template <typename K>
cudaError_t plan_grid(K kern, size_t smem, S2D &p, const KmbNDLaunch *a, long nstrips,
                      double max_per_sm, dim3 &grid, cudaStream_t s) {
    const long groups = a->D / kCh;
    const int sms = sm_count();
    p.batch = a->batch;
    p.split = split_wanted(a->batch * groups, nstrips, sms, max_per_sm) ? 1 : 0;
    p.prog = reinterpret_cast<int *>(a->scratch + edge_elems(a));
    p.work = p.prog + prog_ints(a) - 1;
    if (!p.split) {
        grid = dim3((unsigned)groups, (unsigned)a->batch);
        return cudaSuccess;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem);
    if (e != cudaSuccess) return e;
    const long items = nstrips * a->batch * groups;
    long ctas = (long)(per_sm > 0 ? per_sm : 1) * sms;
    if (ctas > items) ctas = items;
    grid = dim3((unsigned)ctas, 1);
    return cudaMemsetAsync(p.prog, 0, sizeof(int) * prog_ints(a), s);
}

__global__ void k_f32_to_bf16_2d(const float *src, __nv_bfloat16 *dst, long n) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

template <typename T>
int launch_fwd(const KmbNDLaunch *a, cudaStream_t s) {
    if (!kmb_scan2d_supported(a)) return kmb_fail(KMB_EUNSUPPORTED, "scan2d: unsupported shape");
    if (!a->scratch || a->scratch_elems < kmb_scan2d_scratch_elems(a))
        return kmb_fail(KMB_EINVAL, "scan2d: scratch too small");
    S2D p = make_s2d(a);
    p.hout = a->h;
    p.y = a->y;
    p.edge = a->scratch;
    const size_t smem = sizeof(float) * ((size_t)kWarps * kRing * FL<T>::SLOT + kWarps * 2 * 32 * 4);
    cudaError_t e = cudaFuncSetAttribute(k_scan2d_fwd<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    dim3 grid;
    if (e == cudaSuccess)
        e = plan_grid(k_scan2d_fwd<T>, smem, p, a, (a->dims[1] + kStrip - 1) / kStrip, 0.5, grid, s);
    if (e == cudaSuccess) {
        k_scan2d_fwd<T><<<grid, kWarps * 32, smem, s>>>(p);
        e = cudaGetLastError();
    }
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "scan2d forward");
}

/* dB32 / dC32: the fp32 buffers the channel sums are accumulated in (the
 * outputs themselves for fp32). */
template <typename T>
int launch_bwd(const KmbNDLaunch *a, float *dB32, float *dC32, cudaStream_t s) {
    if (!kmb_scan2d_supported(a)) return kmb_fail(KMB_EUNSUPPORTED, "scan2d: unsupported shape");
    if (!a->scratch || a->scratch_elems < kmb_scan2d_scratch_elems(a))
        return kmb_fail(KMB_EINVAL, "scan2d: scratch too small");
    S2D p = make_s2d(a);
    p.h = a->h;
    p.edge = a->scratch;
    p.dx = a->dx;
    p.dd0 = a->ddelta[0];
    p.dd1 = a->ddelta[1];
    p.dA0 = a->dA[0];
    p.dA1 = a->dA[1];
    p.dB = dB32;
    p.dC = dC32;
    cudaError_t e = cudaMemsetAsync(a->dA[0], 0, sizeof(float) * a->D * a->M, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(a->dA[1], 0, sizeof(float) * a->D * a->M, s);
    const size_t nb = sizeof(float) * a->batch * a->P * a->M;
    if (e == cudaSuccess) e = cudaMemsetAsync(dB32, 0, nb, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dC32, 0, nb, s);
    const size_t smem = sizeof(float) * ((size_t)kWarps * kBRing * BL<T>::SLOT + kWarps * 2 * 32 * 4);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_scan2d_bwd<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
    dim3 grid;
    if (e == cudaSuccess)
        e = plan_grid(k_scan2d_bwd<T>, smem, p, a, (a->dims[1] + kBStrip - 1) / kBStrip, 1.0, grid,
                      s);
    if (e == cudaSuccess) {
        k_scan2d_bwd<T><<<grid, kWarps * 32, smem, s>>>(p);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && sizeof(T) == 2) {
        const long n = a->batch * a->P * a->M;
        const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
        k_f32_to_bf16_2d<<<blocks, 256, 0, s>>>(dB32, reinterpret_cast<__nv_bfloat16 *>(a->dB), n);
        k_f32_to_bf16_2d<<<blocks, 256, 0, s>>>(dC32, reinterpret_cast<__nv_bfloat16 *>(a->dC), n);
        e = cudaGetLastError();
    }
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "scan2d backward");
}

} // namespace

extern "C" int kmb_launch_scan2d_fwd(const KmbNDLaunch *a, cudaStream_t s) {
    return launch_fwd<float>(a, s);
}

extern "C" int kmb_launch_scan2d_bwd(const KmbNDLaunch *a, cudaStream_t s) {
    return launch_bwd<float>(a, a->dB, a->dC, s);
}

/* bf16 tensors: the 16-byte staging chunks hold 8 states, so M must be 8
 * or 16. */
extern "C" int kmb_scan2d_bf16_supported(const KmbNDLaunch *a) {
    return kmb_scan2d_supported(a) && a->M % 8 == 0;
}

extern "C" int kmb_launch_scan2d_fwd_bf16(const KmbNDLaunch *a, cudaStream_t s) {
    if (!kmb_scan2d_bf16_supported(a)) return kmb_fail(KMB_EUNSUPPORTED, "scan2d bf16: unsupported shape");
    return launch_fwd<__nv_bfloat16>(a, s);
}

extern "C" int kmb_launch_scan2d_bwd_bf16(const KmbNDLaunch *a, float *dB32, float *dC32,
                                          cudaStream_t s) {
    if (!kmb_scan2d_bf16_supported(a)) return kmb_fail(KMB_EUNSUPPORTED, "scan2d bf16: unsupported shape");
    return launch_bwd<__nv_bfloat16>(a, dB32, dC32, s);
}

namespace {
__global__ void k_bf16_to_f32(const __nv_bfloat16 *src, float *dst, long n) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dst[i] = __bfloat162float(src[i]);
}
unsigned conv_blocks(long n) { return (unsigned)((n + 255) / 256 < 8192 ? (n + 255) / 256 : 8192); }
} // namespace

extern "C" int kmb_launch_bf16_to_f32(const void *src, float *dst, long n, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    k_bf16_to_f32<<<conv_blocks(n), 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(src), dst, n);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "bf16 -> fp32");
}

extern "C" int kmb_launch_f32_to_bf16(const float *src, void *dst, long n, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    k_f32_to_bf16_2d<<<conv_blocks(n), 256, 0, s>>>(src, static_cast<__nv_bfloat16 *>(dst), n);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "fp32 -> bf16");
}

/* KMB_ETIMEOUT (and the word cleared) when a strip-split wait gave up
 * since the last check. */
extern "C" int kmb_scan2d_check_error(void) {
    int flag = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&flag, g_scan2d_error, sizeof flag);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan2d: error word");
    if (flag) {
        const int zero = 0;
        (void)cudaMemcpyToSymbol(g_scan2d_error, &zero, sizeof zero);
        return kmb_fail(KMB_ETIMEOUT, "scan2d: a wait on another strip's progress expired");
    }
    return KMB_OK;
}
