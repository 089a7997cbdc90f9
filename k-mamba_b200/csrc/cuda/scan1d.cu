/*
 * 1D selective scan, forward and backward, for sm_100a.
 *
 * Recurrence (reference cpu/scan1d.asm:88-152, cuda/scan1d.cu:57-89):
 *   h_t[d,n] = exp(dt_t[d]*A[d,n]) * h_{t-1}[d,n] + dt_t[d]*B_t[n]*x_t[d]
 *   y_t[d]   = sum_n C_t[n] * h_t[d,n]
 * Backward = the reverse adjoint of cpu/scan1d_backward.c:248-295.
 *
 * Work decomposition.  The recurrence is sequential in t and independent
 * per (batch, channel, state): every (b, d) owns P lanes and every lane
 * owns G = 4 consecutive states, i.e. 4 independent chains over the whole
 * sequence.  A CTA of 128 threads covers DT = 128/P channels of one batch
 * item.  Per step and state the forward costs one MUFU ex2 plus four
 * FMA-pipe operations: exp(dt*A) is fused (A is pre-scaled by log2 e) and
 * no [L,D,N] temporary reaches memory unless the caller asks for h_all.
 *
 * Inputs are staged through shared memory by a 3-stage cp.async pipeline
 * (x, dt as [TT][DT] tiles; B, C as [TT][N] rows when shared across
 * channels).  Full tiles run fully unrolled: every P steps the P lanes of
 * a channel fold their partial y values with a reduce-scatter (P-1
 * shuffles for P outputs), the result goes to a shared [TT][DT] tile that
 * is written to global memory with coalesced 128-bit stores.
 *
 * The backward walks the sequence in reverse in chunks of
 * KMB_SCAN1D_CHUNK steps.  Each chunk re-runs the forward from the state
 * the forward checkpointed at the chunk start (or reads h from h_all),
 * keeps the chunk's states in registers and sweeps it backwards carrying
 * the adjoint g = dL/dh.  With q = (g + dy C) a and qh = q h_{t-1}:
 *   dA += dt qh,  ddt = sum_n A qh + x sum_n (g + dy C) B,
 *   dx = dt sum_n (g + dy C) B,  dB = (g + dy C) dt x,  dC = dy h.
 * dx / ddt fold across the P lanes with a batched reduce-scatter; when
 * B and C are shared across channels dB / dC are channel sums: a shuffle
 * reduce-scatter folds the warp's channels, shared memory folds the CTA's
 * warps and one 128-bit atomic per (step, 4 states, CTA) folds the CTAs.
 */
#include <stdlib.h>

#include <type_traits>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

constexpr int kNT = 128;   /* threads per CTA */
constexpr int kG = 4;      /* states per lane */
constexpr int kChunk = KMB_SCAN1D_CHUNK;
constexpr unsigned kFull = 0xffffffffu;

struct Scan1DDev {
    const float *x, *dt, *A, *B, *C, *h0;
    float *y, *h_last, *h_all, *ckpt;
    const float *dy;
    float *dx, *ddt, *dA, *dB, *dC;
    const float *ckpt_in;
    long L, D, N, nslots;
    int vec_xd;   /* x / dt / dy / y rows can use 16-byte accesses */
    int vec_bc;   /* B / C rows can use 16-byte accesses */
};

__device__ __forceinline__ float clamp1000(float v) {
    /* min first, then max: NaN becomes +1000 as with SSE minss/maxss. */
    return fmaxf(fminf(v, 1000.f), -1000.f);
}

template <bool VEC>
__device__ __forceinline__ void lds4(const float *row, bool gok, int N, int n0,
                                     float (&v)[kG]) {
    if (VEC) {
        if (gok) {
            const float4 t = *reinterpret_cast<const float4 *>(row);
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
            v[0] = v[1] = v[2] = v[3] = 0.f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < kG; ++j) v[j] = (n0 + j < N) ? row[j] : 0.f;
    }
}

template <bool VEC>
__device__ __forceinline__ void stg4(float *dst, bool gok, int N, int n0, const float (&v)[kG]) {
    if (VEC) {
        if (gok) *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
        for (int j = 0; j < kG; ++j)
            if (n0 + j < N) dst[j] = v[j];
    }
}

template <bool VEC>
__device__ __forceinline__ void ldg4(const float *src, bool gok, int N, int n0, float (&v)[kG]) {
    if (VEC) {
        if (gok) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(src));
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
            v[0] = v[1] = v[2] = v[3] = 0.f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < kG; ++j) v[j] = (n0 + j < N) ? __ldg(src + j) : 0.f;
    }
}

/* Reduce-scatter of P values across P consecutive lanes: on return lane
 * (lane % P) holds the group sum of value index (lane % P).  P - 1
 * shuffles in total. */
template <int P>
__device__ __forceinline__ float rs_sum(float (&v)[P], int lane) {
#pragma unroll
    for (int h = P / 2; h > 0; h >>= 1) {
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

__host__ __device__ inline int bc_row_stride(bool shared, int np, int N) {
    /* Shared-memory floats per step row of channel-shared B (or C): at
     * least the np = 4*P states the lanes cover, zero-filled past N, so
     * every lane reads its 4 states with one unconditional 128-bit load.
     * Per-channel B/C ([.., L, D, N]) are read straight from global memory:
     * the lanes of a warp cover consecutive channels, so each step's rows
     * are contiguous and the loads coalesce without staging. */
    const int n4 = (N + 3) & ~3;
    return shared ? (n4 > np ? n4 : np) : 0;
}

/* 4 consecutive states of a padded shared-memory row (16-byte aligned). */
__device__ __forceinline__ void lds4u(const float *row, float (&v)[kG]) {
    const float4 t = *reinterpret_cast<const float4 *>(row);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}

/* G-state versions of the helpers above, for the forward kernel that runs
 * with 2 or 4 states per lane. */
template <int G>
__device__ __forceinline__ void ldsv(const float *row, float (&v)[G]) {
    if constexpr (G == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(row);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
        static_assert(G == 2, "2 or 4 states per lane");
        const float2 t = *reinterpret_cast<const float2 *>(row);
        v[0] = t.x; v[1] = t.y;
    }
}

template <int G, bool VEC>
__device__ __forceinline__ void ldgv(const float *src, bool gok, int N, int n0, float (&v)[G]) {
    if constexpr (G == 4) {
        ldg4<VEC>(src, gok, N, n0, v);
    } else {
        if (VEC) {
            if (gok) {
                const float2 t = __ldg(reinterpret_cast<const float2 *>(src));
                v[0] = t.x; v[1] = t.y;
            } else {
                v[0] = v[1] = 0.f;
            }
        } else {
#pragma unroll
            for (int j = 0; j < G; ++j) v[j] = (n0 + j < N) ? __ldg(src + j) : 0.f;
        }
    }
}

template <int G, bool VEC>
__device__ __forceinline__ void stgv(float *dst, bool gok, int N, int n0, const float (&v)[G]) {
    if constexpr (G == 4) {
        stg4<VEC>(dst, gok, N, n0, v);
    } else {
        if (VEC) {
            if (gok) *reinterpret_cast<float2 *>(dst) = make_float2(v[0], v[1]);
        } else {
#pragma unroll
            for (int j = 0; j < G; ++j)
                if (n0 + j < N) dst[j] = v[j];
        }
    }
}

/* ------------------------------------------------------------------ */
/* forward                                                             */
/* ------------------------------------------------------------------ */

template <int P, bool SHARED>
struct FwdCfg {
    static constexpr int DT = kNT / P;
    static constexpr int TT = SHARED ? 32 : 16;
    static constexpr int ST = 3;
};

template <int P, int G, bool SHARED, bool VEC, bool CLAMP>
__global__ void __launch_bounds__(kNT, 3) k_scan1d_fwd(Scan1DDev p) {
    using Cfg = FwdCfg<P, SHARED>;
    constexpr int DT = Cfg::DT, TT = Cfg::TT, ST = Cfg::ST;
    static_assert(TT % P == 0 && TT % kChunk == 0, "tile must hold whole groups");
    extern __shared__ __align__(16) float smem[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int g = tid % P;
    const int dl = tid / P;
    const int n0 = g * G;
    const long b = blockIdx.y;
    const long D = p.D, L = p.L;
    const int N = (int)p.N;
    const long d0 = (long)blockIdx.x * DT;
    const long d = d0 + dl;
    const bool dok = d < D;
    const bool gok = n0 < N;
    const int dvalid = (int)min((long)DT, D - d0);

    /* shared-memory row of channel-shared B / C: bc_row_stride(true, G*P, N),
     * which is G*P (at least 4) for every N the launcher maps to this P */
    constexpr int BW = SHARED ? (G * P >= 4 ? G * P : 4) : 0;
    constexpr int xs_sz = TT * DT;
    constexpr int bs_sz = TT * BW;
    constexpr int stage_sz = 3 * xs_sz + 2 * bs_sz; /* x, dt, y, B, C */

    float A2[G], h[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        const bool ok = dok && n0 + j < N;
        A2[j] = ok ? __ldg(p.A + d * N + n0 + j) * KMB_LOG2E : 0.f;
        h[j] = (ok && p.h0) ? p.h0[(b * D + d) * N + n0 + j] : 0.f;
    }

    const long xoff = b * L * D + d0;
    const float *xg = p.x + xoff;
    const float *dg = p.dt + xoff;
    const long bld = SHARED ? (long)N : D * N;
    const long boff = SHARED ? b * L * N : (b * L * D + d0) * N;
    const float *Bg = p.B + boff;
    const float *Cg = p.C + boff;
    const bool vxd = p.vec_xd, vbc = p.vec_bc;
    float *const hall = p.h_all ? p.h_all + (b * L * D + d) * N + n0 : nullptr;
    float *const ckpt = p.ckpt ? p.ckpt + (b * p.nslots * D + d) * N + n0 : nullptr;
    const long hstride = D * N; /* one step in h_all, one slot in ckpt */

    const int ntiles = (int)((L + TT - 1) / TT);
    auto load = [&](int k) {
        float *st = smem + (k % ST) * stage_sz;
        const long t0 = (long)k * TT;
        const int rv = (int)min((long)TT, L - t0);
        kmb_load_tile_c<kNT, TT, DT>(st, DT, xg + t0 * D, D, rv, dvalid, vxd, tid);
        kmb_load_tile_c<kNT, TT, DT>(st + xs_sz, DT, dg + t0 * D, D, rv, dvalid, vxd, tid);
        if constexpr (SHARED) {
            /* columns past N are zero-filled */
            kmb_load_tile_c<kNT, TT, BW>(st + 3 * xs_sz, BW, Bg + t0 * bld, bld, rv, N, vbc,
                                         tid);
            kmb_load_tile_c<kNT, TT, BW>(st + 3 * xs_sz + bs_sz, BW, Cg + t0 * bld, bld, rv, N,
                                         vbc, tid);
        }
    };
    /* coalesced store of the y tile of tile k (rows rv, channels dvalid) */
    auto flush_y = [&](int k) {
        const float *ys = smem + (k % ST) * stage_sz + 2 * xs_sz;
        const long t0 = (long)k * TT;
        const int rv = (int)min((long)TT, L - t0);
        float *yg = p.y + b * L * D + t0 * D + d0;
        if (vxd) {
            constexpr int C4 = DT / 4;
            for (int e = tid; e < rv * C4; e += kNT) {
                const int r = e / C4, c = (e - r * C4) * 4;
                if (c < dvalid)
                    *reinterpret_cast<float4 *>(yg + (long)r * D + c) =
                        *reinterpret_cast<const float4 *>(ys + r * DT + c);
            }
        } else {
            for (int e = tid; e < rv * DT; e += kNT) {
                const int r = e / DT, c = e - r * DT;
                if (c < dvalid) yg[(long)r * D + c] = ys[r * DT + c];
            }
        }
    };

#pragma unroll
    for (int k = 0; k < ST - 1; ++k) {
        if (k < ntiles) load(k);
        kmb_cp_async_commit();
    }

    const int brow = n0;
    /* per-channel B/C row of this lane at step 0 (SHARED == false) */
    const float *bgl = SHARED ? nullptr : p.B + (b * L * D + d) * N + n0;
    const float *cgl = SHARED ? nullptr : p.C + (b * L * D + d) * N + n0;
    for (int k = 0; k < ntiles; ++k) {
        kmb_cp_async_wait<ST - 2>();
        __syncthreads();
        if (k > 0 && p.y) flush_y(k - 1);
        if (k + ST - 1 < ntiles) load(k + ST - 1);
        kmb_cp_async_commit();

        const float *st = smem + (k % ST) * stage_sz;
        const float *xs = st + dl;
        const float *ds = st + xs_sz + dl;
        float *ys = const_cast<float *>(st) + 2 * xs_sz + dl;
        const float *bs = st + 3 * xs_sz + brow;
        const float *cs = bs + bs_sz;
        const long t0 = (long)k * TT;
        const int rv = (int)min((long)TT, L - t0);

        /* exact path: partial last tile, or a tile the clamp detector flagged */
        auto slow_tile = [&](int rows) {
            for (int i = 0; i < rows; ++i) {
                const float dv = ds[i * DT];
                const float u = dv * xs[i * DT];
                float bv[G], cv[G];
                if (SHARED) {
                    ldsv<G>(bs + i * BW, bv);
                    ldsv<G>(cs + i * BW, cv);
                } else {
                    ldgv<G, VEC>(bgl + (t0 + i) * hstride, gok && dok, N, dok ? n0 : N, bv);
                    ldgv<G, VEC>(cgl + (t0 + i) * hstride, gok && dok, N, dok ? n0 : N, cv);
                }
                float yp = 0.f;
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    const float a = kmb_exp2_decay(dv * A2[j]);
                    float hn = fmaf(a, h[j], bv[j] * u);
                    if (CLAMP) hn = clamp1000(hn);
                    h[j] = hn;
                    yp = fmaf(cv[j], hn, yp);
                }
#pragma unroll
                for (int o = P / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(kFull, yp, o);
                if (g == 0) ys[i * DT] = yp;
                if (hall && dok) stgv<G, VEC>(hall + (t0 + i) * hstride, gok, N, n0, h);
                if (((i + 1) & (kChunk - 1)) == 0 && ckpt && dok)
                    stgv<G, VEC>(ckpt + ((t0 + i) / kChunk) * hstride, gok, N, n0, h);
            }
        };

        if (rv == TT && !hall) {
            /* fast path: no clamp on the critical path; a detector sums h^2
             * over the tile (any |h| > 1000, or a NaN, pushes the sum to at
             * least 1e6) and a flagged tile is replayed exactly from its
             * start.  The tile is straight-line code: decays are
             * kmb_exp2_decay2 (MUFU ex2 and the weak-decay polynomial,
             * selected per element), because a warp-uniform branch per step
             * that skips the polynomial splits the tile into blocks the
             * scheduler cannot overlap and measured slower.  Callers asking
             * for the state history (h_all) take the exact per-step path
             * below instead. */
            float hst[G];
#pragma unroll
            for (int j = 0; j < G; ++j) hst[j] = h[j];
            float2 sq[G / 2];
#pragma unroll
            for (int jp = 0; jp < G / 2; ++jp) sq[jp] = kmb_f2s(0.f);
#pragma unroll
            for (int i0 = 0; i0 < TT; i0 += P) {
                float yq[P];
#pragma unroll
                for (int s = 0; s < P; ++s) {
                    const int i = i0 + s;
                    const float dv = ds[i * DT];
                    const float u = dv * xs[i * DT];
                    float bv[G], cv[G];
                    if (SHARED) {
                        ldsv<G>(bs + i * BW, bv);
                        ldsv<G>(cs + i * BW, cv);
                    } else {
                        ldgv<G, VEC>(bgl + (t0 + i) * hstride, gok && dok, N, dok ? n0 : N, bv);
                        ldgv<G, VEC>(cgl + (t0 + i) * hstride, gok && dok, N, dok ? n0 : N, cv);
                    }
                    /* state pairs on FFMA2 / FMUL2 (same per-element rounding) */
                    const float2 dv2 = kmb_f2s(dv), u2 = kmb_f2s(u);
                    float2 a[G / 2];
#pragma unroll
                    for (int jp = 0; jp < G / 2; ++jp)
                        a[jp] = kmb_exp2_decay2(kmb_mul2(dv2, kmb_f2(A2[2 * jp], A2[2 * jp + 1])));
                    float2 y2 = kmb_f2s(0.f);
#pragma unroll
                    for (int jp = 0; jp < G / 2; ++jp) {
                        const int j = 2 * jp;
                        const float2 hn = kmb_fma2(a[jp], kmb_f2(h[j], h[j + 1]),
                                                   kmb_mul2(kmb_f2(bv[j], bv[j + 1]), u2));
                        if (CLAMP) sq[jp] = kmb_fma2(hn, hn, sq[jp]);
                        h[j] = hn.x;
                        h[j + 1] = hn.y;
                        y2 = kmb_fma2(kmb_f2(cv[j], cv[j + 1]), hn, y2);
                    }
                    yq[s] = y2.x + y2.y;
                    if ((i + 1) % kChunk == 0 && ckpt && dok)
                        stgv<G, VEC>(ckpt + ((t0 + i) / kChunk) * hstride, gok, N, n0, h);
                }
                ys[(i0 + g) * DT] = rs_sum<P>(yq, lane);
            }
            if (CLAMP) {
                float ss = 0.f;
#pragma unroll
                for (int jp = 0; jp < G / 2; ++jp) ss += sq[jp].x + sq[jp].y;
                if (__any_sync(kFull, !(ss < 1e6f))) {
#pragma unroll
                    for (int j = 0; j < G; ++j) h[j] = hst[j];
                    slow_tile(TT);
                }
            }
        } else {
            slow_tile(rv);
        }
    }
    kmb_cp_async_wait<0>();
    __syncthreads();
    if (p.y) flush_y(ntiles - 1);
    if (p.h_last && dok) stgv<G, VEC>(p.h_last + (b * D + d) * N + n0, gok, N, n0, h);
}

/* ------------------------------------------------------------------ */
/* backward                                                            */
/* ------------------------------------------------------------------ */

/*
 * Reduce-scatter of 8 values across the lanes of a warp that share the
 * same lane-group index g (lanes differing in bits >= log2(P)).  After the
 * call lane holds `cnt` sums starting at index `base`; lanes with
 * (lane & dup) != 0 hold duplicates of another lane's sums.
 */
template <int P>
__device__ __forceinline__ void reduce_scatter8(float (&v)[8], int lane, int &base,
                                                int &cnt, int &dup) {
    cnt = 8;
    base = 0;
    dup = 0;
#pragma unroll
    for (int o = 16; o >= P; o >>= 1) {
        if (cnt > 1) {
            const int half = cnt >> 1;
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (k < half) {
                    const float send = up ? v[k] : v[k + half];
                    const float keep = up ? v[k + half] : v[k];
                    v[k] = keep + __shfl_xor_sync(kFull, send, o);
                }
            }
            if (up) base += half;
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(kFull, v[0], o);
            dup |= o;
        }
    }
}

template <int P, bool SHARED, bool VEC, bool HALL, bool CLAMP>
__global__ void __launch_bounds__(kNT, 3) k_scan1d_bwd(Scan1DDev p) {
    constexpr int DT = kNT / P;
    constexpr int T = kChunk;
    constexpr int NP = kG * P;
    /* steps per dx/ddt reduce-scatter group (2 values per step, one value
     * per lane of the channel; slots past 2*S are zero when P > 2*T) */
    constexpr int S = P >= 2 ? (P / 2 < T ? P / 2 : T) : 1;
    constexpr int NV = P >= 2 ? P : 2;      /* values per reduce-scatter */
    static_assert(T % S == 0, "chunk must hold whole groups");
    extern __shared__ __align__(16) float smem[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int g = tid % P;
    const int dl = tid / P;
    const int n0 = g * kG;
    const long b = blockIdx.y;
    const long D = p.D, L = p.L;
    const int N = (int)p.N;
    const long d0 = (long)blockIdx.x * DT;
    const long d = d0 + dl;
    const bool dok = d < D;
    const bool gok = n0 < N;
    const int dvalid = (int)min((long)DT, D - d0);

    /* shared-memory row of channel-shared B / C: bc_row_stride(true, NP, N),
     * which is NP for every N the launcher maps to this P */
    constexpr int BW = SHARED ? NP : 0;
    constexpr int xs_sz = T * DT;
    constexpr int bs_sz = T * BW;
    constexpr int ck_sz = HALL ? 0 : DT * NP; /* checkpointed chunk-start states [DT][NP] */
    constexpr int stage_sz = 3 * xs_sz + 2 * bs_sz + ck_sz;
    /* per-thread dB / dC contributions of the chunk, [T][DT][NP] each
     * (SHARED only): thread (dl, g) writes 16 bytes at 16 * tid, so the
     * 128-bit stores are conflict-free; folded once per chunk */
    float *partB = smem + 2 * stage_sz;
    float *partC = partB + T * DT * NP;

    /* per-state values live as pairs: the FFMA2 / FMUL2 operands */
    float2 A2p[2], Arp[2], gcp[2], dAp[2];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        const int j = n0 + 2 * jp;
        const float a0 = (dok && j < N) ? __ldg(p.A + d * N + j) : 0.f;
        const float a1 = (dok && j + 1 < N) ? __ldg(p.A + d * N + j + 1) : 0.f;
        Arp[jp] = kmb_f2(a0, a1);
        A2p[jp] = kmb_f2(a0 * KMB_LOG2E, a1 * KMB_LOG2E);
        gcp[jp] = kmb_f2s(0.f);
        dAp[jp] = kmb_f2s(0.f);
    }

    const long xoff = b * L * D + d0;
    const float *xg = p.x + xoff;
    const float *dg = p.dt + xoff;
    const float *yg = p.dy + xoff;
    const long bld = SHARED ? (long)N : D * N;
    const long boff = SHARED ? b * L * N : (b * L * D + d0) * N;
    const float *Bg = p.B + boff;
    const float *Cg = p.C + boff;
    const bool vxd = p.vec_xd, vbc = p.vec_bc;
    const long hstride = D * N;
    const float *hall = HALL ? p.h_all + (b * L * D + d) * N + n0 : nullptr;

    const int nch = (int)((L + T - 1) / T);
    auto load = [&](int c, int stage) {
        float *st = smem + stage * stage_sz;
        const long t0 = (long)c * T;
        const int rv = (int)min((long)T, L - t0);
        kmb_load_tile_c<kNT, T, DT>(st, DT, xg + t0 * D, D, rv, dvalid, vxd, tid);
        kmb_load_tile_c<kNT, T, DT>(st + xs_sz, DT, dg + t0 * D, D, rv, dvalid, vxd, tid);
        kmb_load_tile_c<kNT, T, DT>(st + 2 * xs_sz, DT, yg + t0 * D, D, rv, dvalid, vxd, tid);
        if constexpr (SHARED) {
            /* columns past N are zero-filled */
            kmb_load_tile_c<kNT, T, BW>(st + 3 * xs_sz, BW, Bg + t0 * bld, bld, rv, N, vbc, tid);
            kmb_load_tile_c<kNT, T, BW>(st + 3 * xs_sz + bs_sz, BW, Cg + t0 * bld, bld, rv, N,
                                        vbc, tid);
        }
        if (!HALL && c > 0) {
            /* the forward's checkpoint of the state before this chunk: the
             * CTA's DT channels x N states are contiguous */
            const float *src = p.ckpt_in + ((b * p.nslots + c - 1) * D + d0) * N;
            kmb_load_tile_c<kNT, DT, NP>(st + 3 * xs_sz + 2 * bs_sz, NP, src, N, dvalid, N, VEC,
                                         tid);
        }
    };

    load(nch - 1, 0);
    kmb_cp_async_commit();

    const int brow = n0;
    const float *bgl = SHARED ? nullptr : p.B + (b * L * D + d) * N + n0;
    const float *cgl = SHARED ? nullptr : p.C + (b * L * D + d) * N + n0;
    float *dxg = p.dx + b * L * D + d;
    float *dtg = p.ddt + b * L * D + d;

    /* 4 states of a B / C row as two pairs (shared tile or global row) */
    auto row_pairs = [&](const float *srow, const float *grow, long t, float2 (&v)[2]) {
        float4 t4;
        if (SHARED) {
            t4 = *reinterpret_cast<const float4 *>(srow);
        } else {
            float f[kG];
            ldg4<VEC>(grow + t * hstride, gok && dok, N, dok ? n0 : N, f);
            t4 = make_float4(f[0], f[1], f[2], f[3]);
        }
        v[0] = kmb_f2(t4.x, t4.y);
        v[1] = kmb_f2(t4.z, t4.w);
    };

    for (int c = nch - 1, it = 0; c >= 0; --c, ++it) {
        kmb_cp_async_wait<0>();
        __syncthreads();
        if (c > 0) load(c - 1, (it + 1) & 1);
        kmb_cp_async_commit();

        const float *st = smem + (it & 1) * stage_sz;
        const float *xs = st + dl;
        const float *ds = st + xs_sz + dl;
        const float *dys = st + 2 * xs_sz + dl;
        const float *bs = st + 3 * xs_sz + brow;
        const float *cs = bs + bs_sz;
        const long t0 = (long)c * T;
        const int len = (int)min((long)T, L - t0);

        /* state before the chunk's first step */
        float2 hsp[2];
        if (c > 0) {
            float hs[kG];
            if (HALL) {
                if (dok) ldg4<VEC>(hall + (t0 - 1) * hstride, gok, N, n0, hs);
                else hs[0] = hs[1] = hs[2] = hs[3] = 0.f;
            } else {
                /* 16-byte aligned row of the staged checkpoint, zero-filled
                 * past N and for channels past D */
                lds4u(st + 3 * xs_sz + 2 * bs_sz + dl * NP + n0, hs);
            }
            hsp[0] = kmb_f2(hs[0], hs[1]);
            hsp[1] = kmb_f2(hs[2], hs[3]);
        } else {
            float hs[kG];
#pragma unroll
            for (int j = 0; j < kG; ++j)
                hs[j] = (dok && n0 + j < N && p.h0) ? p.h0[(b * D + d) * N + n0 + j] : 0.f;
            hsp[0] = kmb_f2(hs[0], hs[1]);
            hsp[1] = kmb_f2(hs[2], hs[3]);
        }

        /* With channel-shared B/C and no h_all, steps past the end of the
         * sequence (only in the last chunk, which is processed first) are
         * exact identity steps: the staged x, dt, dy, B, C rows are
         * zero-filled there, so dt = 0 gives a decay of exactly 1, u = 0
         * leaves h unchanged and dy = C = 0 with a zero carry makes every
         * gradient term 0.  Those steps need no bounds; the other modes
         * read global memory per step and keep them. */
        constexpr bool FULL = SHARED && !HALL;
        {
            /* forward recompute of the chunk's states (registers).  Without
             * the clamp on the critical path: a detector sums h^2 over the
             * chunk (any |h| > 1000, or a NaN, pushes it to at least 1e6),
             * and a flagged chunk is recomputed with the exact clamp, so the
             * states match the forward's bit for bit either way.  Decays are
             * kmb_exp2_decay2 (MUFU ex2 and the weak-decay polynomial,
             * selected per element): a warp-uniform branch per step, as in
             * the forward, costs registers that the chunk's states need. */
            float2 hr[HALL ? 1 : T][2]; /* states h_t of the chunk */
            float2 ar[HALL ? 1 : T][2]; /* decays a_t, reused by the reverse sweep */
            if (!HALL) {
                auto recompute = [&](auto exact_tag) {
                    constexpr bool EXACT = decltype(exact_tag)::value;
                    float2 hh[2] = {hsp[0], hsp[1]};
                    float2 sq = kmb_f2s(0.f);
#pragma unroll
                    for (int i = 0; i < T; ++i) {
                        if (FULL || i < len) {
                            const float dv = ds[i * DT];
                            const float2 dv2 = kmb_f2s(dv), u2 = kmb_f2s(dv * xs[i * DT]);
                            float2 bp[2], a[2];
                            row_pairs(bs + i * BW, bgl, t0 + i, bp);
#pragma unroll
                            for (int jp = 0; jp < 2; ++jp) a[jp] = kmb_exp2_decay2(kmb_mul2(dv2, A2p[jp]));
#pragma unroll
                            for (int jp = 0; jp < 2; ++jp) {
                                float2 hn = kmb_fma2(a[jp], hh[jp], kmb_mul2(bp[jp], u2));
                                if (EXACT) {
                                    hn.x = clamp1000(hn.x);
                                    hn.y = clamp1000(hn.y);
                                } else if (CLAMP) {
                                    sq = kmb_fma2(hn, hn, sq);
                                }
                                hh[jp] = hn;
                                hr[i][jp] = hn;
                                ar[i][jp] = a[jp];
                            }
                        }
                    }
                    return CLAMP && !EXACT && !(sq.x + sq.y < 1e6f);
                };
                if (__any_sync(kFull, recompute(std::false_type{})))
                    recompute(std::true_type{});
            }

            /* reverse sweep, S steps per dx/ddt reduce-scatter group */
#pragma unroll
            for (int i0 = T - 1; i0 >= 0; i0 -= S) {
                float rv[NV];
#pragma unroll
                for (int k = 0; k < NV; ++k) rv[k] = 0.f;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int i = i0 - s;
                    if (FULL || i < len) {
                        const float xv = xs[i * DT];
                        const float dv = ds[i * DT];
                        const float dyv = dys[i * DT];
                        const float2 dv2 = kmb_f2s(dv), dyv2 = kmb_f2s(dyv);
                        const float2 u2 = kmb_f2s(dv * xv);
                        float2 bp[2], cp[2], hp[2], ht[2];
                        row_pairs(bs + i * BW, bgl, t0 + i, bp);
                        row_pairs(cs + i * BW, cgl, t0 + i, cp);
                        if (HALL) {
                            float f[kG], q[kG];
                            if (dok) {
                                ldg4<VEC>(hall + (t0 + i) * hstride, gok, N, n0, f);
                                if (i > 0) {
                                    ldg4<VEC>(hall + (t0 + i - 1) * hstride, gok, N, n0, q);
                                } else {
                                    q[0] = hsp[0].x; q[1] = hsp[0].y;
                                    q[2] = hsp[1].x; q[3] = hsp[1].y;
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < kG; ++j) f[j] = q[j] = 0.f;
                            }
                            ht[0] = kmb_f2(f[0], f[1]);
                            ht[1] = kmb_f2(f[2], f[3]);
                            hp[0] = kmb_f2(q[0], q[1]);
                            hp[1] = kmb_f2(q[2], q[3]);
                        } else {
#pragma unroll
                            for (int jp = 0; jp < 2; ++jp) {
                                ht[jp] = hr[HALL ? 0 : i][jp];
                                hp[jp] = i > 0 ? hr[HALL ? 0 : (i > 0 ? i - 1 : 0)][jp] : hsp[jp];
                            }
                        }
                        float2 dxs2 = kmb_f2s(0.f), dts2 = kmb_f2s(0.f), vb[2], vc[2];
#pragma unroll
                        for (int jp = 0; jp < 2; ++jp) {
                            const float2 a = HALL ? kmb_exp2_decay2(kmb_mul2(dv2, A2p[jp]))
                                                  : ar[HALL ? 0 : i][jp];
                            const float2 ah = kmb_fma2(dyv2, cp[jp], gcp[jp]);
                            const float2 q = kmb_mul2(ah, a);
                            const float2 qh = kmb_mul2(q, hp[jp]);
                            dAp[jp] = kmb_fma2(dv2, qh, dAp[jp]);
                            dts2 = kmb_fma2(Arp[jp], qh, dts2);
                            dxs2 = kmb_fma2(ah, bp[jp], dxs2);
                            vb[jp] = kmb_mul2(ah, u2);      /* dB contribution */
                            vc[jp] = kmb_mul2(dyv2, ht[jp]); /* dC contribution */
                            gcp[jp] = q;
                        }
                        const float dxs = dxs2.x + dxs2.y;
                        rv[2 * s] = dxs;
                        rv[2 * s + 1] = fmaf(xv, dxs, dts2.x + dts2.y);
                        if (SHARED) {
                            const int o = (i * DT + dl) * NP + n0;
                            *reinterpret_cast<float4 *>(partB + o) =
                                make_float4(vb[0].x, vb[0].y, vb[1].x, vb[1].y);
                            *reinterpret_cast<float4 *>(partC + o) =
                                make_float4(vc[0].x, vc[0].y, vc[1].x, vc[1].y);
                        } else if (dok) {
                            const float fb[kG] = {vb[0].x, vb[0].y, vb[1].x, vb[1].y};
                            const float fc[kG] = {vc[0].x, vc[0].y, vc[1].x, vc[1].y};
                            const long o = ((b * L + t0 + i) * D + d) * N + n0;
                            stg4<VEC>(p.dB + o, gok, N, n0, fb);
                            stg4<VEC>(p.dC + o, gok, N, n0, fc);
                        }
                    }
                }
                /* fold dx / ddt over the P lanes of the channel */
                if (P >= 2) {
                    const float r = rs_sum<NV>(rv, lane);
                    const int s = g >> 1;
                    const int i = i0 - s;
                    if (dok && g < 2 * S && i >= 0 && i < len) {
                        const long t = t0 + i;
                        if (g & 1) dtg[t * D] = r;
                        else dxg[t * D] = r * ds[i * DT];
                    }
                } else {
                    const int i = i0;
                    if (dok && i < len) {
                        const long t = t0 + i;
                        dxg[t * D] = rv[0] * ds[i * DT];
                        dtg[t * D] = rv[1];
                    }
                }
            }
        }

        if (SHARED) {
            __syncthreads();
            /* channel sums of the chunk's dB / dC: HR threads per 4-state
             * output, each summing every HR-th channel (interleaved so that
             * a quarter-warp reads adjacent rows), folded by shuffles; one
             * 128-bit atomic per output and CTA */
            constexpr int NQ = NP / 4;
            constexpr int HR = NP >= 32 ? 1 : 32 / NP;
            constexpr int OUTS = 2 * T * NQ;
            constexpr int ITER = (OUTS * HR + kNT - 1) / kNT;
#pragma unroll
            for (int r = 0; r < ITER; ++r) {
                const int e = r * kNT + tid;
                const int o = e / HR, hh = e % HR;
                const int arr = o / (T * NQ);
                const int i = (o % (T * NQ)) / NQ;
                const int q = o % NQ;
                const bool live = o < OUTS && i < len && q * 4 < N;
                float2 lo = kmb_f2s(0.f), hi = kmb_f2s(0.f);
                if (live) {
                    const float *src = (arr ? partC : partB) + i * DT * NP + q * 4;
#pragma unroll 8
                    for (int k = 0; k < DT / HR; ++k) {
                        const int dlx = k * HR + hh;
                        if (dlx < dvalid) {
                            const float4 t4 = *reinterpret_cast<const float4 *>(src + dlx * NP);
                            lo = kmb_add2(lo, kmb_f2(t4.x, t4.y));
                            hi = kmb_add2(hi, kmb_f2(t4.z, t4.w));
                        }
                    }
                }
#pragma unroll
                for (int m = HR / 2; m > 0; m >>= 1) {
                    lo.x += __shfl_xor_sync(kFull, lo.x, m);
                    lo.y += __shfl_xor_sync(kFull, lo.y, m);
                    hi.x += __shfl_xor_sync(kFull, hi.x, m);
                    hi.y += __shfl_xor_sync(kFull, hi.y, m);
                }
                if (live && hh == 0) {
                    const int n = q * 4;
                    float *dst = (arr ? p.dC : p.dB) + (b * L + t0 + i) * N + n;
                    if (VEC && vbc) {
                        atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(lo.x, lo.y, hi.x, hi.y));
                    } else {
                        const float sv[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            if (n + k < N) atomicAdd(dst + k, sv[k]);
                    }
                }
            }
        }
    }
    kmb_cp_async_wait<0>();

    {
        const float dAs[kG] = {dAp[0].x, dAp[0].y, dAp[1].x, dAp[1].y};
#pragma unroll
        for (int j = 0; j < kG; ++j)
            if (dok && n0 + j < N) atomicAdd(p.dA + d * N + n0 + j, dAs[j]);
    }
}

/*
 * Backward for channel-shared B/C with 16-byte aligned rows (x / dt / dy
 * rows of D floats, B / C rows of N floats, D and N multiples of 4): the
 * arithmetic of k_scan1d_bwd (checkpointed chunk recompute, reverse sweep
 * on state pairs) with the per-chunk bookkeeping reduced:
 *
 *  - staging: every 16-byte unit of a chunk's x, dt, dy, B, C rows and of
 *    its checkpoint row is a fixed copy job; a thread's jobs (source at
 *    chunk 0, destination in the stage, row, column bytes) are set up once,
 *    so a chunk costs each thread NJ cp.async plus an address update;
 *  - dx / ddt: each lane stores its partial (sum_n e B, sum_n A q h) to a
 *    shared [T][DT][P] tile; after the sweep the CTA folds the P partials
 *    of every (step, channel) and writes dx / ddt rows with coalesced
 *    stores (no shuffles, no per-lane scattered stores);
 *  - dB / dC: the shared-tile fold of k_scan1d_bwd, without per-channel
 *    bounds checks when the CTA's channel tile is full.
 */
template <int P, bool CLAMP>
__global__ void __launch_bounds__(kNT, 3) k_scan1d_bwd_sh(Scan1DDev p) {
    constexpr int DT = kNT / P;
    constexpr int T = kChunk;
    constexpr int NP = kG * P;
    constexpr int XS = T * DT;  /* x / dt / dy tile [T][DT] */
    constexpr int BS = T * NP;  /* B / C tile [T][NP] */
    constexpr int CK = DT * NP; /* checkpointed chunk-start states [DT][NP] */
    constexpr int STAGE = 3 * XS + 2 * BS + CK;
    constexpr int UX = XS / 4, UB = BS / 4, UC = CK / 4;
    constexpr int UTOT = 3 * UX + 2 * UB + UC;
    constexpr int NJ = (UTOT + kNT - 1) / kNT;
    static_assert(XS % 4 == 0 && DT % 4 == 0 && STAGE < 65536, "stage layout");
    static_assert((2 * STAGE + 2 * T * DT * NP) % 4 == 0, "partX alignment");
    extern __shared__ __align__(16) float smem[];
    float *partB = smem + 2 * STAGE;    /* [T][DT][NP] dB contributions */
    float *partC = partB + T * DT * NP; /* [T][DT][NP] dC contributions */
    float2 *partX = reinterpret_cast<float2 *>(partC + T * DT * NP); /* [T][DT][P] */

    const int tid = threadIdx.x;
    const int g = tid % P;
    const int dl = tid / P;
    const int n0 = g * kG;
    const long b = blockIdx.y;
    const long D = p.D, L = p.L;
    const int N = (int)p.N;
    const long d0 = (long)blockIdx.x * DT;
    const long d = d0 + dl;
    const bool dok = d < D;
    const int dvalid = (int)min((long)DT, D - d0);
    const int nch = (int)((L + T - 1) / T);

    /* Copy jobs.  Every 16-byte unit of a stage is one job; thread tid
     * runs jobs tid + k * kNT.  Per job: the source at the last chunk
     * (row jobs) or at the last checkpoint slot, moved back by a fixed
     * stride per chunk; the destination offset in the stage (bits 0-15),
     * the row within the chunk (16-23, 255 for checkpoint jobs) and the
     * bytes of the unit inside the tensor's columns (24-28).  Rows past
     * the sequence exist only in the first chunk processed (the last one),
     * so later chunks skip the row check. */
    const float *jsrc[NJ];
    int jstr[NJ];
    unsigned jinfo[NJ];
    const long clast = nch - 1;
#pragma unroll
    for (int k = 0; k < NJ; ++k) {
        const int e = tid + k * kNT;
        const float *src = p.x;
        unsigned info = 0;
        int stride = 0;
        auto cbytes = [](int left) { return left >= 4 ? 16 : (left > 0 ? 4 * left : 0); };
        if (e < 3 * UX) {
            const int arr = e / UX, u = e % UX;
            const int r = u / (DT / 4), col = (u % (DT / 4)) * 4;
            const float *base = arr == 0 ? p.x : (arr == 1 ? p.dt : p.dy);
            const int cb = cbytes(dvalid - col);
            src = base + (b * L + clast * T + r) * D + d0 + col;
            stride = T * (int)D;
            info = (unsigned)(arr * XS + r * DT + col) | ((unsigned)r << 16) | ((unsigned)cb << 24);
        } else if (e < 3 * UX + 2 * UB) {
            const int u0 = e - 3 * UX;
            const int arr = u0 / UB, u = u0 % UB;
            const int r = u / (NP / 4), col = (u % (NP / 4)) * 4;
            const int cb = cbytes(N - col);
            src = (arr ? p.C : p.B) + (b * L + clast * T + r) * N + col;
            stride = T * N;
            info = (unsigned)(3 * XS + arr * BS + r * NP + col) | ((unsigned)r << 16) |
                   ((unsigned)cb << 24);
        } else if (e < UTOT) {
            const int u = e - 3 * UX - 2 * UB;
            const int r = u / (NP / 4), col = (u % (NP / 4)) * 4;
            const int cb = r < dvalid ? cbytes(N - col) : 0;
            /* chunk c reads slot c - 1; the first chunk with a checkpoint
             * is nch - 1 */
            src = p.ckpt_in + ((b * p.nslots + (clast > 0 ? clast - 1 : 0)) * D + d0 + r) * N + col;
            stride = (int)(D * N);
            info = (unsigned)(3 * XS + 2 * BS + r * NP + col) | (255u << 16) | ((unsigned)cb << 24);
        }
        jsrc[k] = src;
        jstr[k] = stride;
        jinfo[k] = info;
    }
    /* issue the copies of chunk c (chunks are loaded from the last one
     * down, once each) and move every job one chunk back */
    auto load = [&](int c, int stage, bool first) {
        float *st = smem + stage * STAGE;
#pragma unroll
        for (int k = 0; k < NJ; ++k) {
            if (tid + k * kNT < UTOT) {
                const unsigned info = jinfo[k];
                const unsigned row = (info >> 16) & 0xffu;
                int bytes = (int)(info >> 24);
                if (row == 255u) {
                    if (c == 0) continue; /* no checkpoint before chunk 0 */
                } else if (first && (long)c * T + row >= L) {
                    bytes = 0;
                }
                kmb_cp_async16(st + (info & 0xffffu), bytes ? jsrc[k] : p.x, bytes);
                if (row != 255u || c > 1) jsrc[k] -= jstr[k];
            }
        }
    };

    /* per-state values live as pairs: the FFMA2 / FMUL2 operands */
    float2 A2p[2], Arp[2], gcp[2], dAp[2];
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
        const int j = n0 + 2 * jp;
        const float a0 = (dok && j < N) ? __ldg(p.A + d * N + j) : 0.f;
        const float a1 = (dok && j + 1 < N) ? __ldg(p.A + d * N + j + 1) : 0.f;
        Arp[jp] = kmb_f2(a0, a1);
        A2p[jp] = kmb_f2(a0 * KMB_LOG2E, a1 * KMB_LOG2E);
        gcp[jp] = kmb_f2s(0.f);
        dAp[jp] = kmb_f2s(0.f);
    }

    load(nch - 1, 0, true);
    kmb_cp_async_commit();

    /* dx / ddt rows this thread writes (see the fold below): outputs
     * o = tid + r kNT of a chunk are (step o / DT, channel o % DT) */
    constexpr int NXO = (T * DT + kNT - 1) / kNT;
    const int xdd = tid % DT;
    const bool xok = xdd < dvalid;
    long xoff = (b * L + clast * T + tid / DT) * D + d0 + xdd;

    for (int c = nch - 1, it = 0; c >= 0; --c, ++it) {
        kmb_cp_async_wait<0>();
        __syncthreads();
        if (c > 0) load(c - 1, (it + 1) & 1, false);
        kmb_cp_async_commit();

        const float *st = smem + (it & 1) * STAGE;
        const float *xs = st + dl;
        const float *ds = st + XS + dl;
        const float *dys = st + 2 * XS + dl;
        const float *bs = st + 3 * XS + n0;
        const float *cs = bs + BS;
        const long t0 = (long)c * T;
        const int len = (int)min((long)T, L - t0);

        /* state before the chunk's first step */
        float2 hsp[2];
        if (c > 0) {
            float hs[kG];
            lds4u(st + 3 * XS + 2 * BS + dl * NP + n0, hs);
            hsp[0] = kmb_f2(hs[0], hs[1]);
            hsp[1] = kmb_f2(hs[2], hs[3]);
        } else {
            float hs[kG];
#pragma unroll
            for (int j = 0; j < kG; ++j)
                hs[j] = (dok && n0 + j < N && p.h0) ? p.h0[(b * D + d) * N + n0 + j] : 0.f;
            hsp[0] = kmb_f2(hs[0], hs[1]);
            hsp[1] = kmb_f2(hs[2], hs[3]);
        }

        /* forward recompute of the chunk's states, as in k_scan1d_bwd.
         * Steps past the end of the sequence (last chunk only) have
         * zero-filled rows: dt = 0 gives a decay of exactly 1 and u = 0,
         * so they are identity steps with zero gradient terms. */
        float2 hr[T][2], ar[T][2];
        auto recompute = [&](auto exact_tag) {
            constexpr bool EXACT = decltype(exact_tag)::value;
            float2 hh[2] = {hsp[0], hsp[1]};
            float2 sq = kmb_f2s(0.f);
#pragma unroll
            for (int i = 0; i < T; ++i) {
                const float dv = ds[i * DT];
                const float2 dv2 = kmb_f2s(dv), u2 = kmb_f2s(dv * xs[i * DT]);
                const float4 b4 = *reinterpret_cast<const float4 *>(bs + i * NP);
                const float2 bp[2] = {kmb_f2(b4.x, b4.y), kmb_f2(b4.z, b4.w)};
#pragma unroll
                for (int jp = 0; jp < 2; ++jp) {
                    const float2 a = kmb_exp2_decay2(kmb_mul2(dv2, A2p[jp]));
                    float2 hn = kmb_fma2(a, hh[jp], kmb_mul2(bp[jp], u2));
                    if (EXACT) {
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
            return CLAMP && !EXACT && !(sq.x + sq.y < 1e6f);
        };
        if (__any_sync(kFull, recompute(std::false_type{}))) recompute(std::true_type{});

        /* reverse sweep */
#pragma unroll
        for (int i = T - 1; i >= 0; --i) {
            const float xv = xs[i * DT];
            const float dv = ds[i * DT];
            const float dyv = dys[i * DT];
            const float2 dv2 = kmb_f2s(dv), dyv2 = kmb_f2s(dyv);
            const float2 u2 = kmb_f2s(dv * xv);
            const float4 b4 = *reinterpret_cast<const float4 *>(bs + i * NP);
            const float4 c4 = *reinterpret_cast<const float4 *>(cs + i * NP);
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
                vb[jp] = kmb_mul2(ah, u2);        /* dB contribution */
                vc[jp] = kmb_mul2(dyv2, hr[i][jp]); /* dC contribution */
                gcp[jp] = q;
            }
            partX[(i * DT + dl) * P + g] = kmb_f2(dxs2.x + dxs2.y, dts2.x + dts2.y);
            const int o = (i * DT + dl) * NP + n0;
            *reinterpret_cast<float4 *>(partB + o) = make_float4(vb[0].x, vb[0].y, vb[1].x, vb[1].y);
            *reinterpret_cast<float4 *>(partC + o) = make_float4(vc[0].x, vc[0].y, vc[1].x, vc[1].y);
        }
        __syncthreads();

        /* dx / ddt of the chunk: fold the P lane partials of each (step,
         * channel); a warp writes consecutive channels of one step */
#pragma unroll
        for (int r = 0; r < NXO; ++r) {
            const int o = tid + r * kNT;
            if ((T * DT) % kNT == 0 || o < T * DT) {
                const int i = o / DT;
                const float2 *src = partX + o * P;
                float2 sum = src[0];
#pragma unroll
                for (int q = 1; q < P; ++q) sum = kmb_add2(sum, src[q]);
                if (xok && i < len) {
                    const long t = xoff + (long)(r * (kNT / DT)) * D;
                    p.dx[t] = sum.x * st[XS + o];
                    p.ddt[t] = fmaf(st[o], sum.x, sum.y);
                }
            }
        }
        xoff -= (long)T * D;

        /* channel sums of the chunk's dB / dC: HR threads per 4-state
         * output, each summing every HR-th channel, folded by shuffles; one
         * 128-bit atomic per output and CTA */
        {
            constexpr int NQ = NP / 4;
            constexpr int HR = NP >= 32 ? 1 : 32 / NP;
            constexpr int OUTS = 2 * T * NQ;
            constexpr int ITER = (OUTS * HR + kNT - 1) / kNT;
            const bool full = dvalid == DT;
#pragma unroll
            for (int r = 0; r < ITER; ++r) {
                const int e = r * kNT + tid;
                const int o = e / HR, hh = e % HR;
                const int arr = o / (T * NQ);
                const int i = (o % (T * NQ)) / NQ;
                const int q = o % NQ;
                const bool live = o < OUTS && i < len && q * 4 < N;
                float2 lo = kmb_f2s(0.f), hi = kmb_f2s(0.f);
                if (live) {
                    const float *src = (arr ? partC : partB) + i * DT * NP + q * 4;
                    if (full) {
#pragma unroll
                        for (int k = 0; k < DT / HR; ++k) {
                            const float4 t4 =
                                *reinterpret_cast<const float4 *>(src + (k * HR + hh) * NP);
                            lo = kmb_add2(lo, kmb_f2(t4.x, t4.y));
                            hi = kmb_add2(hi, kmb_f2(t4.z, t4.w));
                        }
                    } else {
                        for (int k = 0; k < DT / HR; ++k) {
                            const int dlx = k * HR + hh;
                            if (dlx < dvalid) {
                                const float4 t4 = *reinterpret_cast<const float4 *>(src + dlx * NP);
                                lo = kmb_add2(lo, kmb_f2(t4.x, t4.y));
                                hi = kmb_add2(hi, kmb_f2(t4.z, t4.w));
                            }
                        }
                    }
                }
#pragma unroll
                for (int m = HR / 2; m > 0; m >>= 1) {
                    lo.x += __shfl_xor_sync(kFull, lo.x, m);
                    lo.y += __shfl_xor_sync(kFull, lo.y, m);
                    hi.x += __shfl_xor_sync(kFull, hi.x, m);
                    hi.y += __shfl_xor_sync(kFull, hi.y, m);
                }
                if (live && hh == 0) {
                    float *dst = (arr ? p.dC : p.dB) + (b * L + t0 + i) * N + q * 4;
                    atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(lo.x, lo.y, hi.x, hi.y));
                }
            }
        }
    }
    kmb_cp_async_wait<0>();

    {
        const float dAs[kG] = {dAp[0].x, dAp[0].y, dAp[1].x, dAp[1].y};
#pragma unroll
        for (int j = 0; j < kG; ++j)
            if (dok && n0 + j < N) atomicAdd(p.dA + d * N + n0 + j, dAs[j]);
    }
}

/* M = 1 backward with per-channel A/B/C and a per-step delta shared by all
 * channels (reference cpu/scan1d_backward.c:23-191).  One thread per
 * channel walks t downwards; ddelta[t] is a sum over channels. */
__global__ void __launch_bounds__(128)
k_scan1d_bwd_m1_shared(const float *x, const float *A, const float *A_diag,
                       const float *B, const float *C, const float *delta,
                       const float *h0, const float *h, const float *dy,
                       float *dx, float *dA, float *dB, float *dC,
                       float *ddelta, long L, long D) {
    const long d = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool ok = d < D;
    const float a = ok ? A[d] : 0.f, bb = ok ? B[d] : 0.f, cc = ok ? C[d] : 0.f;
    float adj = 0.f, sA = 0.f, sB = 0.f, sC = 0.f;
    for (long t = L - 1; t >= 0; --t) {
        float ddt = 0.f;
        if (ok) {
            const long td = t * D + d;
            const float dt = delta[t];
            const float xt = x[td];
            const float gy = dy[td];
            const float da = A_diag ? A_diag[td] : kmb_exp2_decay(dt * a * KMB_LOG2E);
            const float hprev = t > 0 ? h[(t - 1) * D + d] : (h0 ? h0[d] : 0.f);
            const float ah = fmaf(gy, cc, adj);
            sC = fmaf(gy, h[td], sC);
            sB = fmaf(ah * dt, xt, sB);
            sA = fmaf(ah * dt * da, hprev, sA);
            dx[td] = ah * dt * bb;
            ddt = ah * fmaf(a * da, hprev, bb * xt);
            adj = ah * da;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ddt += __shfl_xor_sync(kFull, ddt, o);
        if ((threadIdx.x & 31) == 0) atomicAdd(ddelta + t, ddt);
    }
    if (ok) {
        dA[d] = sA;
        dB[d] = sB;
        dC[d] = sC;
    }
}

int pick_p(long N) {
    long q = (N + kG - 1) / kG;
    int p = 1;
    while (p < q) p <<= 1;
    return p;
}

Scan1DDev make_dev(const KmbScan1D *a) {
    Scan1DDev p;
    p.x = a->x; p.dt = a->dt; p.A = a->A; p.B = a->B; p.C = a->C; p.h0 = a->h0;
    p.y = a->y; p.h_last = a->h_last; p.h_all = a->h_all; p.ckpt = a->ckpt;
    p.dy = a->dy; p.dx = a->dx; p.ddt = a->ddt; p.dA = a->dA; p.dB = a->dB; p.dC = a->dC;
    p.ckpt_in = nullptr;
    p.L = a->L; p.D = a->D; p.N = a->N;
    p.nslots = (a->L + kChunk - 1) / kChunk;
    auto al = [](const void *q) { return ((uintptr_t)q & 15u) == 0; };
    p.vec_xd = (a->D % 4 == 0) && al(a->x) && al(a->dt) && (!a->dy || al(a->dy)) &&
               (!a->y || al(a->y));
    p.vec_bc = (a->N % 4 == 0) && al(a->B) && al(a->C) && (!a->dB || al(a->dB)) &&
               (!a->dC || al(a->dC));
    return p;
}

template <int P, int G, bool SHARED, bool VEC, bool CLAMP>
cudaError_t launch_fwd_t(const Scan1DDev &p, long batch, cudaStream_t s) {
    using Cfg = FwdCfg<P, SHARED>;
    const int BWr = bc_row_stride(SHARED, G * P, (int)p.N);
    if (SHARED && BWr != (G * P >= 4 ? G * P : 4)) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * Cfg::ST * (3 * Cfg::TT * Cfg::DT + 2 * Cfg::TT * BWr);
    auto kern = k_scan1d_fwd<P, G, SHARED, VEC, CLAMP>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((unsigned)((p.D + Cfg::DT - 1) / Cfg::DT), (unsigned)batch);
    kern<<<grid, kNT, smem, s>>>(p);
    return cudaGetLastError();
}

template <int P, bool SHARED, bool VEC, bool HALL, bool CLAMP>
cudaError_t launch_bwd_t(const Scan1DDev &p, long batch, cudaStream_t s) {
    constexpr int DT = kNT / P;
    const int BWr = bc_row_stride(SHARED, kG * P, (int)p.N);
    if (SHARED && BWr != kG * P) return cudaErrorInvalidValue;
    const int ck = HALL ? 0 : DT * kG * P;
    size_t smem = sizeof(float) * 2 * (3 * kChunk * DT + 2 * kChunk * BWr + ck);
    if (SHARED) smem += sizeof(float) * 2 * kChunk * DT * (kG * P);
    auto kern = k_scan1d_bwd<P, SHARED, VEC, HALL, CLAMP>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((unsigned)((p.D + DT - 1) / DT), (unsigned)batch);
    kern<<<grid, kNT, smem, s>>>(p);
    return cudaGetLastError();
}

template <int P, bool CLAMP>
cudaError_t launch_bwd_sh_t(const Scan1DDev &p, long batch, cudaStream_t s) {
    constexpr int DT = kNT / P;
    constexpr int NP = kG * P;
    constexpr int STAGE = 3 * kChunk * DT + 2 * kChunk * NP + DT * NP;
    const size_t smem = sizeof(float) * (2 * STAGE + 2 * kChunk * DT * NP) +
                        sizeof(float2) * kChunk * DT * P;
    auto kern = k_scan1d_bwd_sh<P, CLAMP>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((unsigned)((p.D + DT - 1) / DT), (unsigned)batch);
    kern<<<grid, kNT, smem, s>>>(p);
    return cudaGetLastError();
}

template <int P>
cudaError_t bwd_sh(const Scan1DDev &p, long batch, bool clamp, cudaStream_t s) {
    return clamp ? launch_bwd_sh_t<P, true>(p, batch, s) : launch_bwd_sh_t<P, false>(p, batch, s);
}

template <int P, bool SHARED>
cudaError_t fwd_ps(const Scan1DDev &p, long batch, bool vec, bool clamp, cudaStream_t s) {
    if (vec) return clamp ? launch_fwd_t<P, 4, SHARED, true, true>(p, batch, s)
                          : launch_fwd_t<P, 4, SHARED, true, false>(p, batch, s);
    return clamp ? launch_fwd_t<P, 4, SHARED, false, true>(p, batch, s)
                 : launch_fwd_t<P, 4, SHARED, false, false>(p, batch, s);
}

/* 2 states per lane: twice the lanes (and warps) per channel, for
 * channel-shared B/C with 16-byte aligned rows. */
template <int P>
cudaError_t fwd_g2(const Scan1DDev &p, long batch, bool clamp, cudaStream_t s) {
    return clamp ? launch_fwd_t<P, 2, true, true, true>(p, batch, s)
                 : launch_fwd_t<P, 2, true, true, false>(p, batch, s);
}

template <int P>
cudaError_t fwd_p(const Scan1DDev &p, long batch, bool shared, bool vec, bool clamp,
                  cudaStream_t s) {
    return shared ? fwd_ps<P, true>(p, batch, vec, clamp, s)
                  : fwd_ps<P, false>(p, batch, vec, clamp, s);
}

template <int P, bool SHARED, bool VEC>
cudaError_t bwd_psv(const Scan1DDev &p, long batch, bool hall, bool clamp, cudaStream_t s) {
    if (hall) return launch_bwd_t<P, SHARED, VEC, true, false>(p, batch, s);
    return clamp ? launch_bwd_t<P, SHARED, VEC, false, true>(p, batch, s)
                 : launch_bwd_t<P, SHARED, VEC, false, false>(p, batch, s);
}

template <int P>
cudaError_t bwd_p(const Scan1DDev &p, long batch, bool shared, bool vec, bool hall,
                  bool clamp, cudaStream_t s) {
    if (shared) return vec ? bwd_psv<P, true, true>(p, batch, hall, clamp, s)
                           : bwd_psv<P, true, false>(p, batch, hall, clamp, s);
    return vec ? bwd_psv<P, false, true>(p, batch, hall, clamp, s)
               : bwd_psv<P, false, false>(p, batch, hall, clamp, s);
}

} // namespace

/* States per lane of the forward on channel-shared B/C: 4 (default) or 2
 * (twice the warps, more cross-lane folding).  KMB_SCAN1D_LANE_STATES=2
 * selects the latter; any other value keeps 4. */
static int lane_states() {
    static int g = 0;
    if (!g) {
        const char *e = getenv("KMB_SCAN1D_LANE_STATES");
        g = (e && e[0] == '2' && e[1] == 0) ? 2 : 4;
    }
    return g;
}

extern "C" int kmb_launch_scan1d_fwd(const KmbScan1D *a, cudaStream_t s) {
    Scan1DDev p = make_dev(a);
    const bool vec = (a->N % 4) == 0;
    const bool shared = a->bc_shared != 0;
    const bool clamp = a->clamp != 0;
    const int P = pick_p(a->N);
    cudaError_t e;
    if (!shared && P > 16)
        return kmb_fail(KMB_EUNSUPPORTED, "scan1d: per-channel B/C support N <= 64 (N=%ld)", a->N);
    if (shared && vec && p.vec_bc && a->N <= 64 && lane_states() == 2) {
        int p2 = 1;
        while (p2 < (a->N + 1) / 2) p2 <<= 1;
        switch (p2) {
        case 2: e = fwd_g2<2>(p, a->batch, clamp, s); break;
        case 4: e = fwd_g2<4>(p, a->batch, clamp, s); break;
        case 8: e = fwd_g2<8>(p, a->batch, clamp, s); break;
        case 16: e = fwd_g2<16>(p, a->batch, clamp, s); break;
        default: e = fwd_g2<32>(p, a->batch, clamp, s); break;
        }
        if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d forward launch");
        return KMB_OK;
    }
    switch (P) {
    case 1: e = fwd_p<1>(p, a->batch, shared, vec, clamp, s); break;
    case 2: e = fwd_p<2>(p, a->batch, shared, vec, clamp, s); break;
    case 4: e = fwd_p<4>(p, a->batch, shared, vec, clamp, s); break;
    case 8: e = fwd_p<8>(p, a->batch, shared, vec, clamp, s); break;
    case 16: e = fwd_p<16>(p, a->batch, shared, vec, clamp, s); break;
    case 32: e = fwd_ps<32, true>(p, a->batch, vec, clamp, s); break;
    default: return kmb_fail(KMB_EUNSUPPORTED, "scan1d: N=%ld exceeds 128 states", a->N);
    }
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d forward launch");
    return KMB_OK;
}

extern "C" int kmb_launch_scan1d_bwd(const KmbScan1D *a, const float *ckpt_in,
                                     cudaStream_t s) {
    Scan1DDev p = make_dev(a);
    p.ckpt_in = ckpt_in;
    const bool vec = (a->N % 4) == 0;
    const bool shared = a->bc_shared != 0;
    const bool hall = a->h_all != nullptr;
    const bool clamp = a->clamp != 0;
    const int P = pick_p(a->N);
    if (!shared && P > 16)
        return kmb_fail(KMB_EUNSUPPORTED, "scan1d: per-channel B/C support N <= 64 (N=%ld)", a->N);
    /* KMB_SCAN1D_DA_ACCUM (host layer only): add to dA instead of
     * overwriting it, for batch slices of one call */
    cudaError_t e = (a->flags & KMB_SCAN1D_DA_ACCUM)
                        ? cudaSuccess
                        : cudaMemsetAsync(a->dA, 0, sizeof(float) * a->D * a->N, s);
    if (e == cudaSuccess && shared) {
        const size_t nb = sizeof(float) * a->batch * a->L * a->N;
        e = cudaMemsetAsync(a->dB, 0, nb, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(a->dC, 0, nb, s);
    }
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d backward memset");
    /* channel-shared B/C, 16-byte rows and checkpoints: the lean kernel */
    if (shared && !hall && p.vec_xd && p.vec_bc && ckpt_in && ((uintptr_t)ckpt_in & 15u) == 0 &&
        P <= 32 && a->D * a->N < (1L << 31) && kChunk * a->D < (1L << 31)) {
        switch (P) {
        case 1: e = bwd_sh<1>(p, a->batch, clamp, s); break;
        case 2: e = bwd_sh<2>(p, a->batch, clamp, s); break;
        case 4: e = bwd_sh<4>(p, a->batch, clamp, s); break;
        case 8: e = bwd_sh<8>(p, a->batch, clamp, s); break;
        case 16: e = bwd_sh<16>(p, a->batch, clamp, s); break;
        default: e = bwd_sh<32>(p, a->batch, clamp, s); break;
        }
        if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d backward launch");
        return KMB_OK;
    }
    switch (P) {
    case 1: e = bwd_p<1>(p, a->batch, shared, vec, hall, clamp, s); break;
    case 2: e = bwd_p<2>(p, a->batch, shared, vec, hall, clamp, s); break;
    case 4: e = bwd_p<4>(p, a->batch, shared, vec, hall, clamp, s); break;
    case 8: e = bwd_p<8>(p, a->batch, shared, vec, hall, clamp, s); break;
    case 16: e = bwd_p<16>(p, a->batch, shared, vec, hall, clamp, s); break;
    case 32:
        e = vec ? bwd_psv<32, true, true>(p, a->batch, hall, clamp, s)
                : bwd_psv<32, true, false>(p, a->batch, hall, clamp, s);
        break;
    default: return kmb_fail(KMB_EUNSUPPORTED, "scan1d: N=%ld exceeds 128 states", a->N);
    }
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d backward launch");
    return KMB_OK;
}

extern "C" int kmb_launch_scan1d_bwd_m1_shared(const float *x, const float *A,
                                               const float *A_diag, const float *B,
                                               const float *C, const float *delta,
                                               const float *h0, const float *h,
                                               const float *dy, float *dx, float *dA,
                                               float *dB, float *dC, float *ddelta,
                                               long L, long D, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(ddelta, 0, sizeof(float) * L, s);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d m1 backward memset");
    const unsigned blocks = (unsigned)((D + 127) / 128);
    k_scan1d_bwd_m1_shared<<<blocks, 128, 0, s>>>(x, A, A_diag, B, C, delta, h0, h, dy, dx,
                                                  dA, dB, dC, ddelta, L, D);
    e = cudaGetLastError();
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d m1 backward launch");
    return KMB_OK;
}
