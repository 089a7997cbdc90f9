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
    p->P = a->P; p->D = a->D; p->M = a->M; p->nd = a->nd; p->nlevels = a->nlevels;
    p->x_bs = a->P * a->D;
    p->dl_bs = a->delta_bstride;
    p->bc_ds = a->bc_shared ? 0 : a->M;
    p->bc_ps = a->bc_shared ? a->M : a->D * a->M;
    p->bc_bs = a->P * p->bc_ps;
    p->h_bs = a->P * a->D * a->M;
}

} // namespace

extern "C" int kmb_launch_scannd_fwd(const KmbNDLaunch *a, cudaStream_t s) {
    NDDev p;
    fill_dev(a, &p);
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
