/*
 * Mamba-3 block and LM-model kernels (sm_100a), fp32.
 *
 * Semantics of the reference CPU block (src/mamba_block.c:89-120 for the
 * controller projections, :413-465 for the scan, :471-502 for the block)
 * and model step (src/kmamba.c:344-466):
 *
 *   u_t = silu(W_in x_t)                        [R]
 *   dt_t = clamp(softplus(delta_proj . x_t), dt_min, dt_max)
 *   lam_t = sigmoid(lambda_proj . x_t)
 *   B_t = W_B x_t + b_B,  C_t = W_C x_t + b_C   [R*N], index r*N + n
 *   Bu_t[n] = sum_r B_t[r*N+n] u_t[r]
 *   h_t = exp(dt_t A) * R(theta) h_{t-1} + (1-lam_t) dt_t exp(dt_t A) Bu_{t-1}
 *         + lam_t dt_t Bu_t                     (R rotates state pairs)
 *   y_t[r] = sum_n C_t[r*N+n] h_t[n],   out_t = x_t + W_out y_t
 *
 * The projections of all tokens are one GEMM against the concatenated
 * weight [W_in; delta_proj; lambda_proj; W_B; W_C] (fp32 SIMT GEMM: fp32
 * parity with the reference excludes tf32/bf16 tensor-core GEMMs here),
 * followed by one elementwise activation pass.  The scan runs one CTA per
 * sequence with one thread per state pair, sequential in t; y is folded
 * across the CTA each step.  The backward is the adjoint of the scan (the
 * reference's CPU backward is an empty stub), walked in reverse with the
 * adjoint carried through the transposed rotation.
 */
#include "kmb_common.cuh"
#include "../kmb_internal.h"

namespace {

/* ------------------------------------------------------------------ */
/* strided fp32 GEMM                                                    */
/* ------------------------------------------------------------------ */

constexpr int kTM = 64, kTN = 64, kTK = 16;

/* C[m*ldc + n] (+)= sum_k A[m*am + k*ak] * B[k*bk + n*bn].  With ws set,
 * CTA z of blockIdx.z sums k in [z*kchunk, (z+1)*kchunk) and writes its
 * partial tile to ws[z][M][N] instead (split-K; k_gemm_reduce adds the
 * partials in z order, so the result does not depend on scheduling). */
__global__ void __launch_bounds__(256)
k_gemm(int M, int N, int K, const float *A, long am, long ak, const float *B, long bk,
       long bn, float *C, long ldc, int accumulate, float *ws, int kchunk) {
    __shared__ float As[kTK][kTM + 4];
    __shared__ float Bs[kTK][kTN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    const bool a_kfast = ak == 1, b_nfast = bn == 1;
    const int kbeg = ws ? (int)blockIdx.z * kchunk : 0;
    const int kend = ws ? min(K, kbeg + kchunk) : K;
    for (int k0 = kbeg; k0 < kend; k0 += kTK) {
        for (int e = threadIdx.x; e < kTM * kTK; e += 256) {
            int mm, kk;
            if (a_kfast) { mm = e / kTK; kk = e % kTK; } else { kk = e / kTM; mm = e % kTM; }
            const int gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < M && gk < kend) ? A[gm * am + gk * ak] : 0.f;
        }
        for (int e = threadIdx.x; e < kTK * kTN; e += 256) {
            int nn, kk;
            if (b_nfast) { kk = e / kTN; nn = e % kTN; } else { nn = e / kTK; kk = e % kTK; }
            const int gn = n0 + nn, gk = k0 + kk;
            Bs[kk][nn] = (gn < N && gk < kend) ? B[gk * bk + gn * bn] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kTK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            if (ws) {
                ws[((long)blockIdx.z * M + gm) * N + gn] = acc[i][j];
            } else {
                float *c = C + (long)gm * ldc + gn;
                *c = accumulate ? *c + acc[i][j] : acc[i][j];
            }
        }
    }
}

__global__ void k_gemm_reduce(const float *ws, int S, int M, int N, float *C, long ldc,
                              int accumulate) {
    const long tot = (long)M * N;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < tot;
         e += (long)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int z = 0; z < S; ++z) s += ws[z * tot + e];
        float *c = C + (e / N) * ldc + e % N;
        *c = accumulate ? *c + s : s;
    }
}

/* N = 1: C[m*ldc] (+)= sum_k A[m*am + k*ak] B[k*bk]; one warp per m */
__global__ void k_gemv_n1(int M, int K, const float *A, long am, long ak, const float *B,
                          long bk, float *C, long ldc, int accumulate) {
    const int lane = threadIdx.x & 31;
    const long m = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (m >= M) return;
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s = fmaf(A[m * am + k * ak], B[k * bk], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) C[m * ldc] = accumulate ? C[m * ldc] + s : s;
}

/* M = 1: C[n] (+)= sum_k A[k*ak] B[k*bk + n*bn]; a CTA of 32 n x 8 k
 * slices, the slices folded through shared memory in order */
__global__ void __launch_bounds__(256) k_gemv_m1(int N, int K, const float *A, long ak,
                                                 const float *B, long bk, long bn, float *C,
                                                 int accumulate) {
    __shared__ float red[8][33];
    const int nn = threadIdx.x & 31, ks = threadIdx.x >> 5;
    const long n = (long)blockIdx.x * 32 + nn;
    float s = 0.f;
    if (n < N)
        for (int k = ks; k < K; k += 8) s = fmaf(A[k * ak], B[k * bk + n * bn], s);
    red[ks][nn] = s;
    __syncthreads();
    if (ks == 0 && n < N) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t += red[i][nn];
        C[n] = accumulate ? C[n] + t : t;
    }
}

/* ------------------------------------------------------------------ */
/* projection activations                                               */
/* ------------------------------------------------------------------ */

struct ActArgs {
    const float *zraw;   /* [rows, W] GEMM output */
    float *zact;         /* [rows, W] activated */
    const float *bB, *bC;
    long rows;
    int W, R, NR;
    float dt_min, dt_max;
    int has_dp, has_lp;  /* 0: dt = dt_scale, lambda = 0.5 (no projection) */
    float dt_scale;
};

__global__ void k_block_act(ActArgs a) {
    const long total = a.rows * a.W;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long)gridDim.x * blockDim.x) {
        const int c = (int)(e % a.W);
        const float z = a.zraw[e];
        float v;
        if (c < a.R) {
            v = z / (1.0f + expf(-z));                 /* silu */
        } else if (c == a.R) {
            if (a.has_dp) {
                v = logf(1.0f + expf(z));              /* softplus, then clamp */
                if (v < a.dt_min) v = a.dt_min;
                if (v > a.dt_max) v = a.dt_max;
            } else {
                v = a.dt_scale;
            }
        } else if (c == a.R + 1) {
            v = a.has_lp ? 1.0f / (1.0f + expf(-z)) : 0.5f; /* sigmoid */
        } else if (c < a.R + 2 + a.NR) {
            v = z + a.bB[c - a.R - 2];
        } else {
            v = z + a.bC[c - a.R - 2 - a.NR];
        }
        a.zact[e] = v;
    }
}

/* dZ (in place) from the gradients of the activated values */
__global__ void k_block_act_bwd(ActArgs a, float *dz) {
    const long total = a.rows * a.W;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long)gridDim.x * blockDim.x) {
        const int c = (int)(e % a.W);
        if (c > a.R + 1) continue; /* B / C columns: identity (+bias) */
        const float z = a.zraw[e];
        const float g = dz[e];
        float d;
        if (c < a.R) {
            const float s = 1.0f / (1.0f + expf(-z));
            d = g * s * (1.0f + z * (1.0f - s));
        } else if (c == a.R) {
            const float sp = logf(1.0f + expf(z));
            d = (a.has_dp && sp > a.dt_min && sp < a.dt_max) ? g / (1.0f + expf(-z)) : 0.f;
        } else {
            const float l = a.zact[e];
            d = a.has_lp ? g * l * (1.0f - l) : 0.f;
        }
        dz[e] = d;
    }
}

/* column sums of dZ over the rows for the B / C bias gradients */
__global__ void k_colsum_acc(const float *dz, long rows, int W, int c0, int ncols, float *out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncols) return;
    float s = 0.f;
    for (long r = 0; r < rows; ++r) s += dz[r * W + c0 + c];
    out[c] += s;
}

/* ------------------------------------------------------------------ */
/* Mamba-3 scan                                                         */
/* ------------------------------------------------------------------ */

constexpr int kMaxR = 8;

struct ScanArgs {
    const float *zact;   /* [batch, L, W] */
    const float *A;      /* [N] (A_log used as A) */
    const float *theta;  /* [N/2] */
    float *h_hist;       /* [batch, L, N] or NULL */
    float *h_last;       /* [batch, N] final state, or NULL */
    float *part;         /* [batch, G, L, R (+2 backward)] per-warp partial sums */
    /* backward */
    const float *dy;     /* [batch, L, R] */
    float *dz;           /* [batch, L, W] (u, dt, lam, B, C columns) */
    float *dA;           /* [N], accumulated */
    float *dtheta;       /* [N/2], accumulated */
    int L, N, R, W, G;   /* G = warps (32-pair groups) per sequence */
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

/* The controls of one step as a thread of pair (n0, n0+1) needs them; RT
 * is a compile-time bound on the rank R so the arrays stay in registers. */
template <int RT>
struct StepIn {
    float dt, lam;
    float u[RT];
    float2 b[RT], c[RT];
    float2 h;      /* backward: the stored state pair h_t */
    float dy[RT];  /* backward: dy_t */
};

/* the backward's extra per-step inputs of step t */
template <int RT>
__device__ __forceinline__ void load_step_bwd(const float *hb, const float *dyb, int t, int R,
                                              int N, int n0, bool act, bool has1,
                                              StepIn<RT> &s) {
    s.h = make_float2(act ? hb[(long)t * N + n0] : 0.f, has1 ? hb[(long)t * N + n0 + 1] : 0.f);
#pragma unroll
    for (int r = 0; r < RT; ++r)
        if (r < R) s.dy[r] = dyb[(long)t * R + r];
}

template <int RT>
__device__ __forceinline__ void load_step(const float *row, int R, int N, int n0, bool act,
                                          bool has1, StepIn<RT> &s) {
    s.dt = row[R];
    s.lam = row[R + 1];
    const float *Bt = row + R + 2;
    const float *Ct = Bt + R * N;
#pragma unroll
    for (int r = 0; r < RT; ++r) {
        if (r < R) {
            s.u[r] = row[r];
            s.b[r] = make_float2(act ? Bt[r * N + n0] : 0.f, has1 ? Bt[r * N + n0 + 1] : 0.f);
            s.c[r] = make_float2(act ? Ct[r * N + n0] : 0.f, has1 ? Ct[r * N + n0 + 1] : 0.f);
        }
    }
}

/*
 * Mamba-3 scan.  A sequence runs on G one-warp CTAs, each owning 32 state
 * pairs (2i, 2i+1) (the rotation couples only a pair); the pairs are
 * independent chains, so only the sums over states (y, and in the
 * backward du / ddt / dlambda) need the other warps.  They go to `part`
 * and a second kernel adds the G partials in order.  Each step's controls
 * are loaded one step ahead.
 */
template <int RT>
__global__ void __launch_bounds__(32) k_m3_scan_fwd(ScanArgs a) {
    const int b = blockIdx.y, g = blockIdx.x;
    const int N = a.N, R = a.R, W = a.W, L = a.L;
    const int i = g * 32 + threadIdx.x; /* pair index */
    const int n0 = 2 * i;
    const bool act = n0 < N;
    const bool has1 = n0 + 1 < N; /* an odd N leaves its last state unrotated */
    float cv = 1.f, sv = 0.f, A0 = 0.f, A1 = 0.f;
    if (act) {
        A0 = a.A[n0];
        if (has1) {
            A1 = a.A[n0 + 1];
            const float th = a.theta[i];
            cv = cosf(th);
            sv = sinf(th);
        }
    }
    float h0 = 0.f, h1 = 0.f, pb0 = 0.f, pb1 = 0.f;
    const float *zb = a.zact + (long)b * L * W;
    float *part = a.part + ((long)b * a.G + g) * L * R;
    /* ring of PF steps loaded ahead; slot t % PF, compile-time in the
     * unrolled loop */
    constexpr int PF = RT <= 2 ? 4 : 2;
    StepIn<RT> ring[PF];
#pragma unroll
    for (int k = 0; k < PF; ++k)
        if (k < L) load_step(zb + (long)k * W, R, N, n0, act, has1, ring[k]);
    for (int t0 = 0; t0 < L; t0 += PF)
#pragma unroll
    for (int k = 0; k < PF; ++k) {
        const int t = t0 + k;
        if (t >= L) break;
        StepIn<RT> &cur = ring[k];
        const float dt = cur.dt, lam = cur.lam;
        float bu0 = 0.f, bu1 = 0.f;
        for (int r = 0; r < RT; ++r) {
            if (r >= R) break;
            bu0 += cur.b[r].x * cur.u[r];
            bu1 += cur.b[r].y * cur.u[r];
        }
        const float hr0 = has1 ? cv * h0 - sv * h1 : h0;
        const float hr1 = has1 ? sv * h0 + cv * h1 : h1;
        const float al0 = expf(dt * A0), al1 = expf(dt * A1);
        const float be0 = (1.0f - lam) * dt * al0, be1 = (1.0f - lam) * dt * al1;
        const float ga = lam * dt;
        h0 = act ? al0 * hr0 + be0 * pb0 + ga * bu0 : 0.f;
        h1 = has1 ? al1 * hr1 + be1 * pb1 + ga * bu1 : 0.f;
        pb0 = bu0;
        pb1 = bu1;
        if (a.h_hist && act) {
            float *hh = a.h_hist + ((long)b * L + t) * N;
            hh[n0] = h0;
            if (has1) hh[n0 + 1] = h1;
        }
        for (int r = 0; r < RT; ++r) {
            if (r >= R) break;
            const float yp = warp_sum(cur.c[r].x * h0 + cur.c[r].y * h1);
            if (threadIdx.x == 0) part[t * R + r] = yp;
        }
        if (t + PF < L) load_step(zb + (long)(t + PF) * W, R, N, n0, act, has1, cur);
    }
    if (a.h_last && act) {
        a.h_last[(long)b * N + n0] = h0;
        if (has1) a.h_last[(long)b * N + n0 + 1] = h1;
    }
}

template <int RT>
__global__ void __launch_bounds__(32) k_m3_scan_bwd(ScanArgs a) {
    const int b = blockIdx.y, g = blockIdx.x;
    const int N = a.N, R = a.R, W = a.W, L = a.L;
    const int i = g * 32 + threadIdx.x;
    const int n0 = 2 * i;
    const bool act = n0 < N;
    const bool has1 = n0 + 1 < N;
    const bool rot = has1;
    float cv = 1.f, sv = 0.f, A0 = 0.f, A1 = 0.f;
    if (act) {
        A0 = a.A[n0];
        if (has1) {
            A1 = a.A[n0 + 1];
            const float th = a.theta[i];
            cv = cosf(th);
            sv = sinf(th);
        }
    }
    const float *zb = a.zact + (long)b * L * W;
    float *dzb = a.dz + (long)b * L * W;
    const float *hb = a.h_hist + (long)b * L * N;
    const int RP = R + 2;
    float *part = a.part + ((long)b * a.G + g) * L * RP;
    /* carry = R^T(alpha_{t+1} * G_{t+1});  bg = beta_{t+1} * G_{t+1} */
    float c0 = 0.f, c1 = 0.f, bg0 = 0.f, bg1 = 0.f, sA0 = 0.f, sA1 = 0.f, sth = 0.f;
    /* ring of PF steps t, t-1, ... loaded ahead; step t sits in slot
     * (L-1-t) % PF, compile-time in the unrolled loop */
    constexpr int PF = RT <= 2 ? 4 : 2;
    StepIn<RT> ring[PF];
    const float *dyb = a.dy + (long)b * L * R;
#pragma unroll
    for (int k = 0; k < PF; ++k) {
        if (L - 1 - k >= 0) {
            load_step(zb + (long)(L - 1 - k) * W, R, N, n0, act, has1, ring[k]);
            load_step_bwd(hb, dyb, L - 1 - k, R, N, n0, act, has1, ring[k]);
        }
    }
    for (int j0 = 0; j0 < L; j0 += PF)
#pragma unroll
    for (int k = 0; k < PF; ++k) {
        const int t = L - 1 - (j0 + k);
        if (t < 0) break;
        StepIn<RT> &cur = ring[k];
        const StepIn<RT> &prv = ring[(k + 1) % PF];
        const float dt = cur.dt, lam = cur.lam;
        const float *dyt = cur.dy;
        float bu0 = 0.f, bu1 = 0.f, pb0 = 0.f, pb1 = 0.f;
        for (int r = 0; r < RT; ++r) {
            if (r >= R) break;
            bu0 += cur.b[r].x * cur.u[r];
            bu1 += cur.b[r].y * cur.u[r];
            if (t > 0) {
                pb0 += prv.b[r].x * prv.u[r];
                pb1 += prv.b[r].y * prv.u[r];
            }
        }
        const float hp0 = t > 0 ? prv.h.x : 0.f;
        const float hp1 = t > 0 ? prv.h.y : 0.f;
        const float ht0 = cur.h.x, ht1 = cur.h.y;
        float G0 = c0, G1 = c1;
        for (int r = 0; r < RT; ++r) {
            if (r >= R) break;
            G0 = fmaf(cur.c[r].x, dyt[r], G0);
            G1 = fmaf(cur.c[r].y, dyt[r], G1);
        }
        const float hr0 = rot ? cv * hp0 - sv * hp1 : hp0;
        const float hr1 = rot ? sv * hp0 + cv * hp1 : hp1;
        const float al0 = act ? expf(dt * A0) : 0.f, al1 = has1 ? expf(dt * A1) : 0.f;
        const float oml = 1.0f - lam;
        const float ga0 = G0 * (hr0 + oml * dt * pb0);
        const float ga1 = G1 * (hr1 + oml * dt * pb1);
        /* ddt, dlam */
        const float ddt = ga0 * A0 * al0 + G0 * (oml * al0 * pb0 + lam * bu0) +
                          ga1 * A1 * al1 + G1 * (oml * al1 * pb1 + lam * bu1);
        const float dlm = G0 * dt * (bu0 - al0 * pb0) + G1 * dt * (bu1 - al1 * pb1);
        sA0 = fmaf(ga0 * dt, al0, sA0);
        sA1 = fmaf(ga1 * dt, al1, sA1);
        /* Bu_t feeds h_t (gamma) and h_{t+1} (beta_{t+1}) */
        const float dbu0 = lam * dt * G0 + bg0;
        const float dbu1 = lam * dt * G1 + bg1;
        bg0 = oml * dt * al0 * G0;
        bg1 = oml * dt * al1 * G1;
        float *dzr = dzb + (long)t * W;
        for (int r = 0; r < RT; ++r) {
            if (r >= R) break;
            if (act) {
                dzr[R + 2 + r * N + n0] = dbu0 * cur.u[r];
                dzr[R + 2 + R * N + r * N + n0] = dyt[r] * ht0;
            }
            if (has1) {
                dzr[R + 2 + r * N + n0 + 1] = dbu1 * cur.u[r];
                dzr[R + 2 + R * N + r * N + n0 + 1] = dyt[r] * ht1;
            }
            const float du = warp_sum(dbu0 * cur.b[r].x + dbu1 * cur.b[r].y);
            if (threadIdx.x == 0) part[t * RP + r] = du;
        }
        {
            const float s_dt = warp_sum(ddt), s_lm = warp_sum(dlm);
            if (threadIdx.x == 0) {
                part[t * RP + R] = s_dt;
                part[t * RP + R + 1] = s_lm;
            }
        }
        /* rotation: h_rot = R h_{t-1};  d h_rot = alpha * G */
        const float dr0 = al0 * G0, dr1 = al1 * G1;
        if (rot) {
            sth += dr0 * (-sv * hp0 - cv * hp1) + dr1 * (cv * hp0 - sv * hp1);
            c0 = cv * dr0 + sv * dr1;
            c1 = -sv * dr0 + cv * dr1;
        } else {
            c0 = dr0;
            c1 = dr1;
        }
        if (t - PF >= 0) {
            load_step(zb + (long)(t - PF) * W, R, N, n0, act, has1, cur);
            load_step_bwd(hb, dyb, t - PF, R, N, n0, act, has1, cur);
        }
    }
    if (act) {
        atomicAdd(a.dA + n0, sA0);
        if (has1) atomicAdd(a.dA + n0 + 1, sA1);
        if (rot) atomicAdd(a.dtheta + i, sth);
    }
}

/* out[(b*L + t)*ldo + k] = sum_g part[((b*G + g)*L + t)*K + k], g in order */
__global__ void k_m3_fold(const float *part, int batch, int G, int L, int K, float *out,
                          long ldo) {
    const long tot = (long)batch * L * K;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < tot;
         e += (long)gridDim.x * blockDim.x) {
        const long k = e % K, bt = e / K, t = bt % L, b = bt / L;
        const float *p = part + ((b * G) * L + t) * K + k;
        float s = 0.f;
        for (int g = 0; g < G; ++g) s += p[(long)g * L * K];
        out[bt * ldo + k] = s;
    }
}

/* ------------------------------------------------------------------ */
/* model pieces                                                         */
/* ------------------------------------------------------------------ */

__global__ void k_embed_gather(const float *emb, const unsigned *tok, long L, long D, long V,
                               float *out) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < L * D;
         e += (long)gridDim.x * blockDim.x) {
        const long t = e / D, d = e % D;
        const unsigned id = tok[t];
        out[e] = id < V ? emb[(long)id * D + d] : 0.f;
    }
}

__global__ void k_embed_scatter(const float *dx, const unsigned *tok, long L, long D, long V,
                                float *gemb) {
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < L * D;
         e += (long)gridDim.x * blockDim.x) {
        const long t = e / D, d = e % D;
        const unsigned id = tok[t];
        if (id < V) atomicAdd(gemb + (long)id * D + d, dx[e]);
    }
}

/* One CTA per row: reference softmax (src/kmamba.c:29-52) and CE terms. */
__global__ void __launch_bounds__(256)
k_softmax_ce(const float *logits, const unsigned *tgt, long V, float invL, float *dlogits,
             float *row_loss) {
    __shared__ float red[32];
    __shared__ float bmax, bsum;
    const long t = blockIdx.x;
    const float *x = logits + t * V;
    float m = -INFINITY;
    for (long i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = x[i];
        if (!isnan(v) && !isinf(v)) m = fmaxf(m, v);
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = -INFINITY;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
        bmax = (isinf(mm) || isnan(mm)) ? 0.f : mm;
    }
    __syncthreads();
    const float mx = bmax;
    float s = 0.f;
    for (long i = threadIdx.x; i < V; i += blockDim.x) s += expf(fmaxf(x[i] - mx, -80.0f));
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) ss += red[w];
        bsum = ss < 1e-20f ? 1e-20f : ss;
    }
    __syncthreads();
    const float inv = 1.0f / bsum;
    const unsigned tg = tgt[t];
    if (tg >= (unsigned)V && threadIdx.x == 0) row_loss[t] = NAN; /* host rejects these */
    for (long i = threadIdx.x; i < V; i += blockDim.x) {
        const float p = expf(fmaxf(x[i] - mx, -80.0f)) * inv;
        float d = p * invL;
        if (i == (long)tg) {
            d -= invL;
            row_loss[t] = -logf(p < 1e-20f ? 1e-20f : p);
        }
        dlogits[t * V + i] = d;
    }
}

__global__ void k_adamw(float *p, const float *g, float *m, float *v, long n, float lr,
                        float b1, float b2, float eps, float wd, float bc1, float bc2) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const float gi = g[i];
        const float mi = b1 * m[i] + (1.0f - b1) * gi;
        const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
        m[i] = mi;
        v[i] = vi;
        const float mh = mi / bc1, vh = vi / bc2;
        p[i] = p[i] * (1.0f - lr * wd) - lr * mh / (sqrtf(vh) + eps);
    }
}

/* Up to kMaxTens tensors per launch (blockIdx.y picks the tensor). */
constexpr int kMaxTens = 16;
struct AdamList {
    float *p[kMaxTens];
    const float *g[kMaxTens];
    float *m[kMaxTens], *v[kMaxTens];
    long n[kMaxTens];
};
struct SqList {
    const float *x[kMaxTens];
    long n[kMaxTens];
    double *out[kMaxTens];
};

__global__ void k_adamw_multi(AdamList t, float lr, float b1, float b2, float eps, float wd,
                              float bc1, float bc2) {
    const int k = blockIdx.y;
    float *p = t.p[k], *m = t.m[k], *v = t.v[k];
    const float *g = t.g[k];
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < t.n[k];
         i += (long)gridDim.x * blockDim.x) {
        const float gi = g[i];
        const float mi = b1 * m[i] + (1.0f - b1) * gi;
        const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
        m[i] = mi;
        v[i] = vi;
        const float mh = mi / bc1, vh = vi / bc2;
        p[i] = p[i] * (1.0f - lr * wd) - lr * mh / (sqrtf(vh) + eps);
    }
}

__global__ void __launch_bounds__(256) k_sumsq_multi(SqList t) {
    __shared__ double red[8];
    const int k = blockIdx.y;
    const float *x = t.x[k];
    double s = 0.0;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < t.n[k];
         i += (long)gridDim.x * blockDim.x)
        s += (double)x[i] * x[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double b = 0.0;
        for (int w = 0; w < 8; ++w) b += red[w];
        if (b != 0.0) atomicAdd(t.out[k], b); /* one atomic per block */
    }
}

__global__ void k_sumsq(const float *x, long n, double *out) {
    double s = 0.0;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        s += (double)x[i] * x[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, s);
}

/* y = a*y + b*x */
__global__ void k_axpby(float *y, const float *x, long n, float a, float b) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        y[i] = x ? a * y[i] + b * x[i] : a * y[i];
}

/* dt = clamp(softplus(z), dt_min, dt_max) */
__global__ void k_dt_act(const float *z, float *out, long n, float dt_min, float dt_max) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        float v = logf(1.0f + expf(z[i]));
        if (v < dt_min) v = dt_min;
        if (v > dt_max) v = dt_max;
        out[i] = v;
    }
}

/* m = mu*m + g (momentum of the MUON optimizer) */
__global__ void k_momentum(float *m, const float *g, long n, float mu) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        m[i] = mu * m[i] + g[i];
}

/* G = 1.5 G - 0.5 T (one Newton-Schulz step after T = G G^T G) */
__global__ void k_ns_combine(float *G, const float *T, long n) {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        G[i] = 1.5f * G[i] - 0.5f * T[i];
}

/* p -= lr * x * scale, scale = clip / ||x|| when ||x|| > clip (sumsq from
 * k_sumsq), else 1; sumsq == NULL gives scale 1 (plain SGD) */
__global__ void k_scaled_sub(float *p, const float *x, long n, float lr, float clip,
                             const double *sumsq) {
    float scale = 1.0f;
    if (sumsq) {
        const float norm = sqrtf((float)*sumsq);
        scale = norm > clip ? clip / norm : 1.0f;
    }
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        p[i] -= lr * x[i] * scale;
}

unsigned grid1d(long n) {
    long b = (n + 255) / 256;
    if (b > 148L * 16) b = 148L * 16;
    return (unsigned)(b < 1 ? 1 : b);
}

unsigned long long g_launches = 0; /* kernels launched by this file */

inline void count_launch() { __atomic_fetch_add(&g_launches, 1ULL, __ATOMIC_RELAXED); }

} // namespace

extern "C" unsigned long long kmb_block_launch_count(void) {
    return __atomic_load_n(&g_launches, __ATOMIC_RELAXED);
}

extern "C" int kmb_gemm(int M, int N, int K, const float *A, long am, long ak, const float *B,
                        long bk, long bn, float *C, long ldc, int accumulate, float *ws,
                        size_t ws_elems, cudaStream_t s) {
    if (M <= 0 || N <= 0) return KMB_OK;
    if (K <= 0) {
        if (!accumulate) {
            for (int m = 0; m < M; ++m) {
                cudaError_t e = cudaMemsetAsync(C + (long)m * ldc, 0, sizeof(float) * N, s);
                if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm memset");
            }
        }
        return KMB_OK;
    }
    cudaError_t e;
    if (N == 1) {
        count_launch();
        k_gemv_n1<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(M, K, A, am, ak, B, bk, C, ldc,
                                                            accumulate);
    } else if (M == 1) {
        count_launch();
        k_gemv_m1<<<(unsigned)((N + 31) / 32), 256, 0, s>>>(N, K, A, ak, B, bk, bn, C,
                                                             accumulate);
    } else {
        const long tiles = (long)((N + kTN - 1) / kTN) * ((M + kTM - 1) / kTM);
        /* split K when the output grid leaves most SMs idle: enough slices
         * for ~2 CTAs per SM, each at least 2 k-tiles deep, within ws */
        int S = 1;
        if (ws && tiles < 148) {
            long want = (296 + tiles - 1) / tiles;
            long maxs = K / (2 * kTK);
            long fit = (long)(ws_elems / ((size_t)M * N));
            S = (int)min(want, min(maxs, fit));
            if (S < 2) S = 1;
        }
        dim3 grid((unsigned)((N + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM), (unsigned)S);
        if (S == 1) {
            count_launch();
            k_gemm<<<grid, 256, 0, s>>>(M, N, K, A, am, ak, B, bk, bn, C, ldc, accumulate,
                                        nullptr, K);
        } else {
            const int kchunk = ((K + S - 1) / S + kTK - 1) / kTK * kTK;
            S = (K + kchunk - 1) / kchunk;
            grid.z = (unsigned)S;
            count_launch();
            k_gemm<<<grid, 256, 0, s>>>(M, N, K, A, am, ak, B, bk, bn, C, ldc, accumulate, ws,
                                        kchunk);
            e = cudaGetLastError();
            if (e != cudaSuccess) return kmb_cuda_fail(e, "gemm launch");
            const long tot = (long)M * N;
            count_launch();
            k_gemm_reduce<<<(unsigned)min((tot + 255) / 256, 148L * 8), 256, 0, s>>>(
                ws, S, M, N, C, ldc, accumulate);
        }
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "gemm launch");
}

extern "C" int kmb_block_act(const float *zraw, float *zact, const float *bB, const float *bC,
                             long rows, int W, int R, int NR, float dt_min, float dt_max,
                             int has_dp, int has_lp, float dt_scale, float *dz_inplace,
                             cudaStream_t s) {
    ActArgs a{zraw, zact, bB, bC, rows, W, R, NR, dt_min, dt_max, has_dp, has_lp, dt_scale};
    if (dz_inplace) {
        count_launch();
        k_block_act_bwd<<<grid1d(rows * W), 256, 0, s>>>(a, dz_inplace);
    } else {
        count_launch();
        k_block_act<<<grid1d(rows * W), 256, 0, s>>>(a);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "block activation launch");
}

extern "C" int kmb_colsum_acc(const float *dz, long rows, int W, int c0, int ncols, float *out,
                              cudaStream_t s) {
    count_launch();
    k_colsum_acc<<<(unsigned)((ncols + 127) / 128), 128, 0, s>>>(dz, rows, W, c0, ncols, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "colsum launch");
}

extern "C" int kmb_m3_scan(int batch, int L, int N, int R, int W, const float *zact,
                           const float *A, const float *theta, float *h_hist, float *h_last,
                           float *y, const float *dy, float *dz, float *dA, float *dtheta,
                           float *part, cudaStream_t s) {
    if (R > kMaxR) return kmb_fail(KMB_EUNSUPPORTED, "block: mimo_rank %d exceeds %d", R, kMaxR);
    if (dy && !h_hist) return kmb_fail(KMB_EINVAL, "block scan backward needs the state history");
    const int G = kmb_m3_scan_groups(N);
    ScanArgs a{zact, A, theta, h_hist, h_last, part, dy, dz, dA, dtheta, L, N, R, W, G};
    dim3 grid((unsigned)G, (unsigned)batch);
    const int K = dy ? R + 2 : R;
    count_launch();
    if (dy) {
        if (R <= 1) k_m3_scan_bwd<1><<<grid, 32, 0, s>>>(a);
        else if (R <= 2) k_m3_scan_bwd<2><<<grid, 32, 0, s>>>(a);
        else if (R <= 4) k_m3_scan_bwd<4><<<grid, 32, 0, s>>>(a);
        else k_m3_scan_bwd<8><<<grid, 32, 0, s>>>(a);
    } else {
        if (R <= 1) k_m3_scan_fwd<1><<<grid, 32, 0, s>>>(a);
        else if (R <= 2) k_m3_scan_fwd<2><<<grid, 32, 0, s>>>(a);
        else if (R <= 4) k_m3_scan_fwd<4><<<grid, 32, 0, s>>>(a);
        else k_m3_scan_fwd<8><<<grid, 32, 0, s>>>(a);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return kmb_cuda_fail(e, "block scan launch");
    const long tot = (long)batch * L * K;
    count_launch();
    k_m3_fold<<<(unsigned)min((tot + 255) / 256, 148L * 8), 256, 0, s>>>(
        part, batch, G, L, K, dy ? dz : y, dy ? (long)W : (long)R);
    e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "block scan fold launch");
}

extern "C" int kmb_m3_scan_groups(int N) { return ((N + 1) / 2 + 31) / 32; }

extern "C" int kmb_embed(const float *emb, const unsigned *tok, long L, long D, long V,
                         float *out, const float *dx_for_grad, float *gemb, cudaStream_t s) {
    if (gemb) {
        count_launch();
        k_embed_scatter<<<grid1d(L * D), 256, 0, s>>>(dx_for_grad, tok, L, D, V, gemb);
    } else {
        count_launch();
        k_embed_gather<<<grid1d(L * D), 256, 0, s>>>(emb, tok, L, D, V, out);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "embedding launch");
}

extern "C" int kmb_softmax_ce(const float *logits, const unsigned *tgt, long L, long V,
                              float *dlogits, float *row_loss, cudaStream_t s) {
    count_launch();
    k_softmax_ce<<<(unsigned)L, 256, 0, s>>>(logits, tgt, V, 1.0f / (float)L, dlogits, row_loss);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "softmax-ce launch");
}

extern "C" int kmb_adamw(float *p, const float *g, float *m, float *v, long n, float lr,
                         float b1, float b2, float eps, float wd, float bc1, float bc2,
                         cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_adamw<<<grid1d(n), 256, 0, s>>>(p, g, m, v, n, lr, b1, b2, eps, wd, bc1, bc2);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "adamw launch");
}

extern "C" int kmb_sumsq(const float *x, long n, double *out, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_sumsq<<<grid1d(n), 256, 0, s>>>(x, n, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "sumsq launch");
}

#define KMB_ELEMWISE_RET(what)                                                       \
    do {                                                                             \
        cudaError_t e_ = cudaGetLastError();                                         \
        return e_ == cudaSuccess ? KMB_OK : kmb_cuda_fail(e_, what);                 \
    } while (0)

extern "C" int kmb_axpby(float *y, const float *x, long n, float a, float b, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_axpby<<<grid1d(n), 256, 0, s>>>(y, x, n, a, b);
    KMB_ELEMWISE_RET("axpby launch");
}

extern "C" int kmb_dt_act(const float *z, float *out, long n, float dt_min, float dt_max,
                          cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_dt_act<<<grid1d(n), 256, 0, s>>>(z, out, n, dt_min, dt_max);
    KMB_ELEMWISE_RET("dt activation launch");
}

extern "C" int kmb_momentum(float *m, const float *g, long n, float mu, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_momentum<<<grid1d(n), 256, 0, s>>>(m, g, n, mu);
    KMB_ELEMWISE_RET("momentum launch");
}

extern "C" int kmb_ns_combine(float *G, const float *T, long n, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_ns_combine<<<grid1d(n), 256, 0, s>>>(G, T, n);
    KMB_ELEMWISE_RET("newton-schulz launch");
}

extern "C" int kmb_scaled_sub(float *p, const float *x, long n, float lr, float clip,
                              const double *sumsq, cudaStream_t s) {
    if (n <= 0) return KMB_OK;
    count_launch();
    k_scaled_sub<<<grid1d(n), 256, 0, s>>>(p, x, n, lr, clip, sumsq);
    KMB_ELEMWISE_RET("scaled update launch");
}

/* AdamW over up to 16 tensors at once (the k_adamw rule per element) */
extern "C" int kmb_adamw_multi(int cnt, float *const *p, const float *const *g, float *const *m,
                               float *const *v, const long *n, float lr, float b1, float b2,
                               float eps, float wd, float bc1, float bc2, cudaStream_t s) {
    if (cnt <= 0) return KMB_OK;
    if (cnt > kMaxTens) return kmb_fail(KMB_EINVAL, "adamw: at most %d tensors", kMaxTens);
    AdamList t;
    long mx = 1;
    for (int k = 0; k < cnt; ++k) {
        t.p[k] = p[k];
        t.g[k] = g[k];
        t.m[k] = m[k];
        t.v[k] = v[k];
        t.n[k] = n[k];
        if (n[k] > mx) mx = n[k];
    }
    count_launch();
    k_adamw_multi<<<dim3(grid1d(mx), (unsigned)cnt), 256, 0, s>>>(t, lr, b1, b2, eps, wd, bc1,
                                                                 bc2);
    KMB_ELEMWISE_RET("adamw launch");
}

/* out[k] += sum x_k^2 in double for up to 16 tensors */
extern "C" int kmb_sumsq_multi(int cnt, const float *const *x, const long *n,
                               double *const *out, cudaStream_t s) {
    if (cnt <= 0) return KMB_OK;
    if (cnt > kMaxTens) return kmb_fail(KMB_EINVAL, "sumsq: at most %d tensors", kMaxTens);
    SqList t;
    long mx = 1;
    for (int k = 0; k < cnt; ++k) {
        t.x[k] = x[k];
        t.n[k] = n[k];
        t.out[k] = out[k];
        if (n[k] > mx) mx = n[k];
    }
    const unsigned gx = (unsigned)min((mx + 255) / 256, 148L * 2);
    count_launch();
    k_sumsq_multi<<<dim3(gx, (unsigned)cnt), 256, 0, s>>>(t);
    KMB_ELEMWISE_RET("sumsq launch");
}
