/*
 * CPU ORACLE — test infrastructure only.
 *
 * Plain-C restatement of the reference k-mamba CPU path for the hot path,
 * used by tests/ and by bench.py's CPU-baseline leg to check and time the
 * GPU library.  Nothing in the product links or calls this file.
 *
 * Arithmetic follows the reference's operation order in scalar fp32 with
 * no FMA contraction (build with -ffp-contract=off) and glibc expf:
 *   or_scan1d_fwd    cpu/scan1d.asm:88-152 (the asm cannot be assembled
 *                    here: nasm is absent; this is its instruction order)
 *   or_scan2d_fwd    cpu/scan2d.asm:125-256
 *   or_scan1d_bwd    cpu/scan1d_backward.c:248-295
 *   or_scannd_fwd    src/scan_nd.c:86-230 (theta = lambda = NULL branch)
 *   or_convnd_fwd    src/convnd.c:67-129
 *   or_convnd_bwd    src/convnd.c:135-202
 * The 2D/ND backward (or_scannd_bwd) has no reference implementation: it
 * is the adjoint of or_scannd_fwd written from the recurrence and is
 * pinned by central finite differences in the tests.
 *
 * Every function handles one batch item.  B/C (and dB/dC) are addressed
 * as base + t*sBt + d*sBd + m so that the [L,D,M] reference layout
 * (sBt = D*M, sBd = M) and the channel-shared [L,M] layout (sBt = M,
 * sBd = 0) use the same loop; with sBd = 0 the gradients dB/dC are summed
 * over channels in ascending d order.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* 1D                                                                  */
/* ------------------------------------------------------------------ */

/* h [D,M] is the running state (read and overwritten).  h_all [L,D,M] is
 * optional.  clamp != 0 applies min(h,1000) then max(h,-1000), with NaN
 * becoming 1000 as SSE minss does. */
void or_scan1d_fwd(const float *x, const float *delta, const float *A, const float *B,
                   const float *C, float *h, float *y, float *h_all, long L, long D,
                   long M, long sBt, long sBd, int clamp) {
    for (long t = 0; t < L; t++) {
        for (long d = 0; d < D; d++) {
            const long td = t * D + d;
            float yacc = 0.0f;
            for (long m = 0; m < M; m++) {
                const long dm = d * M + m;
                const long bi = t * sBt + d * sBd + m;
                const float dt = delta[td];
                const float dA = expf(dt * A[dm]);
                const float dB = B[bi] * dt;
                const float xt = x[td];
                float hn = dA * h[dm];
                hn = hn + dB * xt;
                if (clamp) {
                    hn = (hn < 1000.0f) ? hn : 1000.0f;
                    hn = (hn > -1000.0f) ? hn : -1000.0f;
                }
                h[dm] = hn;
                if (h_all) h_all[td * M + m] = hn;
                yacc = yacc + C[bi] * hn;
            }
            y[td] = yacc;
        }
    }
}

/* Generic reverse adjoint; h [L,D,M] stored states, h0 [D,M] or NULL.
 * Gradients are zeroed first.  dB/dC use the B/C strides (sBd = 0 sums
 * over channels). */
void or_scan1d_bwd(const float *x, const float *delta, const float *A, const float *B,
                   const float *C, const float *h0, const float *h, const float *dy,
                   float *dx, float *ddelta, float *dA, float *dB, float *dC, long L, long D,
                   long M, long sBt, long sBd) {
    float *adj = (float *)calloc((size_t)(D * M), sizeof(float));
    const long nbc = (L - 1) * sBt + (D - 1) * sBd + M;
    if (!adj) return;
    memset(dx, 0, sizeof(float) * (size_t)(L * D));
    memset(ddelta, 0, sizeof(float) * (size_t)(L * D));
    memset(dA, 0, sizeof(float) * (size_t)(D * M));
    memset(dB, 0, sizeof(float) * (size_t)nbc);
    memset(dC, 0, sizeof(float) * (size_t)nbc);
    for (long t = L - 1; t >= 0; t--) {
        for (long d = 0; d < D; d++) {
            const long td = t * D + d;
            const float dt = delta[td];
            const float xt = x[td];
            const float g = dy[td];
            float ddt = 0.0f;
            for (long m = 0; m < M; m++) {
                const long dm = d * M + m;
                const long tdm = td * M + m;
                const long bi = t * sBt + d * sBd + m;
                const float a = A[dm];
                const float b = B[bi];
                const float c = C[bi];
                const float e = expf(dt * a);
                float hp = 0.0f;
                float ah;
                if (t > 0) hp = h[tdm - D * M];
                else if (h0) hp = h0[dm];
                ah = adj[dm] + g * c;
                dC[bi] += g * h[tdm];
                dB[bi] += ah * dt * xt;
                dA[dm] += ah * dt * e * hp;
                dx[td] += ah * dt * b;
                ddt += ah * (a * e * hp + b * xt);
                adj[dm] = ah * e;
            }
            ddelta[td] += ddt;
        }
    }
    free(adj);
}

/* ------------------------------------------------------------------ */
/* 2D (scan2d asm order)                                               */
/* ------------------------------------------------------------------ */

void or_scan2d_fwd(const float *x, const float *A1, const float *A2, const float *B,
                   const float *C, const float *delta1, const float *delta2, float *h,
                   float *y, long d1, long d2, long D, long M, long sBp, long sBd) {
    const long DM = D * M;
    for (long k = 0; k < d1 + d2 - 1; k++) {
        long i_min = k - d2 + 1;
        long i_max = k < d1 - 1 ? k : d1 - 1;
        if (i_min < 0) i_min = 0;
        for (long i = i_min; i <= i_max; i++) {
            const long j = k - i;
            const long pos = i * d2 + j;
            for (long d = 0; d < D; d++) {
                const long pd = pos * D + d;
                float yacc = 0.0f;
                for (long m = 0; m < M; m++) {
                    const long dm = d * M + m;
                    const long pdm = pos * DM + dm;
                    const long bi = pos * sBp + d * sBd + m;
                    const float h1 = i > 0 ? h[(pos - d2) * DM + dm] : 0.0f;
                    const float h2 = j > 0 ? h[(pos - 1) * DM + dm] : 0.0f;
                    const float dA1 = expf(delta1[pd] * A1[dm]);
                    const float dA2 = expf(delta2[pd] * A2[dm]);
                    const float hs = (delta1[pd] + delta2[pd]) * 0.5f;
                    const float dB = B[bi] * hs;
                    float hn = dA1 * h1;
                    hn = hn + dA2 * h2;
                    hn = hn + dB * x[pd];
                    h[pdm] = hn;
                    yacc = yacc + C[bi] * hn;
                }
                y[pd] = yacc;
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* ND (scannd_ref order)                                               */
/* ------------------------------------------------------------------ */

static void make_strides(const long *dims, long ndims, long *st) {
    long s = 1;
    for (long a = ndims - 1; a >= 0; a--) {
        st[a] = s;
        s *= dims[a];
    }
}

/* Offsets of the grid in wavefront order: ascending coordinate sum, then
 * ascending row-major offset (the order of km_wavefront_plan_create). */
static long *wave_order(const long *dims, long ndims, long P) {
    long *st = (long *)malloc(sizeof(long) * (size_t)ndims);
    long maxl = 0, *cnt, *ord;
    for (long a = 0; a < ndims; a++) maxl += dims[a] - 1;
    cnt = (long *)calloc((size_t)maxl + 2, sizeof(long));
    ord = (long *)malloc(sizeof(long) * (size_t)P);
    make_strides(dims, ndims, st);
    for (long p = 0; p < P; p++) {
        long lv = 0;
        for (long a = 0; a < ndims; a++) lv += (p / st[a]) % dims[a];
        cnt[lv + 1]++;
    }
    for (long l = 0; l <= maxl; l++) cnt[l + 1] += cnt[l];
    for (long p = 0; p < P; p++) {
        long lv = 0;
        for (long a = 0; a < ndims; a++) lv += (p / st[a]) % dims[a];
        ord[cnt[lv]++] = p;
    }
    free(cnt);
    free(st);
    return ord;
}

/* x [P,D]; A [ndims,D,M]; B, C: base + p*sBp + d*sBd + m; delta
 * [ndims,P,D]; h [P,D,M]; y [P,D]. */
void or_scannd_fwd(const long *dims, long ndims, const float *x, const float *A,
                   const float *B, const float *C, const float *delta, float *h, float *y,
                   long D, long M, long sBp, long sBd) {
    long P = 1, st[16], idx[16];
    long *ord;
    for (long a = 0; a < ndims; a++) P *= dims[a];
    make_strides(dims, ndims, st);
    ord = wave_order(dims, ndims, P);
    for (long q = 0; q < P; q++) {
        const long off = ord[q];
        for (long a = 0; a < ndims; a++) idx[a] = (off / st[a]) % dims[a];
        for (long d = 0; d < D; d++) {
            const float xv = x[off * D + d];
            float dt_bar = 0.0f, yacc = 0.0f;
            for (long a = 0; a < ndims; a++) dt_bar += delta[(a * P + off) * D + d];
            dt_bar /= (float)ndims;
            for (long m = 0; m < M; m++) {
                const long dm = d * M + m;
                const long pdm = off * D * M + dm;
                const long bi = off * sBp + d * sBd + m;
                const float bu = B[bi] * xv;
                float hn = dt_bar * bu;
                for (long a = 0; a < ndims; a++) {
                    if (idx[a] > 0) {
                        const long prev = (off - st[a]) * D * M + dm;
                        const float dta = delta[(a * P + off) * D + d];
                        const float decay = expf(dta * A[(a * D + d) * M + m]);
                        hn += decay * h[prev];
                    }
                }
                h[pdm] = hn;
                yacc += C[bi] * hn;
            }
            y[off * D + d] = yacc;
        }
    }
    free(ord);
}

/* Adjoint of or_scannd_fwd (no reference: written from the recurrence).
 *   G(p)   = C(p) dy(p) + sum_a exp(delta_a(p+e_a) A_a) G(p+e_a)
 *   dC     = dy h;   dB = G dt_bar x;   dx = sum_m G dt_bar B
 *   ddelta_a(p) = (sum_m G B x) / ndims
 *               + sum_m G h(p-e_a) A_a exp(delta_a A_a)
 *   dA_a   = sum_p G h(p-e_a) delta_a exp(delta_a A_a)
 * Levels are visited in reverse wavefront order.  Gradients are zeroed;
 * with sBd = 0, dB/dC are summed over channels. */
void or_scannd_bwd(const long *dims, long ndims, const float *x, const float *A,
                   const float *B, const float *C, const float *delta, const float *h,
                   const float *dy, float *dx, float *dA, float *dB, float *dC, float *ddelta,
                   long D, long M, long sBp, long sBd) {
    long P = 1, st[16], idx[16];
    long *ord;
    float *G;
    for (long a = 0; a < ndims; a++) P *= dims[a];
    make_strides(dims, ndims, st);
    ord = wave_order(dims, ndims, P);
    G = (float *)calloc((size_t)(P * D * M), sizeof(float));
    memset(dx, 0, sizeof(float) * (size_t)(P * D));
    memset(ddelta, 0, sizeof(float) * (size_t)(ndims * P * D));
    memset(dA, 0, sizeof(float) * (size_t)(ndims * D * M));
    {
        const long nbc = (P - 1) * sBp + (D - 1) * sBd + M;
        memset(dB, 0, sizeof(float) * (size_t)nbc);
        memset(dC, 0, sizeof(float) * (size_t)nbc);
    }
    for (long q = P - 1; q >= 0; q--) {
        const long off = ord[q];
        for (long a = 0; a < ndims; a++) idx[a] = (off / st[a]) % dims[a];
        for (long d = 0; d < D; d++) {
            const float xv = x[off * D + d];
            const float g_y = dy[off * D + d];
            float dt_bar = 0.0f, sx = 0.0f, sbar = 0.0f;
            for (long a = 0; a < ndims; a++) dt_bar += delta[(a * P + off) * D + d];
            dt_bar /= (float)ndims;
            for (long m = 0; m < M; m++) {
                const long dm = d * M + m;
                const long pdm = off * D * M + dm;
                const long bi = off * sBp + d * sBd + m;
                /* G(p) already holds the contributions of the successors */
                const float gg = G[pdm] + C[bi] * g_y;
                dC[bi] += g_y * h[pdm];
                dB[bi] += gg * dt_bar * xv;
                sx += gg * dt_bar * B[bi];
                sbar += gg * B[bi] * xv;
                for (long a = 0; a < ndims; a++) {
                    if (idx[a] > 0) {
                        const long prev = (off - st[a]) * D * M + dm;
                        const float dta = delta[(a * P + off) * D + d];
                        const float aa = A[(a * D + d) * M + m];
                        const float e = expf(dta * aa);
                        dA[(a * D + d) * M + m] += gg * h[prev] * dta * e;
                        ddelta[(a * P + off) * D + d] += gg * h[prev] * aa * e;
                        G[prev] += e * gg;
                    }
                }
            }
            dx[off * D + d] = sx;
            for (long a = 0; a < ndims; a++)
                ddelta[(a * P + off) * D + d] += sbar / (float)ndims;
        }
    }
    free(G);
    free(ord);
}

/* ------------------------------------------------------------------ */
/* ConvND                                                              */
/* ------------------------------------------------------------------ */

long or_wavefront_plan(const long *dims, long ndims, long *level_starts, long *level_offsets);

static long ipow(long b, long e) {
    long r = 1;
    while (e-- > 0) r *= b;
    return r;
}

/* Source offset of output `out` for kernel tap kl, or -1 outside. */
static long conv_src(const long *dims, long ndims, const long *st, long K, long out, long kl) {
    long src = 0, tmp = kl;
    for (long a = ndims - 1; a >= 0; a--) {
        const long ka = tmp % K;
        const long c = (out / st[a]) % dims[a] - (K - 1 - ka);
        tmp /= K;
        if (c < 0 || c >= dims[a]) return -1;
        src += c * st[a];
    }
    return src;
}

void or_convnd_fwd(const long *dims, long ndims, long D, long K, const float *input,
                   const float *kernel, const float *bias, float *output) {
    long P = 1, st[16];
    const long KV = ipow(K, ndims);
    long *ord;
    for (long a = 0; a < ndims; a++) P *= dims[a];
    make_strides(dims, ndims, st);
    ord = wave_order(dims, ndims, P);
    for (long q = 0; q < P; q++) {
        const long out = ord[q];
        for (long d = 0; d < D; d++) {
            float s = bias ? bias[d] : 0.0f;
            for (long kl = 0; kl < KV; kl++) {
                const long src = conv_src(dims, ndims, st, K, out, kl);
                if (src < 0) continue;
                s += input[src * D + d] * kernel[kl * D + d];
            }
            output[out * D + d] = s;
        }
    }
    free(ord);
}

void or_convnd_bwd(const long *dims, long ndims, long D, long K, const float *input,
                   const float *kernel, const float *dy, float *dinput, float *dkernel,
                   float *dbias) {
    long P = 1, st[16];
    const long KV = ipow(K, ndims);
    long *ord;
    for (long a = 0; a < ndims; a++) P *= dims[a];
    make_strides(dims, ndims, st);
    ord = wave_order(dims, ndims, P);
    memset(dinput, 0, sizeof(float) * (size_t)(P * D));
    memset(dkernel, 0, sizeof(float) * (size_t)(KV * D));
    if (dbias) memset(dbias, 0, sizeof(float) * (size_t)D);
    /* levels descending, points of a level ascending (src/convnd.c:159-164) */
    long maxl = 0, *lst;
    for (long a = 0; a < ndims; a++) maxl += dims[a] - 1;
    lst = (long *)malloc(sizeof(long) * (size_t)(maxl + 2));
    or_wavefront_plan(dims, ndims, lst, ord);
    for (long q = 0, lv = maxl; lv >= 0; lv--)
    for (long qq = lst[lv]; qq < lst[lv + 1]; qq++, q++) {
        const long out = ord[qq];
        for (long d = 0; d < D; d++) {
            const float g = dy[out * D + d];
            if (dbias) dbias[d] += g;
            for (long kl = 0; kl < KV; kl++) {
                const long src = conv_src(dims, ndims, st, K, out, kl);
                if (src < 0) continue;
                dkernel[kl * D + d] += g * input[src * D + d];
                dinput[src * D + d] += g * kernel[kl * D + d];
            }
        }
    }
    free(lst);
    free(ord);
}

/* ------------------------------------------------------------------ */
/* wavefront plan (integer)                                            */
/* ------------------------------------------------------------------ */

/* Writes level_starts [max_level + 2] and level_offsets [P]; returns P. */
long or_wavefront_plan(const long *dims, long ndims, long *level_starts, long *level_offsets) {
    long P = 1, maxl = 0, st[16];
    long *ord;
    for (long a = 0; a < ndims; a++) {
        P *= dims[a];
        maxl += dims[a] - 1;
    }
    make_strides(dims, ndims, st);
    ord = wave_order(dims, ndims, P);
    memcpy(level_offsets, ord, sizeof(long) * (size_t)P);
    memset(level_starts, 0, sizeof(long) * (size_t)(maxl + 2));
    for (long p = 0; p < P; p++) {
        long lv = 0;
        for (long a = 0; a < ndims; a++) lv += (p / st[a]) % dims[a];
        level_starts[lv + 1]++;
    }
    for (long l = 0; l <= maxl; l++) level_starts[l + 1] += level_starts[l];
    free(ord);
    return P;
}
