/*
 * CPU ORACLE — test infrastructure only (bench.py's CPU-baseline and
 * reference legs).  Nothing in the product links or calls this file.
 *
 * Timed driver of the reference's CPU path for the 1D selective scan
 * forward + backward, run on the host cores:
 *   forward   scannd_ref with ndims = 1      (src/scan_nd.c:235)
 *   backward  scan1d_backward                (cpu/scan1d_backward.c:297)
 * when built into oracle/_ref/libkmamba_ref.so (-DKMB_BENCH_REF), or the
 * C restatement of the same two functions (or_scan1d_fwd / or_scan1d_bwd,
 * kmb_oracle.c) when built into liboracle.so.
 *
 * The work is split into channel slices of one batch item (full L, all N
 * states, B / C expanded to the reference's [L, D, N] layout) and run
 * under one OpenMP parallel loop.  Every worker is an OpenMP thread with
 * its own omp_get_thread_num(), so the reference's thread-local memory
 * pools (src/km_memory_pool.c:117-146, keyed by that number) are distinct
 * per worker; scannd_ref's own inner parallel loop runs nested and
 * therefore single-threaded, which also keeps its shared `idx` buffer
 * (src/scan_nd.c:45, 86, 95) private to one thread.
 *
 * Inputs follow the config-2 distributions from a counter-based generator
 * (splitmix64, Box-Muller): x, dy ~ N(0,1); dt = softplus(N(0,1) - 2);
 * A = -exp(U[0, ln 16]); B, C ~ N(0,1) per (t, n), shared by the slice's
 * channels.  Every buffer is written (first touch) by the worker that
 * later runs its slice, before any timing.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <omp.h>

#ifdef KMB_BENCH_REF
/* layouts of the reference's include/scan_nd.h:26-40 and include/scan.h */
typedef struct {
    const long *dims;
    long ndims, D, M;
    const float *x, *A, *B, *C, *delta;
    float *h, *y;
    const float *theta, *lambda;
} BenchNDParams;
typedef struct {
    float *x, *A, *B, *C, *delta, *h0, *h, *dy;
    float *dx, *dA, *dB, *dC, *ddelta;
    long L, D, M;
} BenchBwdParams;
int scannd_ref(BenchNDParams *p);
void scan1d_backward(BenchBwdParams *p);
#else
void or_scan1d_fwd(const float *x, const float *delta, const float *A, const float *B,
                   const float *C, float *h, float *y, float *h_all, long L, long D, long M,
                   long sBt, long sBd, int clamp);
void or_scan1d_bwd(const float *x, const float *delta, const float *A, const float *B,
                   const float *C, const float *h0, const float *h_all, const float *dy,
                   float *dx, float *ddt, float *dA, float *dB, float *dC, long L, long D,
                   long M, long sBt, long sBd);
#endif

typedef struct {
    float *x, *dt, *A, *B, *C, *dy;       /* inputs */
    float *h, *y, *dx, *ddt, *dA, *dB, *dC; /* outputs (h: the state history) */
    float *state;                          /* [D, N] running state (port only) */
} BenchSlice;

typedef struct {
    int slices, chans, N, threads;
    long L;
    BenchSlice *s;
} BenchRun;

static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* uniform in (0, 1) from a 64-bit counter */
static double unif(uint64_t key) { return ((mix64(key) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

static float normal(uint64_t key) {
    const double u1 = unif(2 * key), u2 = unif(2 * key + 1);
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

static void fill_slice(BenchRun *r, int i, uint64_t seed) {
    BenchSlice *s = &r->s[i];
    const long L = r->L, D = r->chans, N = r->N;
    const uint64_t base = seed * 0x100000000ull + (uint64_t)i * 0x1000000ull * 16;
    uint64_t k = base;
    for (long e = 0; e < L * D; ++e) s->x[e] = normal(k++);
    for (long e = 0; e < L * D; ++e) s->dy[e] = normal(k++);
    for (long e = 0; e < L * D; ++e) s->dt[e] = log1pf(expf(normal(k++) - 2.0f));
    for (long e = 0; e < D * N; ++e) s->A[e] = -expf((float)(unif(k++) * log(16.0)));
    for (long t = 0; t < L; ++t) {
        for (long n = 0; n < N; ++n) {
            const float b = normal(k++), c = normal(k++);
            for (long d = 0; d < D; ++d) {
                s->B[(t * D + d) * N + n] = b;
                s->C[(t * D + d) * N + n] = c;
            }
        }
    }
    memset(s->h, 0, sizeof(float) * (size_t)(L * D * N));
    memset(s->y, 0, sizeof(float) * (size_t)(L * D));
    memset(s->dx, 0, sizeof(float) * (size_t)(L * D));
    memset(s->ddt, 0, sizeof(float) * (size_t)(L * D));
    memset(s->dA, 0, sizeof(float) * (size_t)(D * N));
    memset(s->dB, 0, sizeof(float) * (size_t)(L * D * N));
    memset(s->dC, 0, sizeof(float) * (size_t)(L * D * N));
    memset(s->state, 0, sizeof(float) * (size_t)(D * N));
}

static void run_slice(BenchRun *r, int i) {
    BenchSlice *s = &r->s[i];
    const long L = r->L, D = r->chans, N = r->N;
#ifdef KMB_BENCH_REF
    const long dims[1] = {L};
    BenchNDParams f = {dims, 1, D, N, s->x, s->A, s->B, s->C, s->dt, s->h, s->y, NULL, NULL};
    scannd_ref(&f);
    BenchBwdParams b = {s->x, s->A, s->B, s->C, s->dt, NULL, s->h, s->dy,
                        s->dx, s->dA, s->dB, s->dC, s->ddt, L, D, N};
    scan1d_backward(&b);
#else
    memset(s->state, 0, sizeof(float) * (size_t)(D * N));
    or_scan1d_fwd(s->x, s->dt, s->A, s->B, s->C, s->state, s->y, s->h, L, D, N, D * N, N, 0);
    or_scan1d_bwd(s->x, s->dt, s->A, s->B, s->C, NULL, s->h, s->dy, s->dx, s->ddt, s->dA, s->dB,
                  s->dC, L, D, N, D * N, N);
#endif
}

static void free_run(BenchRun *r) {
    if (!r) return;
    if (r->s) {
        for (int i = 0; i < r->slices; ++i) {
            BenchSlice *s = &r->s[i];
            float *all[] = {s->x, s->dt, s->A, s->B, s->C, s->dy, s->h, s->y,
                            s->dx, s->ddt, s->dA, s->dB, s->dC, s->state};
            for (size_t j = 0; j < sizeof all / sizeof *all; ++j) free(all[j]);
        }
        free(r->s);
    }
    free(r);
}

/* Builds `slices` slices of `chans` channels (L steps, N states), filled
 * by `threads` OpenMP workers.  NULL on allocation failure. */
void *kmb_cpu_bench_create(int slices, int chans, long L, int N, unsigned long long seed,
                           int threads) {
    if (slices < 1 || chans < 1 || L < 1 || N < 1 || threads < 1) return NULL;
    BenchRun *r = (BenchRun *)calloc(1, sizeof *r);
    if (!r) return NULL;
    r->slices = slices;
    r->chans = chans;
    r->L = L;
    r->N = N;
    r->threads = threads;
    r->s = (BenchSlice *)calloc((size_t)slices, sizeof *r->s);
    if (!r->s) {
        free_run(r);
        return NULL;
    }
    const size_t ld = sizeof(float) * (size_t)(L * chans);
    const size_t ldn = ld * (size_t)N, dn = sizeof(float) * (size_t)(chans * N);
    int ok = 1;
    for (int i = 0; i < slices && ok; ++i) {
        BenchSlice *s = &r->s[i];
        s->x = malloc(ld); s->dt = malloc(ld); s->dy = malloc(ld); s->y = malloc(ld);
        s->dx = malloc(ld); s->ddt = malloc(ld);
        s->B = malloc(ldn); s->C = malloc(ldn); s->h = malloc(ldn);
        s->dB = malloc(ldn); s->dC = malloc(ldn);
        s->A = malloc(dn); s->dA = malloc(dn); s->state = malloc(dn);
        ok = s->x && s->dt && s->dy && s->y && s->dx && s->ddt && s->B && s->C && s->h &&
             s->dB && s->dC && s->A && s->dA && s->state;
    }
    if (!ok) {
        free_run(r);
        return NULL;
    }
    omp_set_max_active_levels(1);
#pragma omp parallel for schedule(static, 1) num_threads(threads)
    for (int i = 0; i < slices; ++i) fill_slice(r, i, seed);
    return r;
}

/* One pass over every slice (forward + backward); wall seconds. */
double kmb_cpu_bench_pass(void *h) {
    BenchRun *r = (BenchRun *)h;
    if (!r) return -1.0;
    omp_set_max_active_levels(1);
    const double t0 = omp_get_wtime();
#pragma omp parallel for schedule(static, 1) num_threads(r->threads)
    for (int i = 0; i < r->slices; ++i) run_slice(r, i);
    return omp_get_wtime() - t0;
}

/* A checksum of the last pass's outputs (keeps the work observable). */
double kmb_cpu_bench_checksum(void *h) {
    BenchRun *r = (BenchRun *)h;
    double acc = 0.0;
    if (!r) return 0.0;
    for (int i = 0; i < r->slices; ++i) {
        const BenchSlice *s = &r->s[i];
        for (long e = 0; e < r->L * r->chans; e += 97) acc += (double)s->y[e] + s->dx[e];
        for (long e = 0; e < (long)r->chans * r->N; ++e) acc += s->dA[e];
    }
    return acc;
}

void kmb_cpu_bench_free(void *h) { free_run((BenchRun *)h); }
