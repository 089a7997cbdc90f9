/*
 * Bounded causal wavefront over an N-dimensional grid (host, integer).
 *
 * Contract of the reference src/wavefront_nd.c (k-mamba): level = sum of
 * coordinates, points of a level visited in lexicographic order (which is
 * ascending row-major order), -1 for invalid input or overflow, the
 * callback's non-zero return value stops the walk and is returned as is.
 *
 * Level sizes are the coefficients of prod_axis (1 + z + ... + z^(dims-1)),
 * built axis by axis with a sliding-window sum; the walk of one level is an
 * odometer over the leading axes whose bounds come from how much of the
 * level the trailing axes can still absorb.
 */
#include <limits.h>
#include <stdlib.h>

#include "wavefront_nd.h"

static int add_ok(long a, long b, long *out) {
    if ((b > 0 && a > LONG_MAX - b) || (b < 0 && a < LONG_MIN - b)) return 0;
    *out = a + b;
    return 1;
}

static int mul_ok(long a, long b, long *out) {
    if (a < 0 || b < 0) return 0;
    if (a != 0 && b > LONG_MAX / a) return 0;
    *out = a * b;
    return 1;
}

int wavefront_nd_validate_dims(const long *dims, long ndims) {
    if (!dims || ndims <= 0) return 0;
    for (long i = 0; i < ndims; ++i)
        if (dims[i] <= 0) return 0;
    return 1;
}

long wavefront_nd_total_points(const long *dims, long ndims) {
    long t = 1;
    if (!wavefront_nd_validate_dims(dims, ndims)) return -1;
    for (long i = 0; i < ndims; ++i)
        if (!mul_ok(t, dims[i], &t)) return -1;
    return t;
}

long wavefront_nd_max_level(const long *dims, long ndims) {
    long m = 0;
    if (!wavefront_nd_validate_dims(dims, ndims)) return -1;
    for (long i = 0; i < ndims; ++i)
        if (!add_ok(m, dims[i] - 1, &m)) return -1;
    return m;
}

long wavefront_nd_row_major_offset(const long *dims, const long *idx, long ndims) {
    long off = 0;
    if (!wavefront_nd_validate_dims(dims, ndims) || !idx) return -1;
    for (long i = 0; i < ndims; ++i) {
        if (idx[i] < 0 || idx[i] >= dims[i]) return -1;
        if (!mul_ok(off, dims[i], &off) || !add_ok(off, idx[i], &off)) return -1;
    }
    return off;
}

long wavefront_nd_level_size(const long *dims, long ndims, long level) {
    long maxl, *cnt, *nxt, res;
    if (!wavefront_nd_validate_dims(dims, ndims)) return -1;
    maxl = wavefront_nd_max_level(dims, ndims);
    if (maxl < 0 || level < 0 || level > maxl) return -1;
    cnt = (long *)calloc((size_t)level + 1, sizeof(long));
    nxt = (long *)calloc((size_t)level + 1, sizeof(long));
    if (!cnt || !nxt) {
        free(cnt);
        free(nxt);
        return -1;
    }
    cnt[0] = 1; /* empty product: one way to reach level 0 */
    res = 0;
    for (long ax = 0; ax < ndims && res >= 0; ++ax) {
        /* nxt[l] = sum_{v=0}^{dims-1} cnt[l - v]  (window sum) */
        long win = 0;
        for (long l = 0; l <= level; ++l) {
            if (!add_ok(win, cnt[l], &win)) { res = -1; break; }
            if (l - dims[ax] >= 0) win -= cnt[l - dims[ax]];
            nxt[l] = win;
        }
        { long *t = cnt; cnt = nxt; nxt = t; }
    }
    if (res >= 0) res = cnt[level];
    free(cnt);
    free(nxt);
    return res;
}

/* Walks one level.  cap[ax] = sum_{k > ax} (dims[k] - 1): the most the
 * axes after `ax` can absorb. */
static int walk_level(const long *dims, long ndims, long level, long *idx,
                      const long *cap, WavefrontNDVisitFn visit, void *user) {
    long ordinal = 0;
    long ax;
    long rem; /* level left for axes >= ax */

    /* first point: each leading axis takes the smallest admissible value */
    rem = level;
    for (ax = 0; ax < ndims - 1; ++ax) {
        long lo = rem - cap[ax];
        idx[ax] = lo > 0 ? lo : 0;
        rem -= idx[ax];
    }
    for (;;) {
        int rc;
        idx[ndims - 1] = rem;
        rc = visit(idx, ndims, level, ordinal++, user);
        if (rc != 0) return rc;
        /* advance: find the last leading axis that can still grow */
        for (ax = ndims - 2; ax >= 0; --ax) {
            long hi;
            rem += idx[ax]; /* give this axis' share back */
            hi = dims[ax] - 1 < rem ? dims[ax] - 1 : rem;
            if (idx[ax] < hi) {
                idx[ax] += 1;
                rem -= idx[ax];
                break;
            }
        }
        if (ax < 0) return 0;
        /* reset the axes after `ax` to their smallest admissible values */
        for (long k = ax + 1; k < ndims - 1; ++k) {
            long lo = rem - cap[k];
            idx[k] = lo > 0 ? lo : 0;
            rem -= idx[k];
        }
    }
}

static long *make_caps(const long *dims, long ndims) {
    long *cap = (long *)malloc((size_t)ndims * sizeof(long));
    long s = 0;
    if (!cap) return NULL;
    for (long ax = ndims - 1; ax >= 0; --ax) {
        cap[ax] = s;
        if (!add_ok(s, dims[ax] - 1, &s)) {
            free(cap);
            return NULL;
        }
    }
    return cap;
}

int wavefront_nd_for_level(const long *dims, long ndims, long level, long *idx_scratch,
                           WavefrontNDVisitFn visit, void *user) {
    long maxl, *idx, *cap;
    int rc;
    if (!wavefront_nd_validate_dims(dims, ndims) || !visit) return -1;
    maxl = wavefront_nd_max_level(dims, ndims);
    if (maxl < 0 || level < 0 || level > maxl) return -1;
    cap = make_caps(dims, ndims);
    if (!cap) return -1;
    idx = idx_scratch ? idx_scratch : (long *)malloc((size_t)ndims * sizeof(long));
    if (!idx) {
        free(cap);
        return -1;
    }
    rc = walk_level(dims, ndims, level, idx, cap, visit, user);
    if (!idx_scratch) free(idx);
    free(cap);
    return rc;
}

int wavefront_nd_for_each_level(const long *dims, long ndims, long *idx_scratch,
                                WavefrontNDVisitFn visit, void *user) {
    long maxl, *idx, *cap;
    int rc = 0;
    if (!wavefront_nd_validate_dims(dims, ndims) || !visit) return -1;
    maxl = wavefront_nd_max_level(dims, ndims);
    if (maxl < 0) return -1;
    cap = make_caps(dims, ndims);
    if (!cap) return -1;
    idx = idx_scratch ? idx_scratch : (long *)malloc((size_t)ndims * sizeof(long));
    if (!idx) {
        free(cap);
        return -1;
    }
    for (long l = 0; l <= maxl && rc == 0; ++l)
        rc = walk_level(dims, ndims, l, idx, cap, visit, user);
    if (!idx_scratch) free(idx);
    free(cap);
    return rc;
}
