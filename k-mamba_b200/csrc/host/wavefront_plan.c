/*
 * KMWavefrontPlan construction (contract of the reference
 * src/wavefront_plan.c:35-131, k-mamba).
 *
 * Built in two passes over the row-major offsets: a histogram of the
 * levels (coordinate sums), then a stable scatter of every offset into its
 * level's slot.  Offsets are visited in ascending order, so each level's
 * list comes out ascending, which is the lexicographic order of the
 * reference's enumeration.
 */
#include <limits.h>
#include <stdlib.h>
#include <string.h>

#include "wavefront_plan.h"

void km_wavefront_plan_free(KMWavefrontPlan *plan) {
    if (!plan) return;
    free(plan->dims);
    free(plan->level_starts);
    free(plan->level_offsets);
    free(plan);
}

KMWavefrontPlan *km_wavefront_plan_create(const long *dims, long ndims) {
    KMWavefrontPlan *pl;
    long total, maxl, *coord, *cursor;

    if (!wavefront_nd_validate_dims(dims, ndims)) return NULL;
    total = wavefront_nd_total_points(dims, ndims);
    maxl = wavefront_nd_max_level(dims, ndims);
    if (total <= 0 || maxl < 0) return NULL;
    if ((unsigned long)total > (size_t)-1 / sizeof(long)) return NULL;
    if (maxl > LONG_MAX - 2) return NULL;

    pl = (KMWavefrontPlan *)calloc(1, sizeof *pl);
    if (!pl) return NULL;
    pl->dims = (long *)malloc((size_t)ndims * sizeof(long));
    pl->level_starts = (long *)calloc((size_t)maxl + 2, sizeof(long));
    pl->level_offsets = (long *)malloc((size_t)total * sizeof(long));
    coord = (long *)calloc((size_t)ndims, sizeof(long));
    cursor = (long *)malloc(((size_t)maxl + 1) * sizeof(long));
    if (!pl->dims || !pl->level_starts || !pl->level_offsets || !coord || !cursor) {
        free(coord);
        free(cursor);
        km_wavefront_plan_free(pl);
        return NULL;
    }
    memcpy(pl->dims, dims, (size_t)ndims * sizeof(long));
    pl->ndims = ndims;
    pl->total_points = total;
    pl->max_level = maxl;

    /* pass 1: level histogram (level_starts[l + 1] counts level l) */
    {
        long lvl = 0;
        for (long off = 0; off < total; ++off) {
            pl->level_starts[lvl + 1]++;
            /* odometer increment of coord, keeping lvl = sum(coord) */
            for (long ax = ndims - 1; ax >= 0; --ax) {
                if (++coord[ax] < dims[ax]) {
                    ++lvl;
                    break;
                }
                lvl -= dims[ax] - 1;
                coord[ax] = 0;
            }
        }
    }
    pl->max_level_size = 0;
    for (long l = 0; l <= maxl; ++l) {
        if (pl->level_starts[l + 1] > pl->max_level_size)
            pl->max_level_size = pl->level_starts[l + 1];
        pl->level_starts[l + 1] += pl->level_starts[l];
        cursor[l] = pl->level_starts[l];
    }

    /* pass 2: stable scatter */
    memset(coord, 0, (size_t)ndims * sizeof(long));
    {
        long lvl = 0;
        for (long off = 0; off < total; ++off) {
            pl->level_offsets[cursor[lvl]++] = off;
            for (long ax = ndims - 1; ax >= 0; --ax) {
                if (++coord[ax] < dims[ax]) {
                    ++lvl;
                    break;
                }
                lvl -= dims[ax] - 1;
                coord[ax] = 0;
            }
        }
    }
    free(coord);
    free(cursor);
    return pl;
}

int km_wavefront_plan_matches_dims(const KMWavefrontPlan *plan, const long *dims, long ndims) {
    if (!plan || !dims || ndims <= 0 || plan->ndims != ndims) return 0;
    for (long i = 0; i < ndims; ++i)
        if (plan->dims[i] != dims[i]) return 0;
    return 1;
}

long km_wavefront_plan_level_size(const KMWavefrontPlan *plan, long level) {
    if (!plan || level < 0 || level > plan->max_level) return -1;
    return plan->level_starts[level + 1] - plan->level_starts[level];
}

const long *km_wavefront_plan_level_offsets(const KMWavefrontPlan *plan, long level) {
    if (!plan || level < 0 || level > plan->max_level) return NULL;
    return plan->level_offsets + plan->level_starts[level];
}
