#ifndef KMAMBA_WAVEFRONT_PLAN_H
#define KMAMBA_WAVEFRONT_PLAN_H

#include "wavefront_nd.h"

/*
 * Reusable wavefront schedule of an N-dimensional grid.
 *
 * level_offsets holds every row-major offset of the grid grouped by level,
 * ascending inside each level; level_starts[l] is the index of the first
 * offset of level l and level_starts[max_level + 1] == total_points.
 *
 * The struct layout and the function contracts are those of the reference
 * include/wavefront_plan.h:27-52 (k-mamba), so plans can be passed across
 * the two libraries.  The plan is host memory owned by its creator.
 */

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    long *dims;          /* [ndims] */
    long ndims;
    long total_points;
    long max_level;
    long max_level_size;
    long *level_starts;  /* [max_level + 2] */
    long *level_offsets; /* [total_points] */
} KMWavefrontPlan;

/* NULL on invalid dims or allocation failure. */
KMWavefrontPlan *km_wavefront_plan_create(const long *dims, long ndims);
void km_wavefront_plan_free(KMWavefrontPlan *plan);
/* 1 when the plan was built for exactly these dims. */
int km_wavefront_plan_matches_dims(const KMWavefrontPlan *plan,
                                   const long *dims, long ndims);
/* -1 when level is out of range. */
long km_wavefront_plan_level_size(const KMWavefrontPlan *plan, long level);
/* NULL when level is out of range. */
const long *km_wavefront_plan_level_offsets(const KMWavefrontPlan *plan,
                                            long level);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_WAVEFRONT_PLAN_H */
