#ifndef KMAMBA_WAVEFRONT_ND_H
#define KMAMBA_WAVEFRONT_ND_H

/*
 * Bounded causal wavefront over an N-dimensional grid (host, integer only).
 *
 * The level of a point is the sum of its coordinates.  Points of one level
 * only depend on points of lower levels, so a level is a set of independent
 * work items.  Inside a level the points are visited in lexicographic order
 * of their coordinates, which is ascending row-major offset order.
 *
 * Drop-in for the reference interface include/wavefront_nd.h:1-83 of
 * k-mamba (same names, argument meaning and return conventions).
 */

#ifdef __cplusplus
extern "C" {
#endif

typedef int (*WavefrontNDVisitFn)(const long *idx, long ndims, long level,
                                  long ordinal_in_level, void *user);

/* 1 when ndims > 0 and every dims[i] > 0, else 0. */
int wavefront_nd_validate_dims(const long *dims, long ndims);

/* Product of dims, -1 on invalid input or overflow. */
long wavefront_nd_total_points(const long *dims, long ndims);

/* Sum of (dims[i] - 1), -1 on invalid input or overflow. */
long wavefront_nd_max_level(const long *dims, long ndims);

/* Row-major offset of idx, -1 when idx is out of range or on overflow. */
long wavefront_nd_row_major_offset(const long *dims, const long *idx, long ndims);

/* Number of points whose coordinates sum to `level`, -1 if invalid. */
long wavefront_nd_level_size(const long *dims, long ndims, long level);

/* Visit one level in lexicographic order.  idx_scratch may be NULL.
 * Returns 0 when the whole level was visited, the callback's non-zero code
 * when it asked to stop, -1 on invalid arguments. */
int wavefront_nd_for_level(const long *dims, long ndims, long level,
                           long *idx_scratch, WavefrontNDVisitFn visit,
                           void *user);

/* Visit levels 0..max_level in order; same return convention. */
int wavefront_nd_for_each_level(const long *dims, long ndims,
                                long *idx_scratch, WavefrontNDVisitFn visit,
                                void *user);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_WAVEFRONT_ND_H */
