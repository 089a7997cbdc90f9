#ifndef KMAMBA_TOPOLOGY_H
#define KMAMBA_TOPOLOGY_H

#include <stddef.h>

/*
 * Row-major index helpers shared by the ND scan and ConvND entry points.
 * Same names and contracts as the reference include/km_topology.h:1-60.
 */

#ifdef __cplusplus
extern "C" {
#endif

#define KMAMBA_MAX_NDIMS 8

/* 1 and *product_out = prod(dims) on success, 0 on invalid input/overflow. */
int km_spatial_dims_product(const long *dims, long ndims, size_t *product_out);

/* strides[axis] = prod(dims[axis+1 .. ndims-1]); 1 on success, 0 otherwise. */
int km_make_row_major_strides(const long *dims, long ndims, long *strides_out);

/* coords[axis] = (linear / strides[axis]) % dims[axis]; no-op on bad input. */
void km_unravel_index(long linear, const long *dims, const long *strides,
                      long ndims, long *coords_out);

/* Sum of coords[axis] * strides[axis], -1 when a coordinate is out of range. */
long km_ravel_index(const long *coords, const long *dims, const long *strides,
                    long ndims);

/* base^exp for exp >= 0; 0 when exp < 0 or base == exp == 0. */
long km_power_long(long base, long exp);

/* Fills the implicit 1D topology [seq_len] when *spatial_ndims <= 0, checks
 * that prod(spatial_dims) == seq_len and the ConvND rank.  0 / -1. */
int km_normalize_spatial_topology(long *spatial_ndims, long *spatial_dims,
                                  size_t seq_len, int use_convnd,
                                  long *convnd_ndims, long convnd_K);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_TOPOLOGY_H */
