/*
 * Row-major index helpers of km_topology.h.
 *
 * Contract (reference include/km_topology.h, behaviour of
 * src/km_topology.c:8-110, pinned by tests/test_topology.py):
 *  - a shape is valid when 1 <= ndims <= KMAMBA_MAX_NDIMS and every extent
 *    passes wavefront_nd_validate_dims;
 *  - the last axis is the fastest (stride 1);
 *  - unravel uses the caller's strides: coords[axis] = (linear / stride) mod dim;
 *  - ravel returns -1 for any coordinate outside [0, dim);
 *  - km_power_long(b, e) is b^e for e >= 0, 0 for e < 0 and for 0^0;
 *  - km_normalize_spatial_topology turns "no spatial dims" into the 1D
 *    shape [seq_len] and then requires prod(dims) == seq_len.
 */
#include <limits.h>
#include <string.h>

#include "km_topology.h"
#include "wavefront_nd.h"

/* Rank in range and every extent accepted by the wavefront generator. */
static int shape_ok(const long *dims, long ndims) {
    return dims && ndims >= 1 && ndims <= KMAMBA_MAX_NDIMS &&
           wavefront_nd_validate_dims(dims, ndims);
}

int km_spatial_dims_product(const long *dims, long ndims, size_t *product_out) {
    if (!product_out || !shape_ok(dims, ndims)) return 0;
    size_t total = 1;
    for (const long *e = dims; e != dims + ndims; ++e)
        if (__builtin_mul_overflow(total, (size_t)*e, &total)) return 0;
    *product_out = total;
    return 1;
}

int km_make_row_major_strides(const long *dims, long ndims, long *strides_out) {
    if (!strides_out || !shape_ok(dims, ndims)) return 0;
    /* running product of the extents to the right of each axis */
    long right = 1;
    long ax = ndims;
    while (ax-- > 0) {
        strides_out[ax] = right;
        right *= dims[ax];
    }
    return 1;
}

void km_unravel_index(long linear, const long *dims, const long *strides, long ndims,
                      long *coords_out) {
    if (linear < 0 || !strides || !coords_out || !dims || ndims < 1 ||
        ndims > KMAMBA_MAX_NDIMS)
        return;
    for (long ax = ndims - 1; ax >= 0; --ax) coords_out[ax] = linear / strides[ax] % dims[ax];
}

long km_ravel_index(const long *coords, const long *dims, const long *strides, long ndims) {
    if (!coords || !dims || !strides || ndims < 1 || ndims > KMAMBA_MAX_NDIMS) return -1;
    long offset = 0;
    for (long ax = ndims - 1; ax >= 0; --ax) {
        const long c = coords[ax];
        if (c < 0 || c >= dims[ax]) return -1;
        offset += c * strides[ax];
    }
    return offset;
}

long km_power_long(long base, long exp) {
    if (exp < 0 || (exp == 0 && base == 0)) return 0;
    /* square-and-multiply, wrapping modulo 2^64 like repeated long products */
    unsigned long acc = 1, sq = (unsigned long)base;
    for (unsigned long e = (unsigned long)exp; e; e >>= 1) {
        if (e & 1ul) acc *= sq;
        sq *= sq;
    }
    return (long)acc;
}

int km_normalize_spatial_topology(long *spatial_ndims, long *spatial_dims, size_t seq_len,
                                  int use_convnd, long *convnd_ndims, long convnd_K) {
    if (!spatial_ndims || !spatial_dims || seq_len > (size_t)LONG_MAX) return -1;
    const int implicit_1d = *spatial_ndims <= 0;
    if (implicit_1d) {
        memset(spatial_dims, 0, sizeof(long) * KMAMBA_MAX_NDIMS);
        spatial_dims[0] = (long)seq_len;
        *spatial_ndims = 1;
    }
    size_t points = 0;
    if (!km_spatial_dims_product(spatial_dims, *spatial_ndims, &points) || points != seq_len)
        return -1;
    if (!use_convnd) return 0;
    if (!convnd_ndims || convnd_K < 1) return -1;
    if (*convnd_ndims < 1) *convnd_ndims = *spatial_ndims;
    return *convnd_ndims == *spatial_ndims ? 0 : -1;
}
