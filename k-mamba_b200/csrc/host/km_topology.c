/*
 * Row-major index helpers (contract of the reference src/km_topology.c).
 */
#include <limits.h>
#include <string.h>

#include "km_topology.h"
#include "wavefront_nd.h"

int km_spatial_dims_product(const long *dims, long ndims, size_t *product_out) {
    size_t prod = 1;
    if (!dims || !product_out || ndims <= 0 || ndims > KMAMBA_MAX_NDIMS) return 0;
    if (!wavefront_nd_validate_dims(dims, ndims)) return 0;
    for (long i = 0; i < ndims; ++i) {
        size_t e = (size_t)dims[i];
        if (prod > (size_t)-1 / e) return 0;
        prod *= e;
    }
    *product_out = prod;
    return 1;
}

int km_make_row_major_strides(const long *dims, long ndims, long *strides_out) {
    long s = 1;
    if (!dims || !strides_out || ndims <= 0 || ndims > KMAMBA_MAX_NDIMS) return 0;
    if (!wavefront_nd_validate_dims(dims, ndims)) return 0;
    for (long ax = ndims - 1; ax >= 0; --ax) {
        strides_out[ax] = s;
        s *= dims[ax];
    }
    return 1;
}

void km_unravel_index(long linear, const long *dims, const long *strides, long ndims,
                      long *coords_out) {
    if (!dims || !strides || !coords_out || ndims <= 0 || ndims > KMAMBA_MAX_NDIMS) return;
    if (linear < 0) return;
    for (long ax = 0; ax < ndims; ++ax) coords_out[ax] = (linear / strides[ax]) % dims[ax];
}

long km_ravel_index(const long *coords, const long *dims, const long *strides, long ndims) {
    long off = 0;
    if (!coords || !dims || !strides || ndims <= 0 || ndims > KMAMBA_MAX_NDIMS) return -1;
    for (long ax = 0; ax < ndims; ++ax) {
        if (coords[ax] < 0 || coords[ax] >= dims[ax]) return -1;
        off += coords[ax] * strides[ax];
    }
    return off;
}

long km_power_long(long base, long exp) {
    long r = 1;
    if (exp < 0) return 0;
    if (base == 0 && exp == 0) return 0;
    while (exp-- > 0) r *= base;
    return r;
}

int km_normalize_spatial_topology(long *spatial_ndims, long *spatial_dims, size_t seq_len,
                                  int use_convnd, long *convnd_ndims, long convnd_K) {
    size_t total;
    if (!spatial_ndims || !spatial_dims) return -1;
    if (seq_len > (size_t)LONG_MAX) return -1;
    if (*spatial_ndims <= 0) {
        memset(spatial_dims, 0, (size_t)KMAMBA_MAX_NDIMS * sizeof(long));
        *spatial_ndims = 1;
        spatial_dims[0] = (long)seq_len;
    }
    if (!km_spatial_dims_product(spatial_dims, *spatial_ndims, &total)) return -1;
    if (total != seq_len) return -1;
    if (use_convnd) {
        if (!convnd_ndims || convnd_K <= 0) return -1;
        if (*convnd_ndims <= 0) *convnd_ndims = *spatial_ndims;
        if (*convnd_ndims != *spatial_ndims) return -1;
    }
    return 0;
}
