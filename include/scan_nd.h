#ifndef KMAMBA_SCAN_ND_H
#define KMAMBA_SCAN_ND_H

#include "wavefront_plan.h"

/*
 * ND selective scan over a causal grid (reference include/scan_nd.h).
 *
 *   dt_bar(p,d) = mean over axes of delta(axis,p,d)
 *   h(p,d,m)    = dt_bar * B(p,d,m) * x(p,d)
 *               + sum_axis exp(delta(axis,p,d) * A(axis,d,m)) * h(p - e_axis,d,m)
 *   y(p,d)      = sum_m C(p,d,m) * h(p,d,m)
 *
 * Layout: x, y [P,D]; A [ndims,D,M]; B, C, h [P,D,M]; delta [ndims,P,D];
 * P = prod(dims).  dims is always a host pointer; the tensors may be host
 * or device memory.  All levels of the wavefront run inside one persistent
 * kernel on the GPU.  The Mamba-3 fields theta / lambda are accepted and
 * must be NULL (the GPU path implements the plain recurrence; a non-NULL
 * value is rejected with -1).
 */

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const long  *dims;
    long         ndims;
    long         D;
    long         M;
    const float *x;
    const float *A;
    const float *B;
    const float *C;
    const float *delta;
    float       *h;
    float       *y;
    const float *theta;
    const float *lambda;
} ScanNDParams;

/* 1 when the pointers and sizes are usable, else 0. */
int scannd_validate(const ScanNDParams *p);
/* 0 on success, -1 on invalid input or device failure. */
int scannd_ref(ScanNDParams *p);
int scannd_ref_with_plan(ScanNDParams *p, const KMWavefrontPlan *plan);
int scannd(ScanNDParams *p);
/* Device-pointer variant (reference cuda/scan_nd.cu:337). */
int om_scannd_forward(ScanNDParams *p);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_SCAN_ND_H */
