#ifndef KMAMBA_SCAN_H
#define KMAMBA_SCAN_H

#include <stddef.h>

/*
 * Selective scans, reference-compatible C API (k-mamba include/scan.h).
 *
 * Every function below runs on the GPU.  Pointers may be host or device
 * memory: host buffers are staged through device memory inside the call,
 * device buffers are used in place.  Calls are synchronous (they return
 * after the result is in the caller's buffers), like the reference.
 *
 * 1D recurrence, per channel d and state m:
 *   h_t[d,m] = exp(delta_t[d] * A[d,m]) * h_{t-1}[d,m] + delta_t[d]*B_t[d,m]*x_t[d]
 *   y_t[d]   = sum_m C_t[d,m] * h_t[d,m]
 */

#ifdef __cplusplus
extern "C" {
#endif

/* scan1d: x, delta, y [L,D]; A [D,M]; B, C [L,D,M]; h [D,M] is the running
 * state, read as the initial state and overwritten with the final one.
 * States are clamped to [-1000, 1000] after every step (reference
 * cpu/scan1d.asm:136-140). */
typedef struct {
    float *x;
    float *A;
    float *B;
    float *C;
    float *delta;
    float *h;
    float *y;
    long   L;
    long   D;
    long   M;
} ScanParams;

void scan1d(ScanParams *p);

/* scan1d_backward: h [L,D,M] are the forward states, h0 [D,M] (or NULL =
 * zero) the state before t = 0.  dx, ddelta [L,D]; dA [D,M]; dB, dC
 * [L,D,M]; all outputs are overwritten (reference cpu/scan1d_backward.c). */
typedef struct {
    float *x;
    float *A;
    float *B;
    float *C;
    float *delta;
    float *h0;
    float *h;
    float *dy;
    float *dx;
    float *dA;
    float *dB;
    float *dC;
    float *ddelta;
    long   L;
    long   D;
    long   M;
} ScanBackwardParams;

void scan1d_backward(ScanBackwardParams *p);

/* M = 1 backward with per-channel A, B, C [D] and a per-step delta [L]
 * shared by all channels; A_diag [L,D] optionally holds exp(delta*A).
 * dA, dB, dC [D]; dx [L,D]; ddelta [L]. */
typedef struct {
    float *x;
    float *A;
    float *A_diag;
    float *B;
    float *C;
    float *delta;
    float *h0;
    float *h;
    float *dy;
    float *dx;
    float *dA;
    float *dB;
    float *dC;
    float *ddelta;
    long   L;
    long   D;
} ScanBackwardSharedParams;

void scan1d_backward_m1_shared_bc(ScanBackwardSharedParams *p);
void scan1d_backward_m1_shared_bc_asm(ScanBackwardSharedParams *p);
void scan1d_backward_m1_shared_bc_simple_asm(ScanBackwardSharedParams *p);

/* scan2d: anti-diagonal wavefront over a d1 x d2 grid.
 *   h(i,j) = dA1*h(i-1,j) + dA2*h(i,j-1) + B*((delta1+delta2)/2)*x
 * x, delta1, delta2, y [d1*d2, D]; A1, A2 [D,M]; B, C, h [d1*d2, D, M]. */
typedef struct {
    float *x;
    float *A1;
    float *A2;
    float *B;
    float *C;
    float *delta1;
    float *delta2;
    float *h;
    float *y;
    long   d1;
    long   d2;
    long   D;
    long   M;
} Scan2DParams;

void scan2d(Scan2DParams *p);

/* Device-pointer 1D scan (reference cuda/scan1d.cu:258).  h is the full
 * [L,D,M] state history starting from zero; states are clamped to
 * [-1000, 1000]. */
void om_scan1d_forward(const float *d_x, const float *d_A,
                       const float *d_B, const float *d_C,
                       const float *d_dt,
                       float *d_y, float *d_h,
                       int L, int D, int M);

/* Device-pointer 1D backward (reference cuda/scan1d_backward.cu:113). */
void om_scan1d_backward(const float *d_dy,
                        const float *d_x, const float *d_A,
                        const float *d_B, const float *d_C,
                        const float *d_dt, const float *d_h,
                        float *d_dx, float *d_dA,
                        float *d_dB, float *d_dC, float *d_ddt,
                        int L, int D, int M);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_SCAN_H */
