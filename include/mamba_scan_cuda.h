#ifndef MAMBA_SCAN_CUDA_H
#define MAMBA_SCAN_CUDA_H

#include <stddef.h>
#include "scan_nd.h"

/* Device-pointer wrappers of the reference include/mamba_scan_cuda.h:13-35. */

#ifdef __cplusplus
extern "C" {
#endif

void mamba_scan1d_cuda_forward(const float *d_x, const float *d_A,
                               const float *d_B, const float *d_C,
                               const float *d_dt, float *d_y, float *d_h,
                               int L, int D, int M);

void mamba_scan1d_cuda_backward(const float *d_dy, const float *d_x,
                                const float *d_A, const float *d_B,
                                const float *d_C, const float *d_dt,
                                const float *d_h, float *d_dx, float *d_dA,
                                float *d_dB, float *d_dC, float *d_ddt,
                                int L, int D, int M);

int mamba_scannd_cuda_forward(ScanNDParams *p);

#ifdef __cplusplus
}
#endif

#endif
