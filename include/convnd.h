#ifndef CONVND_H
#define CONVND_H

#include <stddef.h>
#include "wavefront_plan.h"

/*
 * Causal depthwise ND convolution with a dense K^ndims kernel
 * (reference include/convnd.h and src/convnd.c).
 *
 *   output(p,d) = bias[d] + sum_k input(p - (K-1-k_axis)_axis, d) * kernel[k,d]
 *
 * k is the row-major index over the K^ndims kernel offsets (last axis
 * fastest); inputs outside the grid count as zero.  input / output / dy /
 * dinput are [prod(dims), D]; kernel, dkernel [K^ndims, D]; bias, dbias [D].
 * Tensors may be host or device memory; dims is a host pointer.
 */

typedef struct {
    float *input;
    const float *kernel;
    const float *bias;
    float *output;
    float *dy;
    float *dinput;
    float *dkernel;
    float *dbias;
    const long *dims;
    long ndims;
    long D;
    long K;
} ConvNDParams;

typedef enum {
    CONVND_FORWARD = 1,
    CONVND_BACKWARD = 2,
    CONVND_COMPLETE = 3
} ConvNDMode;

#ifdef __cplusplus
extern "C" {
#endif

long convnd_kernel_volume(long ndims, long K);
void convnd_forward_wavefront(ConvNDParams *p, const KMWavefrontPlan *plan);
void convnd_backward_wavefront(ConvNDParams *p, const KMWavefrontPlan *plan);
void convnd(ConvNDParams *p, ConvNDMode mode);
/* Device-pointer variants, 0 on success and -1 on error
 * (reference cuda/convnd.cu:258,332). */
int om_convnd_forward(ConvNDParams *p);
int om_convnd_backward(ConvNDParams *p);

#ifdef __cplusplus
}
#endif

#endif
