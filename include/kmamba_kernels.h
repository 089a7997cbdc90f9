#ifndef KMAMBA_KERNELS_H
#define KMAMBA_KERNELS_H

/*
 * Optimizer configuration shared by the block and model API (reference
 * include/kmamba_kernels.h:78-85).  The reference header also declares its
 * CPU GEMM / activation / optimizer kernels; those are not part of this
 * library (every computation runs on the GPU behind kmamba.h).
 */

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float lr;
    float mu;
    float beta2;
    float eps;
    float clip_norm;
    float weight_decay;
} MBOptimConfig;

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_KERNELS_H */
