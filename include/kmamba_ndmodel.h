#ifndef KMAMBA_NDMODEL_H
#define KMAMBA_NDMODEL_H

/*
 * Mamba-ND model over 3D volumes of byte tokens.
 *
 * No counterpart in the reference: kmamba_create with use_convnd overruns
 * its heap there (src/mamba_block.c:223-234) and its training step holds
 * every layer's activations (src/kmamba.c:387).  This model stacks ND
 * blocks built from the reference's operators -- the causal ConvND
 * (src/convnd.c) and the ND wavefront scan (src/scan_nd.c) -- as follows,
 * per layer (d = dim, 16 states, K = 3, 3 axes, T = batch * points):
 *
 *   a = x W_a^T, z = x W_z^T                    bf16 tensor-core GEMMs
 *   c = silu(ConvND(a) + conv_bias)
 *   q = c W_p^T                                 [T, 35], bf16 GEMM
 *   delta_k = ln 3 + softplus(q[:, k] + dt_bias[k]),  B = q[:, 3:19],
 *   C = q[:, 19:35],  A = -1 - exp(A_log)       (every decay <= 1/3)
 *   y = ScanND(c, delta, A, B, C)               channel-shared B / C
 *   x <- x + (y * silu(z)) W_out^T              residual fused in the GEMM
 *
 * then logits = x H^T and the mean cross entropy of logits[i] against the
 * next token in raster order, tok[(i + 1) mod points], per volume.
 * Embedding E gathers fp32 rows.  Weights are fp32 masters; the GEMMs take
 * bf16 copies of their operands (round to nearest even) and accumulate in
 * fp32; everything else is fp32.  The backward recomputes each layer's
 * activations from its stored input (one layer's activations live at a
 * time).  A batch larger than the micro-batch runs as consecutive passes
 * of micro_batch volumes whose gradients accumulate (each pass's loss
 * weighted by its share of the batch), so the step's gradient is that of
 * the whole batch's mean loss.  The optimizer is AdamW over all
 * parameters.
 *
 * Flat parameter layout (fp32, kmb_ndmodel_params), in order:
 *   embedding [vocab, d], head [vocab, d], then per layer
 *   W_a [d, d], W_z [d, d], W_out [d, d], W_p [35, d], dt_bias [3, d],
 *   A_log [3, d, 16], conv_kernel [27, d], conv_bias [d].
 * Gradients (kmb_ndmodel_grads) use the same layout.
 */

#include <stddef.h>

#include "kmamba_distributed.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    long dims[3];            /* volume; points = dims[0] dims[1] dims[2] */
    long dim;                /* d: a multiple of 32 */
    long n_layers;
    long vocab;              /* token ids < vocab (256 for byte tokens) */
    unsigned long long seed; /* initialisation */
    long micro_batch;        /* volumes per pass (0: as many as fit in free memory) */
} KmbNDModelConfig;

typedef struct KmbNDModel KmbNDModel;

/* NULL on invalid configuration or allocation failure (kmb_last_error). */
KmbNDModel *kmb_ndmodel_create(const KmbNDModelConfig *cfg);
void kmb_ndmodel_free(KmbNDModel *m);

long kmb_ndmodel_param_count(const KmbNDModel *m);
/* Device pointers to the flat fp32 parameters and gradients. */
float *kmb_ndmodel_params(KmbNDModel *m);
float *kmb_ndmodel_grads(KmbNDModel *m);
/* Refreshes the bf16 copies of the GEMM weights after the caller wrote
 * kmb_ndmodel_params directly. */
int kmb_ndmodel_sync_weights(KmbNDModel *m);

/* Data parallelism: gradients are averaged over the context's ranks
 * (bucketed per layer, overlapped with the backward of the layers below)
 * before the optimizer step.  NULL detaches. */
int kmb_ndmodel_set_dist(KmbNDModel *m, KMambaDistributedContext *ctx);

/* tokens: uint32 [batch, points], device or host memory.  loss (host) is
 * the mean cross entropy of this rank's batch. */
int kmb_ndmodel_forward(KmbNDModel *m, const unsigned *tokens, long batch, float *loss);
/* forward + backward: the gradients land in kmb_ndmodel_grads (averaged
 * over ranks when a context is attached). */
int kmb_ndmodel_backward(KmbNDModel *m, const unsigned *tokens, long batch, float *loss);
/* AdamW (beta 0.9 / 0.999, eps 1e-8) on every parameter, then the bf16
 * weight copies are refreshed. */
int kmb_ndmodel_step(KmbNDModel *m, float lr, float weight_decay);
int kmb_ndmodel_train_step(KmbNDModel *m, const unsigned *tokens, long batch, float lr,
                           float weight_decay, float *loss);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_NDMODEL_H */
