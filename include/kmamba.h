#ifndef KMAMBA_H
#define KMAMBA_H

/*
 * k-mamba block and model API (reference include/kmamba.h:20-321), backed
 * by the GPU: block projections, the Mamba-3 scan, the LM head, the
 * softmax cross-entropy and the optimizer all run on the device.
 *
 * The structs keep the reference layout so existing callers compile and
 * link unchanged; the host arrays they point to stay authoritative (they
 * are uploaded before and written back after every GPU call), so callers
 * that read or write weights directly keep working.  Device copies live in
 * a per-object context owned by the library.
 *
 * KMAMBA_BUILD_CUDA must not be defined by callers: the reference's
 * optional in-struct GPU block is not used (device state is internal).
 *
 * Differences from the reference: mamba_backward and friends compute the
 * real gradients of the block (the reference's CPU backward is an empty
 * stub, src/mamba_block.c:834-836), so a training step also updates the
 * blocks and the embedding.  The Rust tokenizer FFI (kmamba_encode, ...)
 * is not part of this library.
 */

#include <stddef.h>
#include <stdint.h>

#include "convnd.h"
#include "km_topology.h"
#include "kmamba_kernels.h"
#include "scan.h"
#include "scan_nd.h"
#include "wavefront_nd.h"
#include "wavefront_plan.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float *data;
    size_t rows;
    size_t cols;
} MBMatrix;

typedef struct {
    size_t dim;
    size_t state_size;
    size_t seq_len;
    size_t mimo_rank;
    float dt_scale;
    float dt_min;
    float dt_max;
    int use_fp16;
    int use_bf16;
    float loss_scale;
    long spatial_ndims;
    long spatial_dims[KMAMBA_MAX_NDIMS];
    int use_convnd;
    long convnd_K;
    long convnd_ndims;
} MBConfig;

typedef enum {
    OPTIMIZER_ADAM_CLIP,
    OPTIMIZER_MUON,
    OPTIMIZER_SGD,
    OPTIMIZER_ADAMW
} OptimizerType;

typedef struct {
    OptimizerType type;
    size_t step;
    float *g_W_in;
    float *g_W_out;
    float *g_A_log;
    float *g_W_B;
    float *g_W_C;
    float *g_b_B;
    float *g_b_C;
    float *g_delta_proj;
    float *g_theta;
    float *g_lambda_proj;
    float *m_W_in;
    float *v_W_in;
    float *m_W_out;
    float *v_W_out;
    float *m_A_log;
    float *v_A_log;
    float *m_W_B;
    float *v_W_B;
    float *m_W_C;
    float *v_W_C;
    float *m_b_B;
    float *v_b_B;
    float *m_b_C;
    float *v_b_C;
    float *m_delta_proj;
    float *v_delta_proj;
    float *m_theta;
    float *v_theta;
    float *m_lambda_proj;
    float *v_lambda_proj;
} MBOptimState;

typedef struct {
    float *hidden;
    float *delta;
    float *scan_B;
    float *scan_C;
    float *scan_delta;
    float *scan_h;
} MambaBlockWorkspace;

typedef struct {
    MBConfig config;
    MBMatrix W_in;        /* [R x dim] */
    MBMatrix W_out;       /* [dim x R] */
    MBMatrix A_log;       /* [state_size], used directly as A */
    MBMatrix W_B;         /* [N*R x dim] */
    MBMatrix W_C;         /* [N*R x dim] */
    MBMatrix delta_proj;  /* [1 x dim] */
    float *b_B;           /* [N*R] */
    float *b_C;           /* [N*R] */
    float *theta;         /* [max(N/2, 1)] */
    MBMatrix lambda_proj; /* [1 x dim] */
    KMWavefrontPlan *wavefront_plan;
    float *convnd_kernel;
    float *convnd_bias;
    float *hidden;
    float *delta;
    float *scan_B;
    float *scan_C;
    float *scan_delta;
    float *scan_h;
    MBOptimState *opt_state;
} MambaBlock;

typedef struct {
    size_t vocab_size;
    size_t dim;
    size_t state_size;
    size_t seq_len;
    size_t n_layers;
    size_t mimo_rank;
    float dt_scale;
    float dt_min;
    float dt_max;
    long spatial_ndims;
    long spatial_dims[KMAMBA_MAX_NDIMS];
    int use_convnd;
    long convnd_K;
    long convnd_ndims;
    int weight_tying;
} KMambaConfig;

typedef struct {
    KMambaConfig cfg;
    float *embedding;     /* [vocab_size, dim] */
    float *head;          /* [dim, vocab_size] */
    MambaBlock **layers;  /* [n_layers] */
    int for_training;
    MBOptimConfig opt_blocks;
    float lr_embed_head;
    float weight_decay;
    float *m_embedding;
    float *v_embedding;
    float *m_head;
    float *v_head;
    size_t step_embed_head;
    float last_grad_norm;
    float last_grad_over_clip;
    int last_grad_would_clip;
} KMamba;

/* ---------------------------------------------------------------- block */
MambaBlock *mamba_block_create(const MBConfig *config);
void mamba_block_free(MambaBlock *block);
void mamba_block_init(MambaBlock *block);
MambaBlockWorkspace *mamba_block_workspace_create(const MambaBlock *block);
void mamba_block_workspace_free(MambaBlockWorkspace *ws);

void mamba_block_forward(MambaBlock *block, float *output, const float *input,
                         size_t batch_size);
void mamba_block_forward_ws(MambaBlock *block, MambaBlockWorkspace *ws, float *output,
                            const float *input, size_t batch_size);

void mamba_attach_optimizer(MambaBlock *block, OptimizerType type, const MBOptimConfig *optconf);
void mamba_free_optimizer(MambaBlock *block);
void mamba_zero_grads(MambaBlock *block);
void mamba_optimizer_step(MambaBlock *block, const MBOptimConfig *conf);
float mamba_block_grad_sqnorm(const MambaBlock *block);

/* Accumulates the block's parameter gradients (into opt_state) and writes
 * d_input for batch item batch_index of the last forward input. */
void mamba_backward(MambaBlock *block, const float *dY, const float *input, float *d_input,
                    size_t batch_index);
void mamba_backward_ws(MambaBlock *block, MambaBlockWorkspace *ws, const float *dY,
                       const float *input, float *d_input, size_t batch_index);
void mamba_backward_ws_local(MambaBlock *block, MambaBlockWorkspace *ws, const float *dY,
                             const float *input, float *d_input, size_t batch_index,
                             MBOptimState *local_grad);

MBOptimState *mamba_local_grad_alloc(const MambaBlock *block);
void mamba_local_grad_reduce(MambaBlock *block, const MBOptimState *local);
void mamba_local_grad_free(MBOptimState *local);

/* ---------------------------------------------------------------- matrix */
MBMatrix *mb_matrix_create(size_t rows, size_t cols);
void mb_matrix_free(MBMatrix *m);
void mb_matrix_zero(MBMatrix *m);
void mb_matrix_copy(MBMatrix *dst, const MBMatrix *src);
void mb_matrix_print(const MBMatrix *m);
void mb_matrix_vec_mult(float *out, const MBMatrix *m, const float *v);
void mb_vec_add(float *y, const float *x, size_t n);
void mb_vec_scale(float *v, float alpha, size_t n);
void mb_compute_delta(float *delta_out, const MambaBlock *block, const float *delta_in,
                      size_t seq_len);

/* ---------------------------------------------------------------- model */
KMamba *kmamba_create(const KMambaConfig *cfg);
void kmamba_free(KMamba *m);
int kmamba_init(KMamba *m, uint32_t seed);
int kmamba_enable_training(KMamba *m, const MBOptimConfig *opt_blocks, float lr_embed_head,
                           float weight_decay);
int kmamba_enable_training_with_optimizer(KMamba *m, OptimizerType opt_type,
                                          const MBOptimConfig *opt_blocks, float lr_embed_head,
                                          float weight_decay);
int kmamba_save(const KMamba *m, const char *path);
KMamba *kmamba_load(const char *path, int for_training, const MBOptimConfig *opt_blocks,
                    float lr_embed_head, float weight_decay);
/* tokens [seq_len]; logits_out [seq_len, vocab_size] */
int kmamba_forward(KMamba *m, const uint32_t *tokens, float *logits_out);
/* tokens_plus1 [seq_len + 1]; returns the loss before the update */
float kmamba_train_step(KMamba *m, const uint32_t *tokens_plus1);
/* batch_tokens [batch_size, seq_len + 1]; returns the mean loss */
float kmamba_train_batch(KMamba *m, const uint32_t *batch_tokens, size_t batch_size);
float kmamba_train_batch_hybrid(KMamba *m, const uint32_t *batch_tokens, size_t batch_size);

float kmamba_last_grad_norm(const KMamba *m);
float kmamba_last_grad_over_clip(const KMamba *m);
int kmamba_last_grad_would_clip(const KMamba *m);
size_t kmamba_step_count(const KMamba *m);
void kmamba_update_lr(KMamba *m, float lr_blocks, float lr_embed);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_H */
