#ifndef KMAMBA_DISTRIBUTED_H
#define KMAMBA_DISTRIBUTED_H

/*
 * Multi-GPU data parallelism over NCCL, with the names, struct layouts and
 * return conventions of the reference include/kmamba_distributed.h (NCCL
 * variant, KMAMBA_USE_NCCL; implementation cuda/kmamba_distributed.cu:
 * 22-138 and src/kmamba_distributed.c:19-158).  This library is always
 * built with NCCL, so the context is the reference's NCCL context; its
 * handles are declared as void * here so that callers need not include
 * nccl.h.
 *
 * What the reference leaves broken is completed here:
 *  - the NCCL unique id is exchanged (the reference never sends rank 0's id
 *    to the other ranks, cuda/kmamba_distributed.cu:46-53): through a
 *    rendezvous file named by the KMAMBA_NCCL_ID_FILE environment variable
 *    for kmamba_distributed_init_nccl, or by the caller with
 *    kmb_dist_get_unique_id / kmb_dist_init_with_id;
 *  - the device is the process's local rank (LOCAL_RANK, else rank modulo
 *    the device count), not the global rank.
 * Every function returns 0 / NULL on success / failure as the reference
 * does; kmb_last_error() (kmamba_b200.h) says why a call failed.
 */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int world_size;   /* total number of GPUs (1 = single GPU) */
    int rank;         /* this process's rank, 0 .. world_size - 1 */
    int local_rank;   /* device index on this node */
    size_t layer_start;
    size_t layer_end;
    size_t batch_start;
    size_t batch_end;
    int use_nccl;
    int use_p2p;
} KMambaDistributedConfig;

static inline KMambaDistributedConfig kmamba_distributed_default(void) {
    KMambaDistributedConfig c;
    c.world_size = 1;
    c.rank = 0;
    c.local_rank = 0;
    c.layer_start = 0;
    c.layer_end = 0;
    c.batch_start = 0;
    c.batch_end = 0;
    c.use_nccl = 0;
    c.use_p2p = 0;
    return c;
}

typedef struct {
    KMambaDistributedConfig config;
    void *nccl_comm;     /* ncclComm_t */
    void *stream;        /* cudaStream_t of the collectives */
    void *nccl_scratch;  /* unused (NULL); kept for the reference layout */
    size_t scratch_size;
} KMambaDistributedContext;

/* NULL for world_size <= 1, as the reference.  The ranks meet through the
 * file named by KMAMBA_NCCL_ID_FILE (rank 0 writes the id, the others wait
 * for it up to KMAMBA_NCCL_TIMEOUT_S seconds, default 120); use a fresh
 * path for every job, since a file left by an earlier job would be read as
 * this job's id. */
KMambaDistributedContext *kmamba_distributed_init_nccl(int world_size, int rank);
void kmamba_distributed_fini_nccl(KMambaDistributedContext *ctx);
/* In-place fp32 sum over the ranks, synchronous (the reference's
 * contract).  0 / -1. */
int kmamba_allreduce_gradients_nccl(KMambaDistributedContext *ctx, float *d_gradients,
                                    size_t n_elements);
/* In-place broadcast of rank 0's values, synchronous.  0 / -1. */
int kmamba_broadcast_params_nccl(KMambaDistributedContext *ctx, float *d_params,
                                 size_t n_elements);

/* Pipeline helpers of the reference (pipeline parallelism itself is not
 * part of this library's hot path): a context over n_gpus devices of this
 * process with peer access enabled where the devices allow it, and a
 * device-to-device copy between two ranks' buffers. */
KMambaDistributedContext *kmamba_distributed_init_pipeline(int n_gpus);
void kmamba_distributed_fini_pipeline(KMambaDistributedContext *ctx);
int kmamba_pipeline_send_recv(KMambaDistributedContext *ctx, float *d_send_buf,
                              float *d_recv_buf, size_t n_elements, int dst_rank,
                              int src_rank);

/* Contiguous shards, earlier ranks taking one extra item (or layer) when
 * the count does not divide evenly; sets world_size. */
void kmamba_distributed_split_batch(KMambaDistributedConfig *cfg, size_t batch_size,
                                    size_t total_gpus);
void kmamba_distributed_split_layers(KMambaDistributedConfig *cfg, size_t n_layers,
                                     size_t total_gpus);

/* ------------------------------------------------------------------ */
/* Extensions (no counterpart in the reference)                        */
/* ------------------------------------------------------------------ */

/* 128-byte NCCL unique id for the caller to send to every rank. */
int kmb_dist_get_unique_id(void *id_out);
/* Context over `device` for rank / world_size, from rank 0's id; also
 * valid for world_size 1.  NULL on failure. */
KMambaDistributedContext *kmb_dist_init_with_id(int world_size, int rank, int device,
                                                const void *id);
/* Rendezvous file exchange used by kmamba_distributed_init_nccl: rank 0
 * writes `bytes` bytes of id to path (atomically, by rename); other ranks
 * read them, waiting up to timeout_s.  KMB_OK / KMB_ETIMEOUT / KMB_EINVAL. */
int kmb_dist_rendezvous_file(const char *path, int rank, void *id, size_t bytes,
                             double timeout_s);

/*
 * Gradient buckets, all-reduced on the context's stream while the caller's
 * stream goes on with other work (the backward of earlier layers, or the
 * next forward).  kmb_dist_bucket_add hands over a gradient range whose
 * producing kernels have been enqueued on `stream`; ranges that are
 * adjacent in memory are coalesced until the pending range reaches the
 * bucket size (kmb_dist_set_bucket_bytes, default 25 MiB), then the
 * context stream waits for `stream` and runs one in-place ncclAllReduce
 * (sum, or mean when `average`) on it.  kmb_dist_bucket_flush issues the
 * pending range; kmb_dist_wait makes `stream` wait for every collective
 * issued so far.  Every rank must add the same ranges in the same order.
 */
int kmb_dist_set_bucket_bytes(KMambaDistributedContext *ctx, size_t bytes);
int kmb_dist_bucket_add(KMambaDistributedContext *ctx, float *d_grad, size_t n_elements,
                        int average, void *stream);
int kmb_dist_bucket_flush(KMambaDistributedContext *ctx, void *stream);
int kmb_dist_wait(KMambaDistributedContext *ctx, void *stream);
/* Collectives issued and bytes reduced by this context so far. */
int kmb_dist_stats(const KMambaDistributedContext *ctx, unsigned long long *collectives,
                   unsigned long long *bytes);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_DISTRIBUTED_H */
