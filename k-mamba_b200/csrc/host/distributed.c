/*
 * kmamba_distributed.h over NCCL (NVLink / NVSwitch inside a node).
 *
 * A context owns one NCCL communicator and one non-blocking CUDA stream on
 * which every collective runs.  Synchronous entry points (the reference's
 * kmamba_allreduce_gradients_nccl / kmamba_broadcast_params_nccl) wait for
 * that stream; the bucket API orders the collectives after the caller's
 * stream with events, so a reduction overlaps whatever the caller enqueues
 * next.
 *
 * Reference: cuda/kmamba_distributed.cu:22-138 (init, all-reduce,
 * broadcast), src/kmamba_distributed.c:19-158 (pipeline helpers, batch and
 * layer splits).
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <dlfcn.h>
#include <pthread.h>

#include <nccl.h>

#include "kmamba_distributed.h"
#include "../kmb_internal.h"

/*
 * NCCL is opened on the first distributed call (dlopen), not linked: a
 * process that already holds a libnccl.so.2 -- a framework's bundled copy,
 * loaded with that framework -- then shares it instead of pinning another
 * version under the same soname before the framework loads.  The
 * KMAMBA_NCCL_LIBRARY environment variable names a specific library.
 */
static struct {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t);
    ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t);
    const char *(*error_string)(ncclResult_t);
    int loaded;
} g_nccl;
static pthread_mutex_t g_nccl_mu = PTHREAD_MUTEX_INITIALIZER;

static int nccl_load(void) {
    pthread_mutex_lock(&g_nccl_mu);
    if (!g_nccl.loaded) {
        const char *name = getenv("KMAMBA_NCCL_LIBRARY");
        void *h = dlopen(name && *name ? name : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            *(void **)&g_nccl.get_unique_id = dlsym(h, "ncclGetUniqueId");
            *(void **)&g_nccl.comm_init_rank = dlsym(h, "ncclCommInitRank");
            *(void **)&g_nccl.comm_destroy = dlsym(h, "ncclCommDestroy");
            *(void **)&g_nccl.all_reduce = dlsym(h, "ncclAllReduce");
            *(void **)&g_nccl.broadcast = dlsym(h, "ncclBroadcast");
            *(void **)&g_nccl.error_string = dlsym(h, "ncclGetErrorString");
            g_nccl.loaded = g_nccl.get_unique_id && g_nccl.comm_init_rank &&
                            g_nccl.comm_destroy && g_nccl.all_reduce && g_nccl.broadcast &&
                            g_nccl.error_string;
        }
    }
    const int ok = g_nccl.loaded;
    const char *why = ok ? NULL : dlerror();
    pthread_mutex_unlock(&g_nccl_mu);
    return ok ? KMB_OK : kmb_fail(KMB_EUNSUPPORTED, "dist: cannot load NCCL (libnccl.so.2): %s",
                                  why ? why : "missing symbols");
}

#define KMB_DIST_MAX_GPUS 64

typedef struct {
    KMambaDistributedContext pub; /* must stay first: callers see this */
    float *pend;                  /* pending (not yet reduced) range */
    size_t pend_n;
    int pend_avg;
    size_t bucket_bytes;
    cudaEvent_t ready;            /* caller stream -> collective stream */
    cudaEvent_t done;             /* collective stream -> caller stream */
    unsigned long long collectives, bytes;
    int device;
    int pipeline;                 /* a pipeline context (no communicator) */
    int n_gpus;
} DistCtx;

static DistCtx *priv(KMambaDistributedContext *c) { return (DistCtx *)c; }

static int nccl_fail(ncclResult_t r, const char *where) {
    return kmb_fail(KMB_ECUDA, "%s: %s", where, g_nccl.error_string(r));
}

/* ------------------------------------------------------------------ */
/* rendezvous of the unique id                                          */
/* ------------------------------------------------------------------ */

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

int kmb_dist_rendezvous_file(const char *path, int rank, void *id, size_t bytes,
                             double timeout_s) {
    if (!path || !*path || !id || bytes == 0 || bytes > 4096 || rank < 0)
        return kmb_fail(KMB_EINVAL, "rendezvous: bad arguments");
    if (rank == 0) {
        char tmp[4200];
        if (snprintf(tmp, sizeof tmp, "%s.tmp.%d", path, (int)getpid()) >= (int)sizeof tmp)
            return kmb_fail(KMB_EINVAL, "rendezvous: path too long");
        FILE *f = fopen(tmp, "wb");
        if (!f) return kmb_fail(KMB_EINVAL, "rendezvous: cannot write %s (%s)", tmp, strerror(errno));
        const size_t w = fwrite(id, 1, bytes, f);
        const int closed = fclose(f);
        if (w != bytes || closed != 0 || rename(tmp, path) != 0) {
            unlink(tmp);
            return kmb_fail(KMB_EINVAL, "rendezvous: cannot publish %s", path);
        }
        return KMB_OK;
    }
    const double t0 = now_s();
    for (;;) {
        FILE *f = fopen(path, "rb");
        if (f) {
            const size_t r = fread(id, 1, bytes, f);
            fclose(f);
            if (r == bytes) return KMB_OK;
        }
        if (now_s() - t0 > timeout_s)
            return kmb_fail(KMB_ETIMEOUT, "rendezvous: no id in %s after %.1f s", path,
                            timeout_s);
        usleep(2000);
    }
}

/* ------------------------------------------------------------------ */
/* contexts                                                             */
/* ------------------------------------------------------------------ */

int kmb_dist_get_unique_id(void *id_out) {
    if (!id_out) return kmb_fail(KMB_EINVAL, "dist: NULL id");
    if (nccl_load()) return KMB_EUNSUPPORTED;
    ncclUniqueId id;
    const ncclResult_t r = g_nccl.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id_out, &id, sizeof id);
    return KMB_OK;
}

static void ctx_free(DistCtx *c) {
    if (!c) return;
    if (c->ready) cudaEventDestroy(c->ready);
    if (c->done) cudaEventDestroy(c->done);
    if (c->pub.stream) cudaStreamDestroy((cudaStream_t)c->pub.stream);
    free(c);
}

KMambaDistributedContext *kmb_dist_init_with_id(int world_size, int rank, int device,
                                                const void *id) {
    if (world_size < 1 || rank < 0 || rank >= world_size || device < 0 || !id) {
        kmb_fail(KMB_EINVAL, "dist: world_size %d, rank %d, device %d", world_size, rank, device);
        return NULL;
    }
    if (nccl_load()) return NULL;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        kmb_cuda_fail(e, "dist: cudaSetDevice");
        return NULL;
    }
    DistCtx *c = (DistCtx *)calloc(1, sizeof *c);
    if (!c) {
        kmb_fail(KMB_ENOMEM, "dist: host allocation failed");
        return NULL;
    }
    c->device = device;
    c->bucket_bytes = (size_t)25 << 20;
    c->pub.config = kmamba_distributed_default();
    c->pub.config.world_size = world_size;
    c->pub.config.rank = rank;
    c->pub.config.local_rank = device;
    c->pub.config.use_nccl = 1;
    cudaStream_t s = NULL;
    if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&c->ready, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming)) != cudaSuccess) {
        c->pub.stream = s;
        kmb_cuda_fail(e, "dist: stream / event");
        ctx_free(c);
        return NULL;
    }
    c->pub.stream = s;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclComm_t comm = NULL;
    const ncclResult_t r = g_nccl.comm_init_rank(&comm, world_size, uid, rank);
    if (r != ncclSuccess) {
        nccl_fail(r, "ncclCommInitRank");
        ctx_free(c);
        return NULL;
    }
    c->pub.nccl_comm = comm;
    return &c->pub;
}

static int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    if (!v || !*v) return dflt;
    char *end = NULL;
    const long x = strtol(v, &end, 10);
    return (end && *end == 0) ? (int)x : dflt;
}

KMambaDistributedContext *kmamba_distributed_init_nccl(int world_size, int rank) {
    if (world_size <= 1) return NULL; /* single GPU: no communicator (reference) */
    if (rank < 0 || rank >= world_size) {
        kmb_fail(KMB_EINVAL, "dist: rank %d outside world %d", rank, world_size);
        return NULL;
    }
    const char *path = getenv("KMAMBA_NCCL_ID_FILE");
    if (!path || !*path) {
        kmb_fail(KMB_EINVAL, "dist: set KMAMBA_NCCL_ID_FILE to a path every rank can reach "
                             "(rank 0 publishes the NCCL id there), or use "
                             "kmb_dist_get_unique_id / kmb_dist_init_with_id");
        return NULL;
    }
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev <= 0) {
        kmb_cuda_fail(e != cudaSuccess ? e : cudaErrorNoDevice, "dist: no CUDA device");
        return NULL;
    }
    const int device = env_int("LOCAL_RANK", rank % ndev);
    unsigned char id[sizeof(ncclUniqueId)];
    if (rank == 0 && kmb_dist_get_unique_id(id) != KMB_OK) return NULL;
    const double timeout = (double)env_int("KMAMBA_NCCL_TIMEOUT_S", 120);
    if (kmb_dist_rendezvous_file(path, rank, id, sizeof id, timeout) != KMB_OK) return NULL;
    return kmb_dist_init_with_id(world_size, rank, device, id);
}

void kmamba_distributed_fini_nccl(KMambaDistributedContext *ctx) {
    if (!ctx) return;
    DistCtx *c = priv(ctx);
    if (c->pipeline) {
        kmamba_distributed_fini_pipeline(ctx);
        return;
    }
    if (c->pub.stream) cudaStreamSynchronize((cudaStream_t)c->pub.stream);
    if (c->pub.nccl_comm) g_nccl.comm_destroy((ncclComm_t)c->pub.nccl_comm);
    ctx_free(c);
}

/* ------------------------------------------------------------------ */
/* collectives                                                          */
/* ------------------------------------------------------------------ */

static int usable(KMambaDistributedContext *ctx, const void *p) {
    if (!ctx || !p) return kmb_fail(KMB_EINVAL, "dist: NULL context or buffer");
    if (priv(ctx)->pipeline || !ctx->nccl_comm)
        return kmb_fail(KMB_EINVAL, "dist: context has no NCCL communicator");
    if (!kmb_is_device_ptr(p)) return kmb_fail(KMB_EINVAL, "dist: buffer must be device memory");
    return KMB_OK;
}

static int reduce_now(DistCtx *c, float *p, size_t n, int avg) {
    if (n == 0) return KMB_OK;
    const ncclResult_t r = g_nccl.all_reduce(p, p, n, ncclFloat, avg ? ncclAvg : ncclSum,
                                         (ncclComm_t)c->pub.nccl_comm,
                                         (cudaStream_t)c->pub.stream);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    c->collectives++;
    c->bytes += (unsigned long long)n * sizeof(float);
    return KMB_OK;
}

int kmamba_allreduce_gradients_nccl(KMambaDistributedContext *ctx, float *d, size_t n) {
    if (usable(ctx, d)) return -1;
    DistCtx *c = priv(ctx);
    /* the reference reduces on the context stream: order it after the
     * caller's (library) stream, where the gradients were produced */
    cudaError_t e = cudaEventRecord(c->ready, kmb_stream());
    if (e == cudaSuccess) e = cudaStreamWaitEvent((cudaStream_t)ctx->stream, c->ready, 0);
    if (e != cudaSuccess) {
        kmb_cuda_fail(e, "dist: order after caller stream");
        return -1;
    }
    if (reduce_now(c, d, n, 0)) return -1;
    e = cudaStreamSynchronize((cudaStream_t)ctx->stream);
    return e == cudaSuccess ? 0 : (kmb_cuda_fail(e, "dist: synchronize"), -1);
}

int kmamba_broadcast_params_nccl(KMambaDistributedContext *ctx, float *d, size_t n) {
    if (usable(ctx, d)) return -1;
    DistCtx *c = priv(ctx);
    cudaError_t e = cudaEventRecord(c->ready, kmb_stream());
    if (e == cudaSuccess) e = cudaStreamWaitEvent((cudaStream_t)ctx->stream, c->ready, 0);
    if (e != cudaSuccess) return (kmb_cuda_fail(e, "dist: order after caller stream"), -1);
    const ncclResult_t r = g_nccl.broadcast(d, d, n, ncclFloat, 0, (ncclComm_t)ctx->nccl_comm,
                                         (cudaStream_t)ctx->stream);
    if (r != ncclSuccess) return (nccl_fail(r, "ncclBroadcast"), -1);
    c->collectives++;
    c->bytes += (unsigned long long)n * sizeof(float);
    e = cudaStreamSynchronize((cudaStream_t)ctx->stream);
    return e == cudaSuccess ? 0 : (kmb_cuda_fail(e, "dist: synchronize"), -1);
}

int kmb_dist_set_bucket_bytes(KMambaDistributedContext *ctx, size_t bytes) {
    if (!ctx || bytes < sizeof(float)) return kmb_fail(KMB_EINVAL, "dist: bucket size");
    priv(ctx)->bucket_bytes = bytes;
    return KMB_OK;
}

int kmb_dist_bucket_flush(KMambaDistributedContext *ctx, void *stream) {
    if (!ctx) return kmb_fail(KMB_EINVAL, "dist: NULL context");
    DistCtx *c = priv(ctx);
    if (!c->pend || c->pend_n == 0) return KMB_OK;
    cudaError_t e = cudaEventRecord(c->ready, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent((cudaStream_t)ctx->stream, c->ready, 0);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "dist: bucket ordering");
    const int rc = reduce_now(c, c->pend, c->pend_n, c->pend_avg);
    c->pend = NULL;
    c->pend_n = 0;
    return rc;
}

int kmb_dist_bucket_add(KMambaDistributedContext *ctx, float *d, size_t n, int average,
                        void *stream) {
    int rc = usable(ctx, d);
    if (rc) return rc;
    DistCtx *c = priv(ctx);
    if (n == 0) return KMB_OK;
    const int avg = average ? 1 : 0;
    if (c->pend && (c->pend + c->pend_n != d || c->pend_avg != avg)) {
        if ((rc = kmb_dist_bucket_flush(ctx, stream))) return rc;
    }
    if (!c->pend) {
        c->pend = d;
        c->pend_avg = avg;
    }
    c->pend_n += n;
    if (c->pend_n * sizeof(float) >= c->bucket_bytes) return kmb_dist_bucket_flush(ctx, stream);
    return KMB_OK;
}

int kmb_dist_wait(KMambaDistributedContext *ctx, void *stream) {
    if (!ctx) return kmb_fail(KMB_EINVAL, "dist: NULL context");
    DistCtx *c = priv(ctx);
    if (c->pipeline) return KMB_OK;
    cudaError_t e = cudaEventRecord(c->done, (cudaStream_t)ctx->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent((cudaStream_t)stream, c->done, 0);
    return e == cudaSuccess ? KMB_OK : kmb_cuda_fail(e, "dist: wait");
}

int kmb_dist_stats(const KMambaDistributedContext *ctx, unsigned long long *collectives,
                   unsigned long long *bytes) {
    if (!ctx) return kmb_fail(KMB_EINVAL, "dist: NULL context");
    const DistCtx *c = (const DistCtx *)ctx;
    if (collectives) *collectives = c->collectives;
    if (bytes) *bytes = c->bytes;
    return KMB_OK;
}

/* ------------------------------------------------------------------ */
/* pipeline helpers (src/kmamba_distributed.c:19-112)                  */
/* ------------------------------------------------------------------ */

KMambaDistributedContext *kmamba_distributed_init_pipeline(int n_gpus) {
    if (n_gpus <= 0 || n_gpus > KMB_DIST_MAX_GPUS) return NULL;
    DistCtx *c = (DistCtx *)calloc(1, sizeof *c);
    if (!c) return NULL;
    c->pipeline = 1;
    c->n_gpus = n_gpus;
    c->pub.config = kmamba_distributed_default();
    c->pub.config.world_size = n_gpus;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess) {
        (void)cudaGetLastError();
        ndev = 0;
    }
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) (void)cudaGetLastError();
    int all = n_gpus > 1 && n_gpus <= ndev;
    for (int i = 0; all && i < n_gpus; ++i) {
        for (int j = 0; j < n_gpus; ++j) {
            if (i == j) continue;
            int can = 0;
            if (cudaDeviceCanAccessPeer(&can, i, j) != cudaSuccess || !can) {
                (void)cudaGetLastError();
                all = 0;
                continue;
            }
            if (cudaSetDevice(i) == cudaSuccess) {
                const cudaError_t e = cudaDeviceEnablePeerAccess(j, 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) all = 0;
                (void)cudaGetLastError();
            }
        }
    }
    if (cudaSetDevice(cur) != cudaSuccess) (void)cudaGetLastError();
    c->pub.config.use_p2p = all;
    return &c->pub;
}

void kmamba_distributed_fini_pipeline(KMambaDistributedContext *ctx) {
    /* peer access stays enabled: it belongs to the process's contexts and
     * other users of the devices in this process may rely on it */
    if (ctx) free(priv(ctx));
}

int kmamba_pipeline_send_recv(KMambaDistributedContext *ctx, float *send, float *recv,
                              size_t n, int dst_rank, int src_rank) {
    (void)ctx;
    (void)dst_rank;
    (void)src_rank;
    if (!send || !recv) return -1;
    const cudaError_t e = cudaMemcpy(recv, send, n * sizeof(float), cudaMemcpyDefault);
    return e == cudaSuccess ? 0 : (kmb_cuda_fail(e, "pipeline copy"), -1);
}

/* ------------------------------------------------------------------ */
/* shard arithmetic (src/kmamba_distributed.c:118-158)                  */
/* ------------------------------------------------------------------ */

/* [start, end) of `rank`'s contiguous share of `count` items over `parts`
 * ranks; the first count % parts ranks hold one extra item. */
static void share(size_t count, size_t parts, size_t rank, size_t *start, size_t *end) {
    const size_t base = count / parts, extra = count % parts;
    *start = rank * base + (rank < extra ? rank : extra);
    *end = *start + base + (rank < extra ? 1 : 0);
}

void kmamba_distributed_split_batch(KMambaDistributedConfig *cfg, size_t batch_size,
                                    size_t total_gpus) {
    if (!cfg || total_gpus == 0) return;
    cfg->world_size = (int)total_gpus;
    share(batch_size, total_gpus, (size_t)cfg->rank, &cfg->batch_start, &cfg->batch_end);
}

void kmamba_distributed_split_layers(KMambaDistributedConfig *cfg, size_t n_layers,
                                     size_t total_gpus) {
    if (!cfg || total_gpus == 0) return;
    cfg->world_size = (int)total_gpus;
    share(n_layers, total_gpus, (size_t)cfg->rank, &cfg->layer_start, &cfg->layer_end);
}
