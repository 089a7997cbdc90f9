/*
 * Host runtime of the B200 k-mamba library: error reporting, the library
 * stream, the device buffer pool and host<->device staging of caller
 * buffers.
 *
 * The reference keeps a thread-local first-fit pool of host chunks
 * (src/km_memory_pool.c:54-117).  Here the scratch lives on the device, so
 * the pool caches cudaMalloc blocks per device and hands them out by size
 * under a mutex.  Every call that staged buffers or used pooled scratch
 * synchronizes its stream before the blocks go back to the pool, so a
 * block is never reused while a kernel may still read it.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../kmb_internal.h"

/* ------------------------------------------------------------------ */
/* errors                                                              */
/* ------------------------------------------------------------------ */

static __thread char t_err[512];
static __thread int t_status;

int kmb_fail(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof t_err, fmt, ap);
    va_end(ap);
    t_status = status;
    return status;
}

int kmb_cuda_fail(cudaError_t e, const char *where) {
    (void)cudaGetLastError(); /* do not leave the error for the next caller */
    return kmb_fail(KMB_ECUDA, "%s: %s (%s)", where, cudaGetErrorString(e),
                    cudaGetErrorName(e));
}

const char *kmb_last_error(void) { return t_err; }
int kmb_last_status(void) { return t_status; }
void kmb_clear_error(void) {
    t_err[0] = 0;
    t_status = 0;
}

/* ------------------------------------------------------------------ */
/* stream and synchronisation mode                                     */
/* ------------------------------------------------------------------ */

static __thread cudaStream_t t_stream;
static int g_sync = 1;

void kmb_set_stream(void *s) { t_stream = (cudaStream_t)s; }
void *kmb_get_stream(void) { return (void *)t_stream; }
cudaStream_t kmb_stream(void) { return t_stream; }
void kmb_set_sync(int on) { __atomic_store_n(&g_sync, on ? 1 : 0, __ATOMIC_RELAXED); }
int kmb_get_sync(void) { return __atomic_load_n(&g_sync, __ATOMIC_RELAXED); }
int kmb_sync_enabled(void) { return kmb_get_sync(); }

int kmb_is_device_ptr(const void *p) {
    struct cudaPointerAttributes at;
    cudaError_t e;
    if (!p) return 0;
    e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

/* ------------------------------------------------------------------ */
/* device pool                                                         */
/* ------------------------------------------------------------------ */

typedef struct PoolBlock {
    void *p;
    size_t bytes;
    int device;
    int used;
    struct PoolBlock *next;
} PoolBlock;

static pthread_mutex_t g_pool_mu = PTHREAD_MUTEX_INITIALIZER;
static PoolBlock *g_pool;
static size_t g_pool_held;

static size_t pool_round(size_t n) {
    const size_t q = 512;
    if (n == 0) n = 1;
    return (n + q - 1) / q * q;
}

static size_t pool_trim_locked(void) {
    size_t freed = 0;
    PoolBlock **pp = &g_pool;
    while (*pp) {
        PoolBlock *b = *pp;
        if (!b->used) {
            int cur = 0;
            cudaGetDevice(&cur);
            if (cur != b->device) cudaSetDevice(b->device);
            cudaFree(b->p);
            if (cur != b->device) cudaSetDevice(cur);
            freed += b->bytes;
            g_pool_held -= b->bytes;
            *pp = b->next;
            free(b);
        } else {
            pp = &b->next;
        }
    }
    return freed;
}

void *kmb_pool_alloc(size_t bytes) {
    int dev = 0;
    PoolBlock *best = NULL;
    void *p = NULL;
    cudaError_t e;

    if (cudaGetDevice(&dev) != cudaSuccess) {
        (void)cudaGetLastError();
        kmb_fail(KMB_ECUDA, "kmb_pool_alloc: no CUDA device");
        return NULL;
    }
    bytes = pool_round(bytes);
    pthread_mutex_lock(&g_pool_mu);
    for (PoolBlock *b = g_pool; b; b = b->next) {
        if (b->used || b->device != dev || b->bytes < bytes || b->bytes > 2 * bytes)
            continue;
        if (!best || b->bytes < best->bytes) best = b;
    }
    if (best) {
        best->used = 1;
        p = best->p;
        pthread_mutex_unlock(&g_pool_mu);
        return p;
    }
    e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        pool_trim_locked();
        e = cudaMalloc(&p, bytes);
    }
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        pthread_mutex_unlock(&g_pool_mu);
        kmb_cuda_fail(e, "kmb_pool_alloc cudaMalloc");
        return NULL;
    }
    best = (PoolBlock *)calloc(1, sizeof *best);
    if (!best) {
        cudaFree(p);
        pthread_mutex_unlock(&g_pool_mu);
        kmb_fail(KMB_ENOMEM, "kmb_pool_alloc: host allocation failed");
        return NULL;
    }
    best->p = p;
    best->bytes = bytes;
    best->device = dev;
    best->used = 1;
    best->next = g_pool;
    g_pool = best;
    g_pool_held += bytes;
    pthread_mutex_unlock(&g_pool_mu);
    return p;
}

void kmb_pool_free(void *p) {
    if (!p) return;
    pthread_mutex_lock(&g_pool_mu);
    for (PoolBlock *b = g_pool; b; b = b->next) {
        if (b->p == p) {
            b->used = 0;
            break;
        }
    }
    pthread_mutex_unlock(&g_pool_mu);
}

size_t kmb_pool_trim(void) {
    size_t f;
    pthread_mutex_lock(&g_pool_mu);
    f = pool_trim_locked();
    pthread_mutex_unlock(&g_pool_mu);
    return f;
}

size_t kmb_pool_bytes_held(void) {
    size_t h;
    pthread_mutex_lock(&g_pool_mu);
    h = g_pool_held;
    pthread_mutex_unlock(&g_pool_mu);
    return h;
}

/* ------------------------------------------------------------------ */
/* device-resident host arrays                                         */
/* ------------------------------------------------------------------ */

/* A host array registered here has a device copy that staging uses in its
 * place: no host->device copy on the way in and no copy back on the way
 * out.  The device copy is then the array's current value until
 * kmb_resident_sync copies it back. */
typedef struct {
    const void *host;
    void *dev;
    size_t bytes;
    int device;
} ResidentBuf;

static ResidentBuf *g_res;
static int g_nres, g_rescap;
static pthread_mutex_t g_res_mu = PTHREAD_MUTEX_INITIALIZER;

static int current_device(void) {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess) {
        (void)cudaGetLastError();
        d = -1;
    }
    return d;
}

/* index of `host` on `device`, or -1 (caller holds g_res_mu) */
static int resident_index(const void *host, int device) {
    for (int i = 0; i < g_nres; ++i)
        if (g_res[i].host == host && g_res[i].device == device) return i;
    return -1;
}

static void *resident_find(const void *host, size_t bytes) {
    void *d = NULL;
    if (!g_nres) return NULL;
    const int dev = current_device();
    pthread_mutex_lock(&g_res_mu);
    const int i = resident_index(host, dev);
    if (i >= 0 && bytes <= g_res[i].bytes) d = g_res[i].dev;
    pthread_mutex_unlock(&g_res_mu);
    return d;
}

int kmb_resident_add(const void *host, size_t bytes) {
    cudaError_t e;
    int rc = KMB_OK;
    if (!host || !bytes) return kmb_fail(KMB_EINVAL, "resident: NULL or empty array");
    if (kmb_is_device_ptr(host)) return KMB_OK; /* already device memory */
    const int dev = current_device();
    pthread_mutex_lock(&g_res_mu);
    int i = resident_index(host, dev);
    if (i >= 0 && bytes > g_res[i].bytes) {
        pthread_mutex_unlock(&g_res_mu);
        return kmb_fail(KMB_EINVAL, "resident: %p registered with %zu bytes, not %zu", host,
                        g_res[i].bytes, bytes);
    }
    if (i < 0) {
        void *d = NULL;
        if (g_nres == g_rescap) {
            const int cap = g_rescap ? 2 * g_rescap : 64;
            ResidentBuf *t = (ResidentBuf *)realloc(g_res, sizeof *t * (size_t)cap);
            if (!t) {
                pthread_mutex_unlock(&g_res_mu);
                return kmb_fail(KMB_ENOMEM, "resident: host allocation failed");
            }
            g_res = t;
            g_rescap = cap;
        }
        e = cudaMalloc(&d, bytes);
        if (e != cudaSuccess) {
            pthread_mutex_unlock(&g_res_mu);
            return kmb_cuda_fail(e, "resident: cudaMalloc");
        }
        i = g_nres++;
        g_res[i].host = host;
        g_res[i].dev = d;
        g_res[i].bytes = bytes;
        g_res[i].device = dev;
    }
    /* (re-)upload the host value; ordered after the library stream's work */
    e = cudaStreamSynchronize(kmb_stream());
    if (e == cudaSuccess) e = cudaMemcpy(g_res[i].dev, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) rc = kmb_cuda_fail(e, "resident: upload");
    pthread_mutex_unlock(&g_res_mu);
    return rc;
}

int kmb_resident_update(const void *host) {
    if (!g_nres) return KMB_OK;
    const int dev = current_device();
    pthread_mutex_lock(&g_res_mu);
    const int i = resident_index(host, dev);
    size_t bytes = i >= 0 ? g_res[i].bytes : 0;
    pthread_mutex_unlock(&g_res_mu);
    return i >= 0 ? kmb_resident_add(host, bytes) : KMB_OK;
}

int kmb_resident_sync(void *host) {
    cudaError_t e;
    int rc = KMB_OK;
    const int dev = current_device();
    pthread_mutex_lock(&g_res_mu);
    const int i = resident_index(host, dev);
    if (i >= 0) {
        e = cudaStreamSynchronize(kmb_stream());
        if (e == cudaSuccess) e = cudaMemcpy(host, g_res[i].dev, g_res[i].bytes, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "resident: download");
    }
    pthread_mutex_unlock(&g_res_mu);
    return rc;
}

int kmb_resident_remove(void *host, int copy_back) {
    int rc = copy_back ? kmb_resident_sync(host) : KMB_OK;
    const int dev = current_device();
    pthread_mutex_lock(&g_res_mu);
    const int i = resident_index(host, dev);
    if (i >= 0) {
        (void)cudaStreamSynchronize(kmb_stream());
        cudaFree(g_res[i].dev);
        g_res[i] = g_res[--g_nres];
    }
    pthread_mutex_unlock(&g_res_mu);
    return rc;
}

int kmb_resident_count(void) {
    pthread_mutex_lock(&g_res_mu);
    const int n = g_nres;
    pthread_mutex_unlock(&g_res_mu);
    return n;
}

/* ------------------------------------------------------------------ */
/* staging                                                             */
/* ------------------------------------------------------------------ */

void kmb_stage_begin(KmbStage *st) {
    /* a call that passed validation starts with a clean error state, so
     * kmb_last_status() always describes the latest call */
    kmb_clear_error();
    memset(st, 0, sizeof *st);
    st->b = st->inl;
    st->cap = KMB_STAGE_MAX;
    st->s = kmb_stream();
}

int kmb_stage_reserve(KmbStage *st, int cap) {
    KmbStageBuf *t;
    if (cap <= st->cap) return KMB_OK;
    t = (KmbStageBuf *)calloc((size_t)cap, sizeof *t);
    if (!t) return st->status = kmb_fail(KMB_ENOMEM, "staging: host allocation failed");
    memcpy(t, st->b, sizeof *t * (size_t)st->n);
    if (st->b != st->inl) free(st->b);
    st->b = t;
    st->cap = cap;
    return KMB_OK;
}

static KmbStageBuf *stage_find(KmbStage *st, const void *p) {
    for (int i = 0; i < st->n; ++i)
        if (st->b[i].user == p) return &st->b[i];
    return NULL;
}

static void *stage_add(KmbStage *st, const void *p, size_t bytes, int out, int copy_in) {
    KmbStageBuf *b;
    cudaError_t e;
    if (st->status) return NULL;
    if (!p) return NULL;
    b = stage_find(st, p);
    if (b) {
        if (bytes > b->bytes && b->owned) {
            st->status = kmb_fail(KMB_EINVAL, "staging: buffer %p reused with a larger size", p);
            return NULL;
        }
        b->out |= out;
        return b->dev;
    }
    if (st->n >= st->cap) {
        st->status = kmb_fail(KMB_EINVAL, "staging: too many buffers");
        return NULL;
    }
    b = &st->b[st->n++];
    b->user = p;
    b->bytes = bytes;
    b->out = out;
    {
        void *rd = resident_find(p, bytes);
        if (rd) { /* a device-resident host array: its device copy, no copies */
            b->dev = rd;
            b->owned = 0;
            return b->dev;
        }
    }
    if (kmb_is_device_ptr(p)) {
        b->dev = (void *)p;
        b->owned = 0;
        return b->dev;
    }
    b->owned = 1;
    b->dev = kmb_pool_alloc(bytes);
    if (!b->dev) {
        st->status = kmb_last_status() ? kmb_last_status() : KMB_ENOMEM;
        return NULL;
    }
    if (copy_in && bytes) {
        e = cudaMemcpyAsync(b->dev, p, bytes, cudaMemcpyHostToDevice, st->s);
        if (e != cudaSuccess) {
            st->status = kmb_cuda_fail(e, "staging host->device copy");
            return NULL;
        }
    }
    return b->dev;
}

void *kmb_stage_in(KmbStage *st, const void *p, size_t bytes) {
    return stage_add(st, p, bytes, 0, 1);
}

void *kmb_stage_out(KmbStage *st, void *p, size_t bytes, int copy_in) {
    return stage_add(st, p, bytes, 1, copy_in);
}

void *kmb_scratch(KmbStage *st, size_t bytes) {
    KmbStageBuf *b;
    if (st->status) return NULL;
    if (st->n >= st->cap) {
        st->status = kmb_fail(KMB_EINVAL, "staging: too many buffers");
        return NULL;
    }
    b = &st->b[st->n++];
    memset(b, 0, sizeof *b);
    b->owned = 1;
    b->bytes = bytes;
    b->dev = kmb_pool_alloc(bytes);
    if (!b->dev) {
        st->status = kmb_last_status() ? kmb_last_status() : KMB_ENOMEM;
        return NULL;
    }
    return b->dev;
}

int kmb_stage_finish(KmbStage *st, int status) {
    int any_owned = 0;
    cudaError_t e;
    if (!status) status = st->status;
    for (int i = 0; i < st->n; ++i) {
        KmbStageBuf *b = &st->b[i];
        if (!b->owned) continue;
        any_owned = 1;
        if (status == KMB_OK && b->out && b->user && b->bytes) {
            e = cudaMemcpyAsync((void *)b->user, b->dev, b->bytes, cudaMemcpyDeviceToHost, st->s);
            if (e != cudaSuccess) status = kmb_cuda_fail(e, "staging device->host copy");
        }
    }
    if (any_owned || kmb_sync_enabled()) {
        e = cudaStreamSynchronize(st->s);
        if (e != cudaSuccess && status == KMB_OK) status = kmb_cuda_fail(e, "stream synchronize");
    }
    for (int i = 0; i < st->n; ++i)
        if (st->b[i].owned) kmb_pool_free(st->b[i].dev);
    st->n = 0;
    if (st->b != st->inl) free(st->b);
    st->b = st->inl;
    st->cap = KMB_STAGE_MAX;
    return status;
}
