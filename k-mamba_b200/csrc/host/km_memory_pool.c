/*
 * km_memory_pool.h over device memory.
 *
 * A KMMemoryPool is a growable table of chunks {device pointer, size,
 * in use}.  Chunks come from kmb_pool_alloc (the library's per-device
 * cache of cudaMalloc blocks, csrc/host/runtime.c), so destroying a pool
 * and creating another reuses the same device blocks without new
 * cudaMalloc calls.  A pool is meant for one thread at a time, as in the
 * reference; the registry of thread-local pools is guarded by a mutex.
 */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "km_memory_pool.h"
#include "../kmb_internal.h"

typedef struct {
    void *ptr;
    size_t size;
    int in_use;
} KmChunk;

struct KMMemoryPool {
    KmChunk *chunk;
    size_t count;
    size_t cap;
    struct KMMemoryPool *next_tl; /* registry link (thread-local pools) */
};

KMMemoryPool *km_memory_pool_create(void) {
    KMMemoryPool *pool = (KMMemoryPool *)calloc(1, sizeof *pool);
    if (!pool) return NULL;
    pool->cap = 16;
    pool->chunk = (KmChunk *)calloc(pool->cap, sizeof *pool->chunk);
    if (!pool->chunk) {
        free(pool);
        return NULL;
    }
    return pool;
}

void km_memory_pool_destroy(KMMemoryPool *pool) {
    if (!pool) return;
    for (size_t i = 0; i < pool->count; ++i) kmb_pool_free(pool->chunk[i].ptr);
    free(pool->chunk);
    free(pool);
}

void *km_pool_alloc(KMMemoryPool *pool, size_t size) {
    if (!pool || size == 0) return NULL;
    for (size_t i = 0; i < pool->count; ++i) {
        KmChunk *c = &pool->chunk[i];
        if (!c->in_use && c->size >= size) {
            c->in_use = 1;
            return c->ptr;
        }
    }
    if (pool->count == pool->cap) {
        KmChunk *grown = (KmChunk *)realloc(pool->chunk, 2 * pool->cap * sizeof *grown);
        if (!grown) {
            kmb_fail(KMB_ENOMEM, "km_pool_alloc: host allocation failed");
            return NULL;
        }
        pool->chunk = grown;
        pool->cap *= 2;
    }
    void *dev = kmb_pool_alloc(size);
    if (!dev) return NULL; /* kmb_pool_alloc recorded the reason */
    pool->chunk[pool->count++] = (KmChunk){dev, size, 1};
    return dev;
}

void km_pool_free(KMMemoryPool *pool, void *ptr) {
    if (!pool || !ptr) return;
    for (size_t i = 0; i < pool->count; ++i) {
        if (pool->chunk[i].ptr == ptr) {
            pool->chunk[i].in_use = 0;
            return;
        }
    }
}

void km_pool_clear(KMMemoryPool *pool) {
    if (!pool) return;
    for (size_t i = 0; i < pool->count; ++i) pool->chunk[i].in_use = 0;
}

/* Thread-local pools: each thread caches its pool together with the
 * registry generation it was created in; destroy_all bumps the
 * generation, so a thread never touches a pool that was destroyed. */
static pthread_mutex_t g_tl_mu = PTHREAD_MUTEX_INITIALIZER;
static KMMemoryPool *g_tl_head;
static unsigned long g_tl_gen = 1;
static __thread KMMemoryPool *t_pool;
static __thread unsigned long t_gen;

KMMemoryPool *km_memory_pool_threadlocal(void) {
    pthread_mutex_lock(&g_tl_mu);
    if (!t_pool || t_gen != g_tl_gen) {
        t_pool = km_memory_pool_create();
        t_gen = g_tl_gen;
        if (t_pool) {
            t_pool->next_tl = g_tl_head;
            g_tl_head = t_pool;
        }
    }
    KMMemoryPool *p = t_pool;
    pthread_mutex_unlock(&g_tl_mu);
    return p;
}

void km_memory_pool_destroy_all_threadlocal(void) {
    pthread_mutex_lock(&g_tl_mu);
    KMMemoryPool *p = g_tl_head;
    g_tl_head = NULL;
    ++g_tl_gen;
    t_pool = NULL;
    pthread_mutex_unlock(&g_tl_mu);
    while (p) {
        KMMemoryPool *next = p->next_tl;
        km_memory_pool_destroy(p);
        p = next;
    }
}
