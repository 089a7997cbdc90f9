#ifndef KM_MEMORY_POOL_H
#define KM_MEMORY_POOL_H

/*
 * Reusable scratch buffers, with the names and contracts of the reference
 * include/km_memory_pool.h (implementation src/km_memory_pool.c:28-178),
 * redone for device memory: km_pool_alloc returns DEVICE memory of the
 * current CUDA device, carved from the library's device pool
 * (kmb_pool_alloc in kmamba_b200.h).  The reference hands out host
 * memory; a caller that passes the buffers to this library's entry points
 * gets them used in place instead of staged.
 *
 * Reuse follows the reference: a request takes the first free chunk of the
 * pool whose size is at least the request, else a new chunk is added.
 * km_pool_free / km_pool_clear only mark chunks free; memory goes back to
 * the library pool when the KMMemoryPool is destroyed.
 *
 * Thread-local pools are keyed by the calling host thread.  (The
 * reference keys them by omp_get_thread_num(), which is 0 on every thread
 * that is not an OpenMP worker, so plain threads share one unsynchronised
 * pool there.)
 */

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct KMMemoryPool KMMemoryPool;

/* NULL when the host allocation of the pool's bookkeeping fails. */
KMMemoryPool *km_memory_pool_create(void);
/* Returns every chunk to the library's device pool.  NULL is ignored. */
void km_memory_pool_destroy(KMMemoryPool *pool);

/* Device pointer of at least `size` bytes (256-byte aligned), or NULL for
 * a NULL pool, size 0 or a failed allocation (kmb_last_error() says why). */
void *km_pool_alloc(KMMemoryPool *pool, size_t size);
/* Marks the chunk starting at ptr free; other pointers are ignored. */
void km_pool_free(KMMemoryPool *pool, void *ptr);
/* Marks every chunk free, keeping the capacity. */
void km_pool_clear(KMMemoryPool *pool);

/* The calling thread's pool, created on first use (NULL if that fails). */
KMMemoryPool *km_memory_pool_threadlocal(void);
/* Destroys the thread-local pools of every thread; a thread's next
 * km_memory_pool_threadlocal() creates a fresh one. */
void km_memory_pool_destroy_all_threadlocal(void);

#ifdef __cplusplus
}
#endif

#endif /* KM_MEMORY_POOL_H */
