/*
 * kmb_scan1d_bwd_noalloc: the 1D selective-scan backward for callers that
 * must not allocate device memory during the call.
 *
 * The backward needs the forward states at every KMB_SCAN1D_CHUNK-th step
 * (checkpoints).  kmb_scan1d_bwd takes them from the caller or allocates a
 * scratch buffer from the library pool; this entry point instead keeps
 * them in the file-scope device array below, of fixed size
 * KMB_NOALLOC_CKPT_ELEMS floats, which every GPU that loads the library
 * holds until the process exits.  It calls no cudaMalloc / cudaFree and no
 * allocating routine, and stages nothing: every tensor must already be in
 * device memory.
 *
 * In host code the array's name only stands for the symbol; its device
 * address is looked up once per device with cudaGetSymbolAddress (with
 * that device current) by the first call on that device, and cached.  With
 * lazy module loading (the CUDA 12 default) that first lookup is also what
 * loads this module onto the device, allocating the array and possibly
 * synchronising: callers make their first call during their own set-up
 * phase.  The cached address is not refreshed after cudaDeviceReset, so
 * the entry point must not be used across a reset.
 *
 * All calls share the array and it keeps the last call's contents: every
 * checkpoint a call reads is written earlier in the same call, so nothing
 * needs clearing, but calls that overlap on the GPU (two streams, two host
 * threads on one device) race on it.
 */
#include <pthread.h>

#include "kmb_common.cuh"
#include "../kmb_internal.h"

static __device__ __align__(256) float g_noalloc_ckpt[KMB_NOALLOC_CKPT_ELEMS];

namespace {

constexpr int kMaxDevices = 64;
pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
float *g_addr[kMaxDevices]; /* device address of g_noalloc_ckpt per device */

/* Device address of the scratch array on the current device (set-up on
 * the first call per device). */
int scratch_address(float **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return kmb_fail(KMB_EUNSUPPORTED, "scan1d noalloc: device %d out of range", dev);
    pthread_mutex_lock(&g_mu);
    if (!g_addr[dev]) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_ckpt);
        if (e != cudaSuccess) {
            pthread_mutex_unlock(&g_mu);
            return kmb_cuda_fail(e, "scan1d noalloc: cudaGetSymbolAddress");
        }
        g_addr[dev] = static_cast<float *>(ptr);
    }
    *out = g_addr[dev];
    pthread_mutex_unlock(&g_mu);
    return KMB_OK;
}

/* NULL, or device (or managed) memory of the current device: memory of
 * another GPU would be read over the peer link, or fault without peer
 * access. */
bool on_device(const void *p, int dev) {
    if (!p) return true;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    if (at.type == cudaMemoryTypeManaged) return true;
    return at.type == cudaMemoryTypeDevice && at.device == dev;
}

} // namespace

extern "C" int kmb_scan1d_bwd_noalloc(const KmbScan1D *a) {
    if (!a) return kmb_fail(KMB_EINVAL, "scan1d noalloc: NULL arguments");
    if (a->batch <= 0 || a->L <= 0 || a->D <= 0 || a->N <= 0)
        return kmb_fail(KMB_EINVAL, "scan1d noalloc: sizes must be positive");
    if (a->N > 128) return kmb_fail(KMB_EUNSUPPORTED, "scan1d noalloc: N=%ld exceeds 128", a->N);
    if (a->flags != 0) return kmb_fail(KMB_EINVAL, "scan1d noalloc: flags must be 0");
    if (!a->x || !a->dt || !a->A || !a->B || !a->C || !a->dy || !a->dx || !a->ddt || !a->dA ||
        !a->dB || !a->dC)
        return kmb_fail(KMB_EINVAL, "scan1d noalloc: x, dt, A, B, C, dy and every gradient "
                                    "are required");
    if (a->h_all || a->ckpt)
        return kmb_fail(KMB_EINVAL, "scan1d noalloc: h_all / ckpt must be NULL (the "
                                    "checkpoints are kept in the library's static scratch)");
    const long need = kmb_scan1d_ckpt_elems(a->batch, a->L, a->D, a->N);
    if (need > (long)KMB_NOALLOC_CKPT_ELEMS)
        return kmb_fail(KMB_EUNSUPPORTED,
                        "scan1d noalloc: needs %ld checkpoint floats, the static scratch holds "
                        "%ld (batch * ceil(L/%d) * D * N must not exceed it)",
                        need, (long)KMB_NOALLOC_CKPT_ELEMS, KMB_SCAN1D_CHUNK);
    int cur = 0;
    const cudaError_t de = cudaGetDevice(&cur);
    if (de != cudaSuccess) return kmb_cuda_fail(de, "scan1d noalloc: cudaGetDevice");
    const void *ptrs[] = {a->x, a->dt, a->A, a->B, a->C, a->h0, a->dy,
                          a->dx, a->ddt, a->dA, a->dB, a->dC};
    for (const void *q : ptrs)
        if (!on_device(q, cur))
            return kmb_fail(KMB_EINVAL, "scan1d noalloc: every tensor must be device memory "
                                        "of the current device (host buffers would need "
                                        "staging allocations)");
    kmb_clear_error();

    float *ck = nullptr;
    int rc = scratch_address(&ck);
    if (rc) return rc;
    const cudaStream_t s = kmb_stream();

    KmbScan1D f = *a;     /* forward pass that only writes the checkpoints */
    f.ckpt = ck;
    f.y = nullptr;
    f.h_last = nullptr;
    f.h_all = nullptr;
    rc = kmb_launch_scan1d_fwd(&f, s);
    if (rc) return rc;
    rc = kmb_launch_scan1d_bwd(a, ck, s);
    if (rc) return rc;
    if (kmb_sync_enabled()) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return kmb_cuda_fail(e, "scan1d noalloc: stream synchronize");
    }
    return KMB_OK;
}
