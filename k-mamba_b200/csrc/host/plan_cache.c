/*
 * Device-resident wavefront schedules, cached per (device, grid shape).
 *
 * Built from km_wavefront_plan_create (levels and their row-major
 * offsets) plus, per point and axis, the offset of the predecessor
 * p - e_axis and of the successor p + e_axis (-1 outside the grid).  The
 * reference rebuilds and re-uploads its schedule on every call
 * (cuda/scan_nd.cu:183-258, 337-400); here it is uploaded once.
 */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "../kmb_internal.h"
#include "km_topology.h"
#include "wavefront_plan.h"

#define KMB_PLAN_SLOTS 16

typedef struct {
    int used;
    int device;
    long nd;
    long dims[KMB_MAX_AXES];
    int *buf; /* device: starts | offsets | prev | next */
    KmbDevPlan plan;
    unsigned long stamp;
} PlanSlot;

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static PlanSlot g_slots[KMB_PLAN_SLOTS];
static unsigned long g_clock;

static int same(const PlanSlot *s, int dev, const long *dims, long nd) {
    if (!s->used || s->device != dev || s->nd != nd) return 0;
    for (long i = 0; i < nd; ++i)
        if (s->dims[i] != dims[i]) return 0;
    return 1;
}

static int build(const long *dims, long nd, PlanSlot *slot) {
    KMWavefrontPlan *pl = km_wavefront_plan_create(dims, nd);
    long strides[KMB_MAX_AXES];
    int *host;
    size_t n_st, n_off, n_pn, total;
    cudaError_t e;

    if (!pl) return kmb_fail(KMB_EINVAL, "scannd: invalid grid");
    if (pl->total_points > 0x7fffffffL || pl->max_level + 2 > 0x7fffffffL) {
        km_wavefront_plan_free(pl);
        return kmb_fail(KMB_EUNSUPPORTED, "scannd: grid exceeds 2^31 points");
    }
    km_make_row_major_strides(dims, nd, strides);
    n_st = (size_t)pl->max_level + 2;
    n_off = (size_t)pl->total_points;
    n_pn = (size_t)pl->total_points * (size_t)nd;
    total = n_st + n_off + 4 * n_pn;
    host = (int *)malloc(total * sizeof(int));
    if (!host) {
        km_wavefront_plan_free(pl);
        return kmb_fail(KMB_ENOMEM, "scannd: host allocation failed");
    }
    for (size_t i = 0; i < n_st; ++i) host[i] = (int)pl->level_starts[i];
    for (size_t i = 0; i < n_off; ++i) host[n_st + i] = (int)pl->level_offsets[i];
    {
        int *prev = host + n_st + n_off;
        int *next = prev + n_pn;
        long co[KMB_MAX_AXES];
        for (long p = 0; p < pl->total_points; ++p) {
            km_unravel_index(p, dims, strides, nd, co);
            for (long a = 0; a < nd; ++a) {
                prev[p * nd + a] = co[a] > 0 ? (int)(p - strides[a]) : -1;
                next[p * nd + a] = co[a] + 1 < dims[a] ? (int)(p + strides[a]) : -1;
            }
        }
        /* the same tables in level-slot order, so a kernel reading slot s
         * gets a point's neighbours without first loading its offset */
        int *sprev = next + n_pn;
        int *snext = sprev + n_pn;
        const int *off = host + n_st;
        for (size_t s = 0; s < n_off; ++s)
            for (long a = 0; a < nd; ++a) {
                sprev[s * nd + a] = prev[(size_t)off[s] * nd + a];
                snext[s * nd + a] = next[(size_t)off[s] * nd + a];
            }
    }
    e = cudaMalloc((void **)&slot->buf, total * sizeof(int));
    if (e == cudaSuccess)
        e = cudaMemcpy(slot->buf, host, total * sizeof(int), cudaMemcpyHostToDevice);
    free(host);
    if (e != cudaSuccess) {
        if (slot->buf) cudaFree(slot->buf);
        slot->buf = NULL;
        km_wavefront_plan_free(pl);
        return kmb_cuda_fail(e, "scannd: schedule upload");
    }
    slot->plan.lvl_start = slot->buf;
    slot->plan.lvl_off = slot->buf + n_st;
    slot->plan.prev = slot->buf + n_st + n_off;
    slot->plan.next = slot->buf + n_st + n_off + n_pn;
    slot->plan.sprev = slot->buf + n_st + n_off + 2 * n_pn;
    slot->plan.snext = slot->buf + n_st + n_off + 3 * n_pn;
    slot->plan.P = pl->total_points;
    slot->plan.nlevels = (int)(pl->max_level + 1);
    slot->plan.nd = (int)nd;
    km_wavefront_plan_free(pl);
    return KMB_OK;
}

int kmb_dev_plan(const long *dims, long nd, KmbDevPlan *out) {
    int dev = 0, rc;
    PlanSlot *victim = NULL;
    if (nd <= 0 || nd > KMB_MAX_AXES) return kmb_fail(KMB_EINVAL, "scannd: ndims out of range");
    if (cudaGetDevice(&dev) != cudaSuccess) {
        (void)cudaGetLastError();
        return kmb_fail(KMB_ECUDA, "scannd: no CUDA device");
    }
    pthread_mutex_lock(&g_mu);
    for (int i = 0; i < KMB_PLAN_SLOTS; ++i) {
        if (same(&g_slots[i], dev, dims, nd)) {
            g_slots[i].stamp = ++g_clock;
            *out = g_slots[i].plan;
            pthread_mutex_unlock(&g_mu);
            return KMB_OK;
        }
    }
    for (int i = 0; i < KMB_PLAN_SLOTS; ++i) {
        if (!g_slots[i].used) { victim = &g_slots[i]; break; }
        if (!victim || g_slots[i].stamp < victim->stamp) victim = &g_slots[i];
    }
    if (victim->used) {
        /* the evicted schedule may still be read by queued kernels */
        cudaDeviceSynchronize();
        cudaFree(victim->buf);
        victim->used = 0;
    }
    memset(victim, 0, sizeof *victim);
    rc = build(dims, nd, victim);
    if (rc == KMB_OK) {
        victim->used = 1;
        victim->device = dev;
        victim->nd = nd;
        memcpy(victim->dims, dims, sizeof(long) * (size_t)nd);
        victim->stamp = ++g_clock;
        *out = victim->plan;
    }
    pthread_mutex_unlock(&g_mu);
    return rc;
}
