/*
 * ND / 2D selective scan entry points with stored states: the reference C
 * API (scan_nd.h, scan2d / mamba_scan2d_forward of scan.h, reference
 * src/scan_nd.c:17-308, cuda/scan_nd.cu:337-400, cpu/scan2d.asm) and the
 * batched kmb_scannd_* extension, routed to csrc/cuda/scannd.cu.
 */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../kmb_internal.h"
#include "mamba_scan_2d.h"
#include "mamba_scan_cuda.h"
#include "scan.h"
#include "scan_nd.h"
#include "wavefront_nd.h"

static void report(int status) {
    if (status != KMB_OK && status != KMB_EINVAL)
        fprintf(stderr, "kmamba_b200: %s\n", kmb_last_error());
}

static int validate(const KmbScanND *a, int bwd) {
    if (!a) return kmb_fail(KMB_EINVAL, "scannd: NULL arguments");
    if (a->ndims <= 0 || a->ndims > KMB_MAX_AXES)
        return kmb_fail(KMB_EINVAL, "scannd: ndims out of range");
    if (!wavefront_nd_validate_dims(a->dims, a->ndims) ||
        wavefront_nd_total_points(a->dims, a->ndims) <= 0)
        return kmb_fail(KMB_EINVAL, "scannd: invalid dims");
    if (a->batch <= 0 || a->D <= 0 || a->M <= 0)
        return kmb_fail(KMB_EINVAL, "scannd: batch, D and M must be positive");
    if (a->flags) return kmb_fail(KMB_EINVAL, "scannd: flags must be 0");
    if (!a->x || !a->delta || !a->A || !a->B || !a->C || !a->h)
        return kmb_fail(KMB_EINVAL, "scannd: x, delta, A, B, C and h are required");
    if (!bwd && !a->y) return kmb_fail(KMB_EINVAL, "scannd: y is required");
    if (bwd && (!a->dy || !a->dx || !a->ddelta || !a->dA || !a->dB || !a->dC))
        return kmb_fail(KMB_EINVAL, "scannd backward: dy and every gradient are required");
    return KMB_OK;
}

/* bf16 I/O (bf16 = 1): x, delta, B, C, y, dy, dx, ddelta, dB, dC are bf16
 * device tensors; A, dA and h stay fp32.  The 2D wavefront kernels read
 * and write bf16 directly (channel-shared B/C, M 8 or 16, D a multiple of
 * 8); other shapes are converted to fp32 scratch around the fp32 kernels
 * (run_bf16_converted). */
static int run(const KmbScanND *a, int bwd, int bf16) {
    KmbStage st;
    KmbNDLaunch L;
    KmbDevPlan plan;
    int rc = validate(a, bwd);
    long P, nd;
    size_t pd, pdm, bc, dn;
    float *delta_d, *dA_d, *ddelta_d;
    if (rc) return rc;
    nd = a->ndims;
    P = wavefront_nd_total_points(a->dims, nd);
    pd = sizeof(float) * (size_t)a->batch * P * a->D;
    pdm = pd * (size_t)a->M;
    bc = sizeof(float) * (size_t)a->batch * P * (a->bc_shared ? 1 : a->D) * a->M;
    dn = sizeof(float) * (size_t)nd * a->D * a->M;
    rc = kmb_dev_plan(a->dims, nd, &plan);
    if (rc) return rc;

    kmb_stage_begin(&st);
    memset(&L, 0, sizeof L);
    L.x = kmb_stage_in(&st, a->x, pd);
    delta_d = (float *)kmb_stage_in(&st, a->delta, pd * (size_t)nd);
    {
        const float *Ad = kmb_stage_in(&st, a->A, dn);
        for (long i = 0; i < nd; ++i) L.A[i] = Ad ? Ad + i * a->D * a->M : NULL;
    }
    L.B = kmb_stage_in(&st, a->B, bc);
    L.C = kmb_stage_in(&st, a->C, bc);
    if (!bwd) {
        L.h = kmb_stage_out(&st, a->h, pdm, 0);
        L.y = kmb_stage_out(&st, a->y, pd, 0);
    } else {
        L.h = (float *)kmb_stage_in(&st, a->h, pdm);
        L.dy = kmb_stage_in(&st, a->dy, pd);
        L.dx = kmb_stage_out(&st, a->dx, pd, 0);
        ddelta_d = kmb_stage_out(&st, a->ddelta, pd * (size_t)nd, 0);
        dA_d = kmb_stage_out(&st, a->dA, dn, 0);
        L.dB = kmb_stage_out(&st, a->dB, bc, 0);
        L.dC = kmb_stage_out(&st, a->dC, bc, 0);
        L.G = kmb_scratch(&st, pdm);
        for (long i = 0; i < nd; ++i) {
            /* bf16 tensors: the axes are P * D two-byte elements apart */
            L.ddelta[i] = ddelta_d ? (float *)((char *)ddelta_d + i * P * a->D * (bf16 ? 2 : 4))
                                   : NULL;
            L.dA[i] = dA_d ? dA_d + i * a->D * a->M : NULL;
        }
    }
    if (st.status) return kmb_stage_finish(&st, st.status);
    for (long i = 0; i < nd; ++i)
        L.delta[i] = (const float *)((const char *)delta_d + i * P * a->D * (bf16 ? 2 : 4));
    L.delta_bstride = nd * P * a->D;
    L.lvl_start = plan.lvl_start;
    L.lvl_off = plan.lvl_off;
    L.prev = plan.prev;
    L.next = plan.next;
    L.sprev = plan.sprev;
    L.snext = plan.snext;
    L.P = P;
    L.D = a->D;
    L.M = a->M;
    L.batch = a->batch;
    L.nd = (int)nd;
    L.nlevels = plan.nlevels;
    L.bc_shared = a->bc_shared;
    for (long i = 0; i < nd; ++i) L.dims[i] = a->dims[i];
    if (bf16) {
        /* the caller checked kmb_scan2d_bf16_supported */
        L.scratch_elems = kmb_scan2d_scratch_elems(&L);
        L.scratch = (float *)kmb_scratch(&st, sizeof(float) * L.scratch_elems);
        float *dB32 = bwd ? (float *)kmb_scratch(&st, bc) : NULL;
        float *dC32 = bwd ? (float *)kmb_scratch(&st, bc) : NULL;
        rc = st.status;
        if (!rc)
            rc = bwd ? kmb_launch_scan2d_bwd_bf16(&L, dB32, dC32, st.s)
                     : kmb_launch_scan2d_fwd_bf16(&L, st.s);
    } else if (kmb_scan2d_supported(&L)) {
        L.scratch_elems = kmb_scan2d_scratch_elems(&L);
        L.scratch = (float *)kmb_scratch(&st, sizeof(float) * L.scratch_elems);
        rc = st.status;
        if (!rc) rc = bwd ? kmb_launch_scan2d_bwd(&L, st.s) : kmb_launch_scan2d_fwd(&L, st.s);
    } else {
        rc = bwd ? kmb_launch_scannd_bwd(&L, st.s) : kmb_launch_scannd_fwd(&L, st.s);
        return kmb_stage_finish(&st, rc);
    }
    rc = kmb_stage_finish(&st, rc);
    /* the 2D kernels' bounded waits (strip split) report through a device
     * word, read when the call is synchronous */
    if (!rc && kmb_sync_enabled()) rc = kmb_scan2d_check_error();
    return rc;
}

int kmb_scannd_fwd(const KmbScanND *a) { return run(a, 0, 0); }
int kmb_scannd_bwd(const KmbScanND *a) { return run(a, 1, 0); }

/* ---------------- bf16 I/O variants -------------------------------- */

/* Shapes the 2D kernels take in bf16 directly. */
static int bf16_direct(const KmbScanND *a) {
    return a->ndims == 2 && a->bc_shared && a->M % 8 == 0 && a->M <= 16 && a->D % 8 == 0 &&
           a->D * a->M < (1L << 24);
}

/* Other shapes: every bf16 input converted into pooled fp32 scratch, the
 * fp32 kernels, the bf16 outputs converted back (round to nearest even). */
static int run_bf16_converted(const KmbScanND *a, int bwd) {
    const long nd = a->ndims, P = wavefront_nd_total_points(a->dims, nd);
    const size_t pd = (size_t)a->batch * P * a->D;
    const size_t bc = (size_t)a->batch * P * (a->bc_shared ? 1 : a->D) * a->M;
    struct { const void *src; void *dst; size_t n; int out; } t[10];
    int nt = 0, rc = KMB_OK;
    KmbScanND f = *a;
#define KMB_CONV(field, count, is_out) do { t[nt].src = a->field; t[nt].n = (count); \
        t[nt].out = (is_out); t[nt].dst = kmb_pool_alloc(sizeof(float) * (count)); \
        if (!t[nt].dst) { rc = kmb_fail(KMB_ENOMEM, "scannd bf16: scratch"); goto done; } \
        f.field = (float *)t[nt].dst; ++nt; } while (0)
    KMB_CONV(x, pd, 0);
    KMB_CONV(delta, pd * nd, 0);
    KMB_CONV(B, bc, 0);
    KMB_CONV(C, bc, 0);
    if (!bwd) {
        KMB_CONV(y, pd, 1);
    } else {
        KMB_CONV(dy, pd, 0);
        KMB_CONV(dx, pd, 1);
        KMB_CONV(ddelta, pd * nd, 1);
        KMB_CONV(dB, bc, 1);
        KMB_CONV(dC, bc, 1);
    }
#undef KMB_CONV
    for (int i = 0; i < nt && !rc; ++i)
        if (!t[i].out) rc = kmb_launch_bf16_to_f32(t[i].src, (float *)t[i].dst, (long)t[i].n, kmb_stream());
    if (!rc) {
        const int sync = kmb_sync_enabled();
        kmb_set_sync(0);
        rc = run(&f, bwd, 0);
        kmb_set_sync(sync);
    }
    for (int i = 0; i < nt && !rc; ++i)
        if (t[i].out)
            rc = kmb_launch_f32_to_bf16((const float *)t[i].dst, (void *)t[i].src, (long)t[i].n,
                                        kmb_stream());
    if (!rc && kmb_sync_enabled()) {
        cudaError_t e = cudaStreamSynchronize(kmb_stream());
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "scannd bf16: synchronize");
    }
done:
    for (int i = 0; i < nt; ++i) kmb_pool_free(t[i].dst);
    return rc;
}

static int run_bf16(const KmbScanND *a, int bwd) {
    int rc = validate(a, bwd);
    if (rc) return rc;
    const void *ptrs[] = {a->x, a->delta, a->A, a->B, a->C, a->h, a->y, a->dy, a->dx,
                          a->ddelta, a->dA, a->dB, a->dC};
    for (size_t i = 0; i < sizeof ptrs / sizeof ptrs[0]; ++i)
        if (ptrs[i] && !kmb_is_device_ptr(ptrs[i]))
            return kmb_fail(KMB_EINVAL, "scannd bf16: every tensor must be device memory");
    if (bf16_direct(a)) {
        const void *al[] = {a->x, a->delta, a->B, a->C, a->dy};
        for (size_t i = 0; i < sizeof al / sizeof al[0]; ++i)
            if (al[i] && ((uintptr_t)al[i] & 15u))
                return kmb_fail(KMB_EUNSUPPORTED, "scannd bf16: inputs must be 16-byte aligned");
        return run(a, bwd, 1);
    }
    return run_bf16_converted(a, bwd);
}

int kmb_scannd_fwd_bf16(const KmbScanND *a) {
    kmb_clear_error();
    const int rc = run_bf16(a, 0);
    report(rc);
    return rc;
}

int kmb_scannd_bwd_bf16(const KmbScanND *a) {
    kmb_clear_error();
    const int rc = run_bf16(a, 1);
    report(rc);
    return rc;
}

/* ------------------------------------------------------------------ */
/* reference API                                                       */
/* ------------------------------------------------------------------ */

/* src/scan_nd.c:17-29 */
int scannd_validate(const ScanNDParams *p) {
    if (!p || !p->dims) return 0;
    if (p->ndims <= 0 || p->D <= 0 || p->M <= 0) return 0;
    if (!p->x || !p->A || !p->B || !p->C || !p->delta || !p->h || !p->y) return 0;
    if (!wavefront_nd_validate_dims(p->dims, p->ndims)) return 0;
    if (wavefront_nd_total_points(p->dims, p->ndims) <= 0) return 0;
    return 1;
}

static int scannd_gpu(ScanNDParams *p) {
    KmbScanND a;
    int rc;
    if (!scannd_validate(p)) return -1;
    /* The Mamba-3 exp-trapezoidal branch (lambda != NULL) is not part of
     * this library; theta alone has no effect in the reference. */
    if (p->lambda) {
        kmb_fail(KMB_EUNSUPPORTED, "scannd: lambda (exp-trapezoidal) is not supported");
        return -1;
    }
    if (p->ndims > KMB_MAX_AXES) return -1;
    memset(&a, 0, sizeof a);
    for (long i = 0; i < p->ndims; ++i) a.dims[i] = p->dims[i];
    a.ndims = p->ndims;
    a.batch = 1;
    a.D = p->D;
    a.M = p->M;
    a.x = p->x;
    a.delta = p->delta;
    a.A = p->A;
    a.B = p->B;
    a.C = p->C;
    a.h = p->h;
    a.y = p->y;
    rc = kmb_scannd_fwd(&a);
    report(rc);
    return rc == KMB_OK ? 0 : -1;
}

int scannd_ref(ScanNDParams *p) { return scannd_gpu(p); }

int scannd_ref_with_plan(ScanNDParams *p, const KMWavefrontPlan *plan) {
    if (!scannd_validate(p)) return -1;
    if (!km_wavefront_plan_matches_dims(plan, p->dims, p->ndims)) return -1;
    return scannd_gpu(p);
}

/* src/scan_nd.c:249-308: every dimension runs on the GPU. */
int scannd(ScanNDParams *p) { return scannd_gpu(p); }

int om_scannd_forward(ScanNDParams *p) { return scannd_gpu(p); }

int mamba_scannd_cuda_forward(ScanNDParams *p) { return om_scannd_forward(p); }

/* cpu/scan2d.asm:48-285: h [P,D,M] and y [P,D] are written in full. */
void scan2d(Scan2DParams *p) {
    KmbStage st;
    KmbNDLaunch L;
    KmbDevPlan plan;
    long dims[2], P;
    size_t pd, pdm, dm;
    int rc;
    if (!p || !p->x || !p->A1 || !p->A2 || !p->B || !p->C || !p->delta1 || !p->delta2 ||
        !p->h || !p->y || p->d1 <= 0 || p->d2 <= 0 || p->D <= 0 || p->M <= 0)
        return;
    dims[0] = p->d1;
    dims[1] = p->d2;
    P = wavefront_nd_total_points(dims, 2);
    if (P <= 0) return;
    rc = kmb_dev_plan(dims, 2, &plan);
    if (rc) {
        report(rc);
        return;
    }
    pd = sizeof(float) * (size_t)P * p->D;
    pdm = pd * (size_t)p->M;
    dm = sizeof(float) * (size_t)p->D * p->M;
    kmb_stage_begin(&st);
    memset(&L, 0, sizeof L);
    L.x = kmb_stage_in(&st, p->x, pd);
    L.A[0] = kmb_stage_in(&st, p->A1, dm);
    L.A[1] = kmb_stage_in(&st, p->A2, dm);
    L.B = kmb_stage_in(&st, p->B, pdm);
    L.C = kmb_stage_in(&st, p->C, pdm);
    L.delta[0] = kmb_stage_in(&st, p->delta1, pd);
    L.delta[1] = kmb_stage_in(&st, p->delta2, pd);
    L.h = kmb_stage_out(&st, p->h, pdm, 0);
    L.y = kmb_stage_out(&st, p->y, pd, 0);
    rc = st.status;
    if (!rc) {
        L.lvl_start = plan.lvl_start;
        L.lvl_off = plan.lvl_off;
        L.prev = plan.prev;
        L.next = plan.next;
        L.sprev = plan.sprev;
        L.snext = plan.snext;
        L.P = P;
        L.D = p->D;
        L.M = p->M;
        L.batch = 1;
        L.nd = 2;
        L.nlevels = plan.nlevels;
        L.delta_bstride = 0;
        rc = kmb_launch_scannd_fwd(&L, st.s);
    }
    rc = kmb_stage_finish(&st, rc);
    report(rc);
}

void mamba_scan2d_forward(MambaScan2DParams *p) { scan2d(p); }
