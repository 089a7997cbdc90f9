/*
 * 1D selective scan entry points: the reference C API (include/scan.h,
 * include/mamba_scan.h, include/mamba_scan_cuda.h of k-mamba) and the
 * batched kmb_scan1d_* extension, all routed to the sm_100a kernels in
 * csrc/cuda/scan1d.cu.
 */
#include <stdio.h>
#include <string.h>

#include "../kmb_internal.h"
#include "scan.h"
#include "mamba_scan.h"
#include "mamba_scan_cuda.h"

static void report(int status) {
    if (status != KMB_OK && status != KMB_EINVAL)
        fprintf(stderr, "kmamba_b200: %s\n", kmb_last_error());
}

long kmb_scan1d_ckpt_elems(long batch, long L, long D, long N) {
    if (batch <= 0 || L <= 0 || D <= 0 || N <= 0) return 0;
    return batch * ((L + KMB_SCAN1D_CHUNK - 1) / KMB_SCAN1D_CHUNK) * D * N;
}

static int validate_common(const KmbScan1D *a) {
    if (!a) return kmb_fail(KMB_EINVAL, "scan1d: NULL arguments");
    if (a->batch <= 0 || a->L <= 0 || a->D <= 0 || a->N <= 0)
        return kmb_fail(KMB_EINVAL, "scan1d: sizes must be positive");
    if (a->N > 128) return kmb_fail(KMB_EUNSUPPORTED, "scan1d: N=%ld exceeds 128", a->N);
    if (!a->x || !a->dt || !a->A || !a->B || !a->C)
        return kmb_fail(KMB_EINVAL, "scan1d: x, dt, A, B and C are required");
    if (a->flags != 0) return kmb_fail(KMB_EINVAL, "scan1d: flags must be 0");
    return KMB_OK;
}

/* Stages every tensor of a KmbScan1D and fills `d` with device pointers. */
static void stage_args(KmbStage *st, const KmbScan1D *a, KmbScan1D *d, int bwd) {
    const size_t e_ld = sizeof(float) * (size_t)a->batch * a->L * a->D;
    const size_t e_bc = sizeof(float) * (size_t)a->batch * a->L * (a->bc_shared ? 1 : a->D) * a->N;
    const size_t e_dn = sizeof(float) * (size_t)a->D * a->N;
    const size_t e_st = sizeof(float) * (size_t)a->batch * a->D * a->N;
    const size_t e_all = sizeof(float) * (size_t)a->batch * a->L * a->D * a->N;
    const size_t e_ck = sizeof(float) * (size_t)kmb_scan1d_ckpt_elems(a->batch, a->L, a->D, a->N);

    *d = *a;
    d->x = kmb_stage_in(st, a->x, e_ld);
    d->dt = kmb_stage_in(st, a->dt, e_ld);
    d->A = kmb_stage_in(st, a->A, e_dn);
    d->B = kmb_stage_in(st, a->B, e_bc);
    d->C = kmb_stage_in(st, a->C, e_bc);
    /* h0 and h_last may alias (in/out running state): stage h_last first so
     * the shared device buffer is created as an output with copy-in. */
    if (!bwd && a->h_last) d->h_last = kmb_stage_out(st, a->h_last, e_st, a->h_last == a->h0);
    d->h0 = kmb_stage_in(st, a->h0, e_st);
    if (!bwd) {
        d->y = kmb_stage_out(st, a->y, e_ld, 0);
        d->h_all = kmb_stage_out(st, a->h_all, e_all, 0);
        d->ckpt = kmb_stage_out(st, a->ckpt, e_ck, 0);
    } else {
        d->h_all = (float *)kmb_stage_in(st, a->h_all, e_all);
        d->ckpt = (float *)kmb_stage_in(st, a->ckpt, e_ck);
        d->dy = kmb_stage_in(st, a->dy, e_ld);
        d->dx = kmb_stage_out(st, a->dx, e_ld, 0);
        d->ddt = kmb_stage_out(st, a->ddt, e_ld, 0);
        d->dA = kmb_stage_out(st, a->dA, e_dn, 0);
        d->dB = kmb_stage_out(st, a->dB, e_bc, 0);
        d->dC = kmb_stage_out(st, a->dC, e_bc, 0);
        d->y = NULL;
        d->h_last = NULL;
    }
}

int kmb_scan1d_fwd(const KmbScan1D *a) {
    KmbStage st;
    KmbScan1D d;
    int rc = validate_common(a);
    if (rc) return rc;
    kmb_stage_begin(&st);
    stage_args(&st, a, &d, 0);
    if (st.status) return kmb_stage_finish(&st, st.status);
    rc = kmb_launch_scan1d_fwd(&d, st.s);
    return kmb_stage_finish(&st, rc);
}

int kmb_scan1d_bwd(const KmbScan1D *a) {
    KmbStage st;
    KmbScan1D d;
    const float *ck;
    int rc = validate_common(a);
    if (rc) return rc;
    if (!a->dy || !a->dx || !a->ddt || !a->dA || !a->dB || !a->dC)
        return kmb_fail(KMB_EINVAL, "scan1d backward: dy and every gradient are required");
    kmb_stage_begin(&st);
    stage_args(&st, a, &d, 1);
    if (st.status) return kmb_stage_finish(&st, st.status);
    ck = d.ckpt;
    if (!d.h_all && !ck) {
        /* No stored states: run the forward once to produce checkpoints. */
        KmbScan1D f = d;
        f.ckpt = (float *)kmb_scratch(
            &st, sizeof(float) * (size_t)kmb_scan1d_ckpt_elems(a->batch, a->L, a->D, a->N));
        if (!f.ckpt) return kmb_stage_finish(&st, st.status);
        f.y = NULL;
        f.h_all = NULL;
        f.h_last = NULL;
        rc = kmb_launch_scan1d_fwd(&f, st.s);
        if (rc) return kmb_stage_finish(&st, rc);
        ck = f.ckpt;
    }
    rc = kmb_launch_scan1d_bwd(&d, ck, st.s);
    return kmb_stage_finish(&st, rc);
}

/* ------------------------------------------------------------------ */
/* reference API                                                       */
/* ------------------------------------------------------------------ */

/* cpu/scan1d.asm:40-179: h [D,M] is the running state (read, then
 * overwritten with the final state); y [L,D] is overwritten; clamp. */
void scan1d(ScanParams *p) {
    KmbScan1D a;
    int rc;
    if (!p || !p->x || !p->A || !p->B || !p->C || !p->delta || !p->h || !p->y) return;
    if (p->L <= 0 || p->D <= 0 || p->M <= 0) return;
    memset(&a, 0, sizeof a);
    a.x = p->x; a.dt = p->delta; a.A = p->A; a.B = p->B; a.C = p->C;
    a.h0 = p->h; a.h_last = p->h; a.y = p->y;
    a.batch = 1; a.L = p->L; a.D = p->D; a.N = p->M;
    a.bc_shared = 0;
    a.clamp = 1;
    rc = kmb_scan1d_fwd(&a);
    report(rc);
}

/* cpu/scan1d_backward.c:297-306 (generic and M = 1 paths). */
void scan1d_backward(ScanBackwardParams *p) {
    KmbScan1D a;
    int rc;
    if (!p || !p->x || !p->A || !p->B || !p->C || !p->delta || !p->h || !p->dy ||
        !p->dx || !p->dA || !p->dB || !p->dC || !p->ddelta || p->L <= 0 || p->D <= 0 ||
        p->M <= 0)
        return;
    memset(&a, 0, sizeof a);
    a.x = p->x; a.dt = p->delta; a.A = p->A; a.B = p->B; a.C = p->C;
    a.h0 = p->h0; a.h_all = p->h; a.dy = p->dy;
    a.dx = p->dx; a.ddt = p->ddelta; a.dA = p->dA; a.dB = p->dB; a.dC = p->dC;
    a.batch = 1; a.L = p->L; a.D = p->D; a.N = p->M;
    rc = kmb_scan1d_bwd(&a);
    report(rc);
}

/* cpu/scan1d_backward.c:173-191: M = 1, per-channel A/B/C, per-step delta. */
void scan1d_backward_m1_shared_bc(ScanBackwardSharedParams *p) {
    KmbStage st;
    int rc;
    size_t ld, l1, d1;
    if (!p || !p->x || !p->A || !p->B || !p->C || !p->delta || !p->h || !p->dy || !p->dx ||
        !p->dA || !p->dB || !p->dC || !p->ddelta || p->L <= 0 || p->D <= 0)
        return;
    ld = sizeof(float) * (size_t)p->L * p->D;
    l1 = sizeof(float) * (size_t)p->L;
    d1 = sizeof(float) * (size_t)p->D;
    kmb_stage_begin(&st);
    {
        const float *x = kmb_stage_in(&st, p->x, ld);
        const float *A = kmb_stage_in(&st, p->A, d1);
        const float *Ad = kmb_stage_in(&st, p->A_diag, ld);
        const float *B = kmb_stage_in(&st, p->B, d1);
        const float *C = kmb_stage_in(&st, p->C, d1);
        const float *dl = kmb_stage_in(&st, p->delta, l1);
        const float *h0 = kmb_stage_in(&st, p->h0, d1);
        const float *h = kmb_stage_in(&st, p->h, ld);
        const float *dy = kmb_stage_in(&st, p->dy, ld);
        float *dx = kmb_stage_out(&st, p->dx, ld, 0);
        float *dA = kmb_stage_out(&st, p->dA, d1, 0);
        float *dB = kmb_stage_out(&st, p->dB, d1, 0);
        float *dC = kmb_stage_out(&st, p->dC, d1, 0);
        float *ddl = kmb_stage_out(&st, p->ddelta, l1, 0);
        rc = st.status;
        if (!rc)
            rc = kmb_launch_scan1d_bwd_m1_shared(x, A, Ad, B, C, dl, h0, h, dy, dx, dA, dB, dC,
                                                 ddl, p->L, p->D, st.s);
    }
    rc = kmb_stage_finish(&st, rc);
    report(rc);
}

/* The reference declares assembly variants of the M = 1 backward
 * (cpu/scan1d_backward_m1_shared_bc*.asm); they compute the same gradients
 * and share the GPU kernel here. */
void scan1d_backward_m1_shared_bc_asm(ScanBackwardSharedParams *p) {
    scan1d_backward_m1_shared_bc(p);
}

void scan1d_backward_m1_shared_bc_simple_asm(ScanBackwardSharedParams *p) {
    scan1d_backward_m1_shared_bc(p);
}

/* cuda/scan1d.cu:258-310: device pointers, h is the full [L,D,M] history
 * from a zero initial state, y overwritten, states clamped. */
void om_scan1d_forward(const float *d_x, const float *d_A, const float *d_B,
                       const float *d_C, const float *d_dt, float *d_y, float *d_h,
                       int L, int D, int M) {
    KmbScan1D a;
    if (!d_x || !d_A || !d_B || !d_C || !d_dt || !d_y || !d_h || L <= 0 || D <= 0 || M <= 0)
        return;
    memset(&a, 0, sizeof a);
    a.x = d_x; a.dt = d_dt; a.A = d_A; a.B = d_B; a.C = d_C;
    a.y = d_y; a.h_all = d_h;
    a.batch = 1; a.L = L; a.D = D; a.N = M;
    a.clamp = 1;
    report(kmb_scan1d_fwd(&a));
}

/* cuda/scan1d_backward.cu:113-137. */
void om_scan1d_backward(const float *d_dy, const float *d_x, const float *d_A,
                        const float *d_B, const float *d_C, const float *d_dt,
                        const float *d_h, float *d_dx, float *d_dA, float *d_dB,
                        float *d_dC, float *d_ddt, int L, int D, int M) {
    KmbScan1D a;
    if (!d_dy || !d_x || !d_A || !d_B || !d_C || !d_dt || !d_h || !d_dx || !d_dA || !d_dB ||
        !d_dC || !d_ddt || L <= 0 || D <= 0 || M <= 0)
        return;
    memset(&a, 0, sizeof a);
    a.x = d_x; a.dt = d_dt; a.A = d_A; a.B = d_B; a.C = d_C;
    a.h_all = (float *)d_h; a.dy = d_dy;
    a.dx = d_dx; a.ddt = d_ddt; a.dA = d_dA; a.dB = d_dB; a.dC = d_dC;
    a.batch = 1; a.L = L; a.D = D; a.N = M;
    report(kmb_scan1d_bwd(&a));
}

/* cpu/mamba_scan.c:8-22 and cuda/mamba_scan.cu:8-37 aliases. */
void mamba_scan1d_forward(MambaScan1DParams *p) { scan1d(p); }
void mamba_scan1d_backward(MambaScan1DBackwardParams *p) { scan1d_backward(p); }
void mamba_scan1d_backward_m1_shared_bc(MambaScan1DBackwardM1Params *p) {
    scan1d_backward_m1_shared_bc(p);
}

void mamba_scan1d_cuda_forward(const float *d_x, const float *d_A, const float *d_B,
                               const float *d_C, const float *d_dt, float *d_y, float *d_h,
                               int L, int D, int M) {
    om_scan1d_forward(d_x, d_A, d_B, d_C, d_dt, d_y, d_h, L, D, M);
}

void mamba_scan1d_cuda_backward(const float *d_dy, const float *d_x, const float *d_A,
                                const float *d_B, const float *d_C, const float *d_dt,
                                const float *d_h, float *d_dx, float *d_dA, float *d_dB,
                                float *d_dC, float *d_ddt, int L, int D, int M) {
    om_scan1d_backward(d_dy, d_x, d_A, d_B, d_C, d_dt, d_h, d_dx, d_dA, d_dB, d_dC, d_ddt,
                       L, D, M);
}
