/*
 * 1D selective scan entry points: the reference C API (include/scan.h,
 * include/mamba_scan.h, include/mamba_scan_cuda.h of k-mamba) and the
 * batched kmb_scan1d_* extension, all routed to the sm_100a kernels in
 * csrc/cuda/scan1d.cu.
 */
#include <stdio.h>
#include <stdlib.h>
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

/* ------------------------------------------------------------------ */
/* batch-sliced host <-> device pipeline                               */
/* ------------------------------------------------------------------ */

/*
 * A call whose large tensors live in host memory runs one batch item at a
 * time through a ring of PIPE_SLOTS device slots: host->device copies of
 * item i+1 (copy stream), the kernels of item i (library stream) and the
 * device->host copies of item i-1 (second copy stream) overlap, so the
 * call takes about as long as its larger copy direction instead of the
 * sum of both directions and the kernels.  Tensors already in device
 * memory are used in place.  Copies overlap only for page-locked host
 * buffers; pageable ones are still correct (the driver stages them).
 */
#define PIPE_SLOTS 3
#define PIPE_MAX_DEV 16
enum { PT_X, PT_DT, PT_B, PT_C, PT_H0, PT_Y, PT_HL, PT_HALL, PT_CK, PT_DY, PT_DX, PT_DDT,
       PT_DB, PT_DC, PT_N };

typedef struct {
    const void *user; /* caller pointer, NULL when absent */
    size_t item;      /* bytes per batch item */
    int in, out;      /* copied in before / out after the item's kernels */
    int host;         /* user points to host memory */
    void *slot[PIPE_SLOTS];
} PipeTensor;

typedef struct {
    cudaStream_t in, out;
    cudaEvent_t start, ev_in[PIPE_SLOTS], ev_comp[PIPE_SLOTS], ev_out[PIPE_SLOTS];
    int ready;
} PipeRes;

/* per host thread and device; created on first use, kept for the thread's
 * lifetime (streams and events are reclaimed with the CUDA context) */
static __thread PipeRes t_pipe[PIPE_MAX_DEV];

static PipeRes *pipe_res(void) {
    int dev = 0;
    PipeRes *r;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= PIPE_MAX_DEV) {
        (void)cudaGetLastError();
        return NULL;
    }
    r = &t_pipe[dev];
    if (!r->ready) {
        int ok = cudaStreamCreateWithFlags(&r->in, cudaStreamNonBlocking) == cudaSuccess &&
                 cudaStreamCreateWithFlags(&r->out, cudaStreamNonBlocking) == cudaSuccess &&
                 cudaEventCreateWithFlags(&r->start, cudaEventDisableTiming) == cudaSuccess;
        for (int k = 0; ok && k < PIPE_SLOTS; ++k)
            ok = cudaEventCreateWithFlags(&r->ev_in[k], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&r->ev_comp[k], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&r->ev_out[k], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            (void)cudaGetLastError();
            return NULL;
        }
        r->ready = 1;
    }
    return r;
}

static void pt_set(PipeTensor *t, const void *user, size_t item, int in, int out) {
    memset(t, 0, sizeof *t);
    t->user = user;
    t->item = item;
    t->in = in;
    t->out = out;
    t->host = user && !kmb_is_device_ptr(user);
}

/* pointer of batch item i: the slot when staged, else in place */
static void *pt_ptr(const PipeTensor *t, long i, int k) {
    if (!t->user) return NULL;
    return t->host ? t->slot[k] : (void *)((const char *)t->user + (size_t)i * t->item);
}

/* 1 when the call should take the sliced pipeline */
static int pipe_wanted(const KmbScan1D *a, int bwd) {
    const void *big[6] = {a->x, a->dt, bwd ? a->dy : a->y, bwd ? a->dx : NULL,
                          bwd ? a->ddt : NULL, a->B};
    if (a->batch < 2) return 0;
    for (int i = 0; i < 6; ++i)
        if (big[i] && !kmb_is_device_ptr(big[i])) return 1;
    return 0;
}

static int scan1d_pipelined(const KmbScan1D *a, int bwd) {
    KmbStage st;
    PipeTensor T[PT_N];
    PipeRes *r = pipe_res();
    const size_t f = sizeof(float);
    const long L = a->L, D = a->D, N = a->N;
    const size_t e_ld = f * (size_t)(L * D);
    const size_t e_bc = f * (size_t)(L * (a->bc_shared ? 1 : D) * N);
    const size_t e_st = f * (size_t)(D * N);
    const size_t e_all = f * (size_t)(L * D * N);
    const size_t e_ck = f * (size_t)kmb_scan1d_ckpt_elems(1, L, D, N);
    const int alias = !bwd && a->h_last && a->h_last == a->h0;
    const int own_ck = bwd && !a->h_all && !a->ckpt;
    const float *dA_in;
    float *dA = NULL;
    void *ck_slot[PIPE_SLOTS] = {0};
    cudaStream_t s;
    int rc = KMB_OK;
    cudaError_t e;

    if (!r) return 1; /* no pipeline resources: the caller runs the single-shot path */
    kmb_stage_begin(&st);
    s = st.s;
    pt_set(&T[PT_X], a->x, e_ld, 1, 0);
    pt_set(&T[PT_DT], a->dt, e_ld, 1, 0);
    pt_set(&T[PT_B], a->B, e_bc, 1, 0);
    pt_set(&T[PT_C], a->C, e_bc, 1, 0);
    pt_set(&T[PT_H0], a->h0, e_st, 1, alias);
    pt_set(&T[PT_Y], bwd ? NULL : a->y, e_ld, 0, 1);
    pt_set(&T[PT_HL], (bwd || alias) ? NULL : a->h_last, e_st, 0, 1);
    pt_set(&T[PT_HALL], a->h_all, e_all, bwd, !bwd);
    pt_set(&T[PT_CK], a->ckpt, e_ck, bwd, !bwd);
    pt_set(&T[PT_DY], bwd ? a->dy : NULL, e_ld, 1, 0);
    pt_set(&T[PT_DX], bwd ? a->dx : NULL, e_ld, 0, 1);
    pt_set(&T[PT_DDT], bwd ? a->ddt : NULL, e_ld, 0, 1);
    pt_set(&T[PT_DB], bwd ? a->dB : NULL, e_bc, 0, 1);
    pt_set(&T[PT_DC], bwd ? a->dC : NULL, e_bc, 0, 1);
    dA_in = (const float *)kmb_stage_in(&st, a->A, e_st);
    if (bwd) dA = (float *)kmb_stage_out(&st, a->dA, e_st, 0);
    for (int t = 0; t < PT_N && !st.status; ++t)
        if (T[t].user && T[t].host)
            for (int k = 0; k < PIPE_SLOTS; ++k) T[t].slot[k] = kmb_scratch(&st, T[t].item);
    for (int k = 0; own_ck && k < PIPE_SLOTS && !st.status; ++k) ck_slot[k] = kmb_scratch(&st, e_ck);
    if (st.status) return kmb_stage_finish(&st, st.status);

    e = cudaEventRecord(r->start, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(r->in, r->start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(r->out, r->start, 0);
    if (e != cudaSuccess) return kmb_stage_finish(&st, kmb_cuda_fail(e, "scan1d pipeline start"));

    for (long i = 0; i < a->batch && rc == KMB_OK; ++i) {
        const int k = (int)(i % PIPE_SLOTS);
        KmbScan1D sl = *a;
        /* slot k is free once the copies out of item i - PIPE_SLOTS are done */
        if (i >= PIPE_SLOTS) e = cudaStreamWaitEvent(r->in, r->ev_out[k], 0);
        for (int t = 0; t < PT_N && e == cudaSuccess; ++t)
            if (T[t].user && T[t].host && T[t].in)
                e = cudaMemcpyAsync(T[t].slot[k], (const char *)T[t].user + (size_t)i * T[t].item,
                                    T[t].item, cudaMemcpyHostToDevice, r->in);
        if (e == cudaSuccess) e = cudaEventRecord(r->ev_in[k], r->in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, r->ev_in[k], 0);
        if (e != cudaSuccess) {
            rc = kmb_cuda_fail(e, "scan1d pipeline copy-in");
            break;
        }
        sl.batch = 1;
        sl.A = dA_in;
        sl.x = (const float *)pt_ptr(&T[PT_X], i, k);
        sl.dt = (const float *)pt_ptr(&T[PT_DT], i, k);
        sl.B = (const float *)pt_ptr(&T[PT_B], i, k);
        sl.C = (const float *)pt_ptr(&T[PT_C], i, k);
        sl.h0 = (const float *)pt_ptr(&T[PT_H0], i, k);
        sl.h_all = (float *)pt_ptr(&T[PT_HALL], i, k);
        sl.ckpt = (float *)pt_ptr(&T[PT_CK], i, k);
        if (!bwd) {
            sl.y = (float *)pt_ptr(&T[PT_Y], i, k);
            sl.h_last = alias ? (float *)sl.h0 : (float *)pt_ptr(&T[PT_HL], i, k);
            rc = kmb_launch_scan1d_fwd(&sl, s);
        } else {
            const float *ck = sl.ckpt;
            sl.dy = (const float *)pt_ptr(&T[PT_DY], i, k);
            sl.dx = (float *)pt_ptr(&T[PT_DX], i, k);
            sl.ddt = (float *)pt_ptr(&T[PT_DDT], i, k);
            sl.dB = (float *)pt_ptr(&T[PT_DB], i, k);
            sl.dC = (float *)pt_ptr(&T[PT_DC], i, k);
            sl.dA = dA;
            sl.y = NULL;
            sl.h_last = NULL;
            if (own_ck) {
                KmbScan1D fw = sl;
                fw.ckpt = (float *)ck_slot[k];
                fw.h_all = NULL;
                rc = kmb_launch_scan1d_fwd(&fw, s);
                ck = fw.ckpt;
            }
            if (i > 0) sl.flags |= KMB_SCAN1D_DA_ACCUM;
            if (rc == KMB_OK) rc = kmb_launch_scan1d_bwd(&sl, ck, s);
        }
        if (rc != KMB_OK) break;
        e = cudaEventRecord(r->ev_comp[k], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(r->out, r->ev_comp[k], 0);
        for (int t = 0; t < PT_N && e == cudaSuccess; ++t)
            if (T[t].user && T[t].host && T[t].out)
                e = cudaMemcpyAsync((char *)T[t].user + (size_t)i * T[t].item, T[t].slot[k],
                                    T[t].item, cudaMemcpyDeviceToHost, r->out);
        if (e == cudaSuccess) e = cudaEventRecord(r->ev_out[k], r->out);
        if (e != cudaSuccess) rc = kmb_cuda_fail(e, "scan1d pipeline copy-out");
    }
    /* every slot goes back to the pool only after both copy streams drain */
    e = cudaStreamSynchronize(r->out);
    if (e != cudaSuccess && rc == KMB_OK) rc = kmb_cuda_fail(e, "scan1d pipeline drain");
    e = cudaStreamSynchronize(r->in);
    if (e != cudaSuccess && rc == KMB_OK) rc = kmb_cuda_fail(e, "scan1d pipeline drain");
    return kmb_stage_finish(&st, rc);
}

/* ------------------------------------------------------------------ */
/* sequence-split kernels (channel-shared B/C, N = 16, D % 32 == 0)     */
/* ------------------------------------------------------------------ */

/* KMB_SCAN1D_SEGMENTS=0 keeps the whole-sequence kernels for fp32 calls
 * (a value >= 1 fixes the number of segments; default: planned). */
static int seg_enabled(void) {
    const char *e = getenv("KMB_SCAN1D_SEGMENTS");
    return !(e && e[0] == '0' && e[1] == 0);
}

/* Forward through the sequence-split kernels on device pointers `d`. */
static int seg_forward(KmbStage *st, const KmbScan1D *d, int bf16) {
    int S = 1, seg_len = 0;
    kmb_scan1d_seg_plan(d->batch, d->L, d->D, &S, &seg_len);
    float *state = (float *)kmb_scratch(st, sizeof(float) * (size_t)d->batch * S * d->D * 16);
    int *flag = (int *)kmb_scratch(st, sizeof(int) * (size_t)d->batch * (d->D / 32) * S);
    if (!state || !flag) return st->status;
    return kmb_launch_scan1d_fwd_seg(d, bf16, S, seg_len, state, flag, st->s);
}

/* Backward through the sequence-split kernels; computes the checkpoints
 * into scratch first when the caller has none. */
static int seg_backward(KmbStage *st, const KmbScan1D *d, int bf16) {
    const float *ck = d->ckpt;
    int rc;
    if (!ck) {
        KmbScan1D f = *d;
        f.ckpt = (float *)kmb_scratch(
            st, sizeof(float) * (size_t)kmb_scan1d_ckpt_elems(d->batch, d->L, d->D, d->N));
        if (!f.ckpt) return st->status;
        f.y = NULL;
        f.h_last = NULL;
        if ((rc = seg_forward(st, &f, bf16))) return rc;
        ck = f.ckpt;
    }
    int S = 1, seg_len = 0;
    kmb_scan1d_seg_plan(d->batch, d->L, d->D, &S, &seg_len);
    float *state = (float *)kmb_scratch(st, sizeof(float) * (size_t)d->batch * S * d->D * 16);
    int *flag = (int *)kmb_scratch(st, sizeof(int) * (size_t)d->batch * (d->D / 32) * S);
    float *dB32 = d->dB, *dC32 = d->dC;
    if (bf16) {
        const size_t nbc = sizeof(float) * (size_t)d->batch * d->L * 16;
        dB32 = (float *)kmb_scratch(st, nbc);
        dC32 = (float *)kmb_scratch(st, nbc);
    }
    if (!state || !flag || !dB32 || !dC32) return st->status;
    return kmb_launch_scan1d_bwd_seg(d, ck, bf16, S, seg_len, state, flag, dB32, dC32, st->s);
}

int kmb_scan1d_fwd(const KmbScan1D *a) {
    KmbStage st;
    KmbScan1D d;
    int rc = validate_common(a);
    if (rc) return rc;
    if (pipe_wanted(a, 0) && (rc = scan1d_pipelined(a, 0)) != 1) return rc;
    kmb_stage_begin(&st);
    stage_args(&st, a, &d, 0);
    if (st.status) return kmb_stage_finish(&st, st.status);
    if (seg_enabled() && kmb_scan1d_seg_supported(&d, 4))
        rc = seg_forward(&st, &d, 0);
    else
        rc = kmb_launch_scan1d_fwd(&d, st.s);
    return kmb_stage_finish(&st, rc);
}

/* bf16 I/O variants: device memory only, the channel-shared layout. */
static int validate_bf16(const KmbScan1D *a, int bwd) {
    int rc = validate_common(a);
    if (rc) return rc;
    if (!kmb_scan1d_seg_supported(a, 2))
        return kmb_fail(KMB_EUNSUPPORTED,
                        "scan1d bf16: needs B/C shared across channels, N = 16, D a multiple of "
                        "32, no h_all and 16-byte aligned tensors");
    if (bwd && (!a->dy || !a->dx || !a->ddt || !a->dA || !a->dB || !a->dC))
        return kmb_fail(KMB_EINVAL, "scan1d bf16 backward: dy and every gradient are required");
    const void *ptrs[] = {a->x, a->dt, a->A, a->B, a->C, a->h0, a->y, a->h_last, a->ckpt,
                          a->dy, a->dx, a->ddt, a->dA, a->dB, a->dC};
    for (size_t i = 0; i < sizeof ptrs / sizeof *ptrs; ++i)
        if (ptrs[i] && !kmb_is_device_ptr(ptrs[i]))
            return kmb_fail(KMB_EINVAL, "scan1d bf16: every tensor must be device memory");
    return KMB_OK;
}

int kmb_scan1d_fwd_bf16(const KmbScan1D *a) {
    KmbStage st;
    int rc = validate_bf16(a, 0);
    if (rc) return rc;
    kmb_stage_begin(&st);
    rc = seg_forward(&st, a, 1);
    return kmb_stage_finish(&st, rc);
}

int kmb_scan1d_bwd_bf16(const KmbScan1D *a) {
    KmbStage st;
    int rc = validate_bf16(a, 1);
    if (rc) return rc;
    kmb_stage_begin(&st);
    rc = seg_backward(&st, a, 1);
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
    if (pipe_wanted(a, 1) && (rc = scan1d_pipelined(a, 1)) != 1) return rc;
    kmb_stage_begin(&st);
    stage_args(&st, a, &d, 1);
    if (st.status) return kmb_stage_finish(&st, st.status);
    if (seg_enabled() && kmb_scan1d_seg_supported(&d, 4))
        return kmb_stage_finish(&st, seg_backward(&st, &d, 0));
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
