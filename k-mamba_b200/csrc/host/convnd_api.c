/*
 * ConvND entry points: the reference C API (convnd.h of k-mamba,
 * src/convnd.c:58-244 and cuda/convnd.cu:258-436) and the batched
 * kmb_convnd_* extension, routed to csrc/cuda/convnd.cu.
 */
#include <stdio.h>
#include <string.h>

#include "../kmb_internal.h"
#include "convnd.h"
#include "km_topology.h"
#include "wavefront_nd.h"

static void report(int status) {
    if (status != KMB_OK && status != KMB_EINVAL)
        fprintf(stderr, "kmamba_b200: %s\n", kmb_last_error());
}

long convnd_kernel_volume(long ndims, long K) {
    if (ndims <= 0 || K <= 0) return 0;
    return km_power_long(K, ndims);
}

static int validate(const KmbConvND *a, int bwd) {
    if (!a) return kmb_fail(KMB_EINVAL, "convnd: NULL arguments");
    if (a->ndims <= 0 || a->ndims > 8) return kmb_fail(KMB_EINVAL, "convnd: ndims out of range");
    if (!wavefront_nd_validate_dims(a->dims, a->ndims))
        return kmb_fail(KMB_EINVAL, "convnd: invalid dims");
    if (a->batch <= 0 || a->D <= 0 || a->K <= 0)
        return kmb_fail(KMB_EINVAL, "convnd: batch, D and K must be positive");
    if (wavefront_nd_total_points(a->dims, a->ndims) <= 0)
        return kmb_fail(KMB_EINVAL, "convnd: grid too large");
    if (convnd_kernel_volume(a->ndims, a->K) > (1L << 20))
        return kmb_fail(KMB_EUNSUPPORTED, "convnd: kernel volume too large");
    if (!a->input || !a->kernel) return kmb_fail(KMB_EINVAL, "convnd: input and kernel required");
    if (!bwd && !a->output) return kmb_fail(KMB_EINVAL, "convnd: output required");
    if (bwd && (!a->dy || !a->dinput || !a->dkernel))
        return kmb_fail(KMB_EINVAL, "convnd: dy, dinput and dkernel required");
    return KMB_OK;
}

static int run(const KmbConvND *a, int bwd) {
    KmbStage st;
    KmbConvND d;
    int rc = validate(a, bwd);
    const long P = rc ? 0 : wavefront_nd_total_points(a->dims, a->ndims);
    const size_t act = sizeof(float) * (size_t)a->batch * P * a->D;
    const size_t ker = sizeof(float) * (size_t)convnd_kernel_volume(a->ndims, a->K) * a->D;
    const size_t vec = sizeof(float) * (size_t)a->D;
    if (rc) return rc;
    kmb_stage_begin(&st);
    d = *a;
    d.input = kmb_stage_in(&st, a->input, act);
    d.kernel = kmb_stage_in(&st, a->kernel, ker);
    if (!bwd) {
        d.bias = kmb_stage_in(&st, a->bias, vec);
        d.output = kmb_stage_out(&st, a->output, act, 0);
    } else {
        d.dy = kmb_stage_in(&st, a->dy, act);
        d.dinput = kmb_stage_out(&st, a->dinput, act, 0);
        d.dkernel = kmb_stage_out(&st, a->dkernel, ker, 0);
        d.dbias = kmb_stage_out(&st, a->dbias, vec, 0);
    }
    if (st.status) return kmb_stage_finish(&st, st.status);
    rc = bwd ? kmb_launch_convnd_bwd(&d, st.s) : kmb_launch_convnd_fwd(&d, st.s);
    return kmb_stage_finish(&st, rc);
}

int kmb_convnd_fwd(const KmbConvND *a) { return run(a, 0); }
int kmb_convnd_bwd(const KmbConvND *a) { return run(a, 1); }

/* bf16 activations on device memory (include/kmamba_b200.h) */
static int run_bf16(const KmbConvND *a, int bwd) {
    KmbStage st;
    int rc = validate(a, bwd);
    if (rc) return rc;
    if (!kmb_convnd_bf16_supported(a, bwd))
        return kmb_fail(KMB_EUNSUPPORTED,
                        "convnd bf16: needs 2D with D a multiple of 64 or 3D with D a multiple "
                        "of 8, K <= 3 and 16-byte aligned tensors");
    const void *fwd_ptrs[] = {a->input, a->kernel, a->bias, a->output};
    const void *bwd_ptrs[] = {a->input, a->kernel, a->dy, a->dinput, a->dkernel, a->dbias};
    const void *const *ptrs = bwd ? bwd_ptrs : fwd_ptrs;
    const size_t n = bwd ? sizeof bwd_ptrs / sizeof *bwd_ptrs : sizeof fwd_ptrs / sizeof *fwd_ptrs;
    for (size_t i = 0; i < n; ++i)
        if (ptrs[i] && !kmb_is_device_ptr(ptrs[i]))
            return kmb_fail(KMB_EINVAL, "convnd bf16: every tensor must be device memory");
    kmb_stage_begin(&st);
    rc = bwd ? kmb_launch_convnd_bwd_bf16(a, st.s) : kmb_launch_convnd_fwd_bf16(a, st.s);
    return kmb_stage_finish(&st, rc);
}

int kmb_convnd_fwd_bf16(const KmbConvND *a) { return run_bf16(a, 0); }
int kmb_convnd_bwd_bf16(const KmbConvND *a) { return run_bf16(a, 1); }

/* Fills a one-item KmbConvND from the reference params. */
static int from_params(const ConvNDParams *p, KmbConvND *a) {
    if (!p || !p->dims || p->ndims <= 0 || p->ndims > 8) return 0;
    memset(a, 0, sizeof *a);
    for (long i = 0; i < p->ndims; ++i) a->dims[i] = p->dims[i];
    a->ndims = p->ndims;
    a->batch = 1;
    a->D = p->D;
    a->K = p->K;
    a->input = p->input;
    a->kernel = p->kernel;
    a->bias = p->bias;
    a->output = p->output;
    a->dy = p->dy;
    a->dinput = p->dinput;
    a->dkernel = p->dkernel;
    a->dbias = p->dbias;
    return 1;
}

void convnd_forward_wavefront(ConvNDParams *p, const KMWavefrontPlan *plan) {
    KmbConvND a;
    if (!p || !p->input || !p->kernel || !p->output || !p->dims || p->ndims <= 0 || p->D <= 0 ||
        p->K <= 0)
        return;
    if (!km_wavefront_plan_matches_dims(plan, p->dims, p->ndims)) return;
    if (!from_params(p, &a)) return;
    report(kmb_convnd_fwd(&a));
}

void convnd_backward_wavefront(ConvNDParams *p, const KMWavefrontPlan *plan) {
    KmbConvND a;
    if (!p || !p->input || !p->kernel || !p->dy || !p->dinput || !p->dkernel || !p->dims ||
        p->ndims <= 0 || p->D <= 0 || p->K <= 0)
        return;
    if (!km_wavefront_plan_matches_dims(plan, p->dims, p->ndims)) return;
    if (!from_params(p, &a)) return;
    report(kmb_convnd_bwd(&a));
}

/* src/convnd.c:208-244.  The convolution has no cross-point dependency, so
 * no plan is built: the GPU kernels cover the whole grid in one pass. */
void convnd(ConvNDParams *p, ConvNDMode mode) {
    KmbConvND a;
    if (!p || !p->dims || p->ndims <= 0) return;
    if (!wavefront_nd_validate_dims(p->dims, p->ndims)) return;
    if (!from_params(p, &a)) return;
    if ((mode & CONVND_FORWARD) && p->input && p->kernel && p->output && p->D > 0 && p->K > 0)
        report(kmb_convnd_fwd(&a));
    if ((mode & CONVND_BACKWARD) && p->input && p->kernel && p->dy && p->dinput && p->dkernel &&
        p->D > 0 && p->K > 0)
        report(kmb_convnd_bwd(&a));
}

/* cuda/convnd.cu:258-329 and 332-436: device pointers, 0 / -1. */
int om_convnd_forward(ConvNDParams *p) {
    KmbConvND a;
    if (!from_params(p, &a)) return -1;
    return kmb_convnd_fwd(&a) == KMB_OK ? 0 : -1;
}

int om_convnd_backward(ConvNDParams *p) {
    KmbConvND a;
    if (!from_params(p, &a)) return -1;
    return kmb_convnd_bwd(&a) == KMB_OK ? 0 : -1;
}
