/*
 * CPU ORACLE — test infrastructure only.
 *
 * C restatement of the two NASM kernels of the reference
 * (cpu/scan1d.asm:40-179 and cpu/scan2d.asm:48-285), which cannot be
 * assembled here because nasm is absent.  Linked with the reference's own
 * C sources into _ref/libkmamba_ref.so so that scan_nd.c's dispatch and
 * every other reference symbol resolve.  Scalar fp32 in the asm's
 * instruction order; build with -ffp-contract=off.
 */
#include <math.h>

#include "scan.h" /* the reference's header (-I$(REF)/include) */

void scan1d(ScanParams *p) {
    for (long t = 0; t < p->L; t++) {
        for (long d = 0; d < p->D; d++) {
            const long td = t * p->D + d;
            float yacc = 0.0f;
            for (long m = 0; m < p->M; m++) {
                const long dm = d * p->M + m;
                const long tdm = td * p->M + m;
                const float dA = expf(p->delta[td] * p->A[dm]); /* mulss; call expf */
                const float dB = p->B[tdm] * p->delta[td];      /* mulss xmm2, xmm1 */
                float hn = dA * p->h[dm];                       /* mulss xmm0, xmm4 */
                hn = hn + dB * p->x[td];                        /* mulss; addss */
                hn = (hn < 1000.0f) ? hn : 1000.0f;             /* minss */
                hn = (hn > -1000.0f) ? hn : -1000.0f;           /* maxss */
                p->h[dm] = hn;
                yacc = yacc + p->C[tdm] * hn;
            }
            p->y[td] = yacc;
        }
    }
}

void scan2d(Scan2DParams *p) {
    const long DM = p->D * p->M;
    for (long k = 0; k < p->d1 + p->d2 - 1; k++) {
        long i = k - p->d2 + 1;
        const long i_max = k < p->d1 - 1 ? k : p->d1 - 1;
        if (i < 0) i = 0;
        for (; i <= i_max; i++) {
            const long j = k - i;
            const long pos = i * p->d2 + j;
            for (long d = 0; d < p->D; d++) {
                const long pd = pos * p->D + d;
                float yacc = 0.0f;
                for (long m = 0; m < p->M; m++) {
                    const long dm = d * p->M + m;
                    const long pdm = pos * DM + dm;
                    const float h1 = i > 0 ? p->h[(pos - p->d2) * DM + dm] : 0.0f;
                    const float h2 = j > 0 ? p->h[(pos - 1) * DM + dm] : 0.0f;
                    const float dA1 = expf(p->delta1[pd] * p->A1[dm]);
                    const float dA2 = expf(p->delta2[pd] * p->A2[dm]);
                    const float hs = (p->delta1[pd] + p->delta2[pd]) * 0.5f;
                    const float dB = p->B[pdm] * hs;
                    float hn = dA1 * h1;
                    hn = hn + dA2 * h2;
                    hn = hn + dB * p->x[pd];
                    p->h[pdm] = hn;
                    yacc = yacc + p->C[pdm] * hn;
                }
                p->y[pd] = yacc;
            }
        }
    }
}
