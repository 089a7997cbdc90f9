#ifndef MAMBA_SCAN_H
#define MAMBA_SCAN_H

#include "scan.h"
#include "mamba_scan_2d.h"

/* Public k-mamba aliases (reference include/mamba_scan.h). */
typedef ScanParams               MambaScan1DParams;
typedef ScanBackwardParams       MambaScan1DBackwardParams;
typedef ScanBackwardSharedParams MambaScan1DBackwardM1Params;

#ifdef __cplusplus
extern "C" {
#endif
void mamba_scan1d_forward(MambaScan1DParams *p);
void mamba_scan1d_backward(MambaScan1DBackwardParams *p);
void mamba_scan1d_backward_m1_shared_bc(MambaScan1DBackwardM1Params *p);
#ifdef __cplusplus
}
#endif

#endif
