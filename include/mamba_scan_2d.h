#ifndef MAMBA_SCAN_2D_H
#define MAMBA_SCAN_2D_H

#include "scan.h"

/* Public k-mamba alias (reference include/mamba_scan_2d.h). */
typedef Scan2DParams MambaScan2DParams;

#ifdef __cplusplus
extern "C" {
#endif
void mamba_scan2d_forward(MambaScan2DParams *p);
#ifdef __cplusplus
}
#endif

#endif
