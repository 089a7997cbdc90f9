/*
 * kmamba_resident.h -- device-resident KMamba models (no counterpart in the
 * reference).
 *
 * The reference API keeps every weight, gradient and optimizer moment of a
 * KMamba in host arrays, so each kmamba_forward / kmamba_train_step of this
 * library copies them to the GPU and the updated ones back.  A model made
 * device-resident keeps its device copies between calls instead: the calls
 * use them in place and copy nothing, and the host arrays are not updated
 * until kmamba_sync_to_host (kmamba_save calls it itself).
 *
 * Order: kmamba_create, kmamba_init, kmamba_enable_training, then
 * kmamba_set_device_resident(m, 1); arrays allocated later are not
 * resident.  kmamba_init re-uploads a resident model's arrays; a caller who
 * writes the host arrays directly calls kmamba_set_device_resident(m, 1)
 * again to upload them.  kmamba_set_device_resident(m, 0) copies the device
 * values back and releases the device copies; kmamba_free releases them
 * without copying.  The device copies belong to the device current at the
 * call; calls on another device stage the host arrays as usual.
 *
 * Both return 0, or a negative KMB_* status (kmamba_b200.h).
 */
#ifndef KMAMBA_RESIDENT_H
#define KMAMBA_RESIDENT_H

#include "kmamba.h"

#ifdef __cplusplus
extern "C" {
#endif

int kmamba_set_device_resident(KMamba *m, int on);
int kmamba_sync_to_host(KMamba *m);

#ifdef __cplusplus
}
#endif

#endif /* KMAMBA_RESIDENT_H */
