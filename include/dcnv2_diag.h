/*
 * dcnv2_diag.h — diagnostics of libdcnv2.so that have no counterpart in the reference plugin.
 */
#ifndef DCNV2_DIAG_H_
#define DCNV2_DIAG_H_

#include <stdint.h>

#include "dcnv2.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Failure-detection self test on the current device: launches one warp that waits on an
 * mbarrier nothing will complete, through the same bounded-wait routine the forward kernels
 * use. After `timeout_us` the wait gives up, records a DCNV2_DEVERR_* bit and the kernel
 * returns normally, so the context stays usable. Synchronous; allocates 4 bytes.
 * Returns DCNV2_ERR_DEVICE_TIMEOUT (expected) with the recorded bits in *device_code. */
DCNV2_API dcnv2_status dcnv2_diag_timeout_selftest(uint32_t timeout_us, int32_t* device_code);

#ifdef __cplusplus
}
#endif

#endif /* DCNV2_DIAG_H_ */
