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

/* dcnv2_forward with a CUDA event recorded on `stream` before each of its launches and one after
 * the last: events[i] (cudaEvent_t) precedes launch i, events[dcnv2_launch_count(desc)] follows
 * the last launch. n_events must be at least dcnv2_launch_count(desc) + 1. Used to time the
 * kernels of one forward separately. */
DCNV2_API dcnv2_status dcnv2_diag_forward_events(const dcnv2_desc* desc, const void* x,
                                                 const void* offset, const void* mask,
                                                 const void* weight, const void* bias, void* y,
                                                 void* workspace, size_t workspace_bytes,
                                                 float x_scale, float w_scale,
                                                 dcnv2_stream_t stream, void* const* events,
                                                 int32_t n_events);

/* Name of the last (main) kernel dcnv2_forward launches for this desc: "dcnv2_fused_ta_kernel"
 * (tensor cores, A operand in TMEM), "dcnv2_fused_kernel" (tensor cores, A in shared memory),
 * "dcnv2_f32_exact_kernel" or "dcnv2_simt_kernel"; NULL on a bad desc. For labelling
 * measurements and matching profiler output. */
DCNV2_API const char* dcnv2_diag_main_kernel(const dcnv2_desc* desc);

/* Kernel selection for measurements and tests, process-wide. kernel: 0 = automatic (A operand in
 * tensor memory for fp16 / int8 layers of at most 256 output channels, in shared memory above),
 * 1 = A in tensor memory for every fp16 / int8 layer (one output-channel chunk of at most 256 per
 * tile), 2 = A in shared memory always. pair (A-in-shared-memory kernel only; the TMEM-A kernel
 * always runs one CTA per tile): 0 = automatic (CTA pairs, tcgen05 cta_group::2, for fp16 / int8
 * tiles with more than 256 output channels, one CTA per tile otherwise), 1 = CTA pairs for every
 * fp16 / int8 tile, 2 = one CTA per tile always.
 * The starting values come from the environment, read once per process: DCNV2_KERNEL=ta|smem,
 * DCNV2_PAIR=1|0. Change the selection only between forwards: dcnv2_workspace_size and
 * dcnv2_forward must see the same one. */
DCNV2_API dcnv2_status dcnv2_diag_set_kernel_override(int32_t kernel, int32_t pair);

/* Architecture of the device code this library runs on the current device, as the runtime
 * reports it for the main fp16 kernel (cudaFuncAttributes::binaryVersion: 100 = sm_100).
 * Returns DCNV2_ERR_NO_DEVICE when the device cannot run the library's code. */
DCNV2_API dcnv2_status dcnv2_diag_binary_arch(int32_t* binary_version);

#ifdef __cplusplus
}
#endif

#endif /* DCNV2_DIAG_H_ */
