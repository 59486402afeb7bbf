/*
 * dcnv2.h — C ABI of libdcnv2.so, the sm_100a DCNv2 (modulated deformable convolution)
 * forward behind the dcn::DCNv2 TensorRT plugin interface.
 *
 * Every entry point replaces one piece of the reference plugin (flairziv/tensorrt-dcnv2-plugin,
 * src/dcn_plugin.cpp); the citation is given beside each declaration. Signatures use plain C
 * types and raw device pointers only, so any FFI (ctypes, cgo, JNI, a TensorRT IPluginV3 shim)
 * can bind them. All functions are thread-safe and reentrant; the library holds no global
 * handles apart from per-device launch attributes and, for dcnv2_forward_host, two copy streams
 * per device, each set up once. Kernel-selection overrides for measurements (dcnv2_diag.h) are
 * read from the environment once per process; the dispatch never calls getenv.
 *
 * Tensor contract (src/dcn_plugin.cpp:76,134; python/01_oracle_and_export.py:73-75):
 *   input 0  x       [N, C, H, W]                 linear NCHW
 *   input 1  offset  [N, 2*dg*K*K, Ho, Wo]         channel 2*(g*K*K+t) = dh, +1 = dw
 *   input 2  mask    [N, dg*K*K, Ho, Wo]
 *   input 3  weight  [O, C, K, K]
 *   input 4  bias    [O]
 *   output 0 y       [N, O, Ho, Wo]                Ho = (H + 2p - d(K-1) - 1)/s + 1
 * Precision combinations (src/dcn_plugin.cpp:94-104):
 *   DCNV2_FLOAT: all six tensors fp32
 *   DCNV2_HALF : all six tensors fp16
 *   DCNV2_INT8 : x and weight int8 (per-tensor symmetric scales), offset/mask/bias/y fp32
 */
#ifndef DCNV2_H_
#define DCNV2_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DCNV2_API __attribute__((visibility("default")))
#else
#define DCNV2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque CUDA stream (cudaStream_t); 0 is the legacy default stream. */
typedef void* dcnv2_stream_t;

/* Element types. Values equal nvinfer1::DataType (kFLOAT=0, kHALF=1, kINT8=2). */
typedef enum {
  DCNV2_FLOAT = 0,
  DCNV2_HALF = 1,
  DCNV2_INT8 = 2
} dcnv2_dtype;

/* Tensor formats. Value equals nvinfer1::TensorFormat::kLINEAR. */
typedef enum { DCNV2_FORMAT_LINEAR = 0 } dcnv2_format;

typedef enum {
  DCNV2_OK = 0,
  DCNV2_ERR_INVALID_ARG = 1,   /* bad shape, attribute, pointer or scale */
  DCNV2_ERR_UNSUPPORTED = 2,   /* dtype/format combination the plugin does not accept */
  DCNV2_ERR_WORKSPACE = 3,     /* workspace pointer null or smaller than dcnv2_workspace_size */
  DCNV2_ERR_CUDA = 4,          /* a CUDA runtime call or kernel launch failed */
  DCNV2_ERR_NO_DEVICE = 5,     /* no usable sm_100 device for the current context */
  DCNV2_ERR_DEVICE_TIMEOUT = 6, /* a kernel gave up waiting on an on-chip barrier (error word) */
  DCNV2_ERR_SCRATCH_LIMIT = 7   /* problem needs more than DCNV2_STATIC_SCRATCH_BYTES of scratch */
} dcnv2_status;

/* Math modes (dcnv2_desc.math). */
enum {
  DCNV2_MATH_DEFAULT = 0,    /* fp16: tensor cores, packed-f16 sampler; int8: tensor cores, exact
                                int32 accumulation; fp32: fused CUDA-core kernel, fp32-exact */
  DCNV2_MATH_PRECISE = 1,    /* fp16: fp32 sampler arithmetic (one rounding per column value);
                                int8: each column value is the reference's fp32 sample
                                m * bilinear(x_q) rounded to nearest and clamped to +-127, on the
                                one-thread-per-output kernel (a cross-check mode, slow) */
  DCNV2_MATH_TF32 = 2,       /* fp32 only: single-pass TF32 tensor cores (own, looser bound) */
  DCNV2_MATH_SIMT = 3,       /* one thread per output on CUDA cores (any shape; cross-check) */
  DCNV2_MATH_TF32X3 = 4      /* fp32 only: 3xTF32 split on tensor cores (own bound, ~5e-5 rel.) */
};

/* Layer description: shapes of x and weight plus the five plugin attributes. */
typedef struct {
  int32_t n, c, h, w;            /* x dims */
  int32_t out_c;                 /* O = weight.d[0] (src/dcn_plugin.cpp:85) */
  int32_t kernel;                /* K (attribute "kernel") */
  int32_t stride;                /* attribute "stride" */
  int32_t padding;               /* attribute "padding" */
  int32_t dilation;              /* attribute "dilation" */
  int32_t deformable_groups;     /* attribute "deformable_groups" */
  int32_t dtype;                 /* dcnv2_dtype of x; selects the precision combination */
  int32_t math;                  /* DCNV2_MATH_* */
} dcnv2_desc;

/* ---- Stateless layer API (what the plugin's enqueue forwards to) ---- */

/* Output shape [N, O, Ho, Wo]. Replaces DCNv2Plugin::getOutputShapes (src/dcn_plugin.cpp:72-89). */
DCNV2_API dcnv2_status dcnv2_output_shape(const dcnv2_desc* desc, int64_t out_dims[4]);

/* Workspace bytes needed by dcnv2_forward for this desc (includes the batch dimension).
 * Replaces DCNv2Plugin::getWorkspaceSize (src/dcn_plugin.cpp:110-118). Returns 0 on a bad desc. */
DCNV2_API size_t dcnv2_workspace_size(const dcnv2_desc* desc);

/* One forward pass, asynchronous on `stream`. All tensor pointers are device pointers; bias may
 * be NULL (treated as zeros). x_scale/w_scale are used only for DCNV2_INT8 (they are the
 * PluginTensorDesc::scale of inputs 0 and 3). Never allocates, never synchronises.
 * Replaces DCNv2Plugin::enqueue (src/dcn_plugin.cpp:122-176). */
DCNV2_API dcnv2_status dcnv2_forward(const dcnv2_desc* desc,
                           const void* x, const void* offset, const void* mask,
                           const void* weight, const void* bias, void* y,
                           void* workspace, size_t workspace_bytes,
                           float x_scale, float w_scale, dcnv2_stream_t stream);

/* ---- Layer with its offset / mask head ---- */

/* Workspace bytes for dcnv2_forward_with_head (0 when the desc is not supported there). */
DCNV2_API size_t dcnv2_forward_with_head_workspace_size(const dcnv2_desc* desc);

/* The DCNv2 block as the reference's detector builds it (python/detector.py:44,50-52;
 * python/01_oracle_and_export.py:42,46-48): om = Conv2d(C -> 3*dg*K*K, K x K, stride 1,
 * padding (K-1)/2, with bias)(x), offset = om[:, :2*dg*K*K], mask = sigmoid(om[:, 2*dg*K*K:]),
 * y = DCNv2(x, offset, mask, weight, bias). There the head is a separate convolution, slice and
 * sigmoid in front of the plugin (the plugin's inputs 1 and 2, src/dcn_plugin.cpp:134); here it
 * runs on tensor cores from the layer's own channels-last copy of x and writes offset and mask
 * in the layout the layer then reads. Supported: fp16 (desc.dtype DCNV2_HALF, math DEFAULT or
 * PRECISE), stride 1, dilation 1, padding (K-1)/2, C a multiple of 8, 3*dg*K*K <= 256;
 * DCNV2_ERR_UNSUPPORTED otherwise. head_weight [3*dg*K*K][C][K][K] and head_bias [3*dg*K*K]
 * (NULL = zeros) are fp16 device pointers. offset_out [N][2*dg*K*K][H][W] and mask_out
 * [N][dg*K*K][H][W] (fp16, device) receive the head's outputs when not NULL; otherwise they stay
 * in the workspace. Asynchronous on `stream`; never allocates or synchronises. */
DCNV2_API dcnv2_status dcnv2_forward_with_head(const dcnv2_desc* desc, const void* x,
                                               const void* head_weight, const void* head_bias,
                                               const void* weight, const void* bias, void* y,
                                               void* offset_out, void* mask_out, void* workspace,
                                               size_t workspace_bytes, dcnv2_stream_t stream);

/* ---- Host-buffer forward (copies overlapped with compute) ---- */

/* Workspace bytes for dcnv2_forward_host with chunks of at most `images_per_chunk` images (0
 * picks the chunk: about an eighth of the batch). Returns 0 on a bad desc. */
DCNV2_API size_t dcnv2_forward_host_workspace_size(const dcnv2_desc* desc,
                                                   int32_t images_per_chunk);

/* dcnv2_forward with x, offset, mask and y in HOST memory (weight and bias stay device pointers,
 * as the plugin's constants are). The batch runs in chunks of images (the first and the last a
 * quarter of the others, when the batch spans more than two): the upload of chunk i+1,
 * the forward of chunk i and the download of chunk i-1 overlap on two library-owned copy streams
 * (created once per device) and `stream`, ordered by events. Asynchronous like cudaMemcpyAsync:
 * y is complete when `stream` has completed. Host buffers must be page-locked for the copies to
 * overlap (pageable memory works, serialised). Results are bit-identical to dcnv2_forward.
 * No counterpart in the reference plugin, whose enqueue only sees device buffers
 * (src/dcn_plugin.cpp:122-176); it serves callers that hold their tensors on the host, as the
 * reference's latency benchmark does (TrtRunner.infer with host feeds, H2D and D2H inside the
 * timed call: python/03_benchmark.py:102-113). */
DCNV2_API dcnv2_status dcnv2_forward_host(const dcnv2_desc* desc, const void* x_host,
                                          const void* offset_host, const void* mask_host,
                                          const void* weight, const void* bias, void* y_host,
                                          void* workspace, size_t workspace_bytes,
                                          float x_scale, float w_scale, int32_t images_per_chunk,
                                          dcnv2_stream_t stream);

/* Size of the library's built-in static scratch buffer used by dcnv2_forward_static_scratch. */
#define DCNV2_STATIC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* dcnv2_forward for callers that cannot allocate device memory: no counterpart in the reference
 * plugin (there TensorRT always hands enqueue a workspace). Some callers must not call cudaMalloc
 * once they run: an engine whose memory plan is fixed at build time, a serving loop where an
 * allocation would synchronise the device and stall other streams, or a process held to a fixed
 * device-memory budget by its own pool. This entry point takes only inputs and outputs; its
 * scratch (the channels-last copy of x, the packed weights and the error word) lives in one
 * file-scope static __device__ buffer of DCNV2_STATIC_SCRATCH_BYTES (32 MiB) that every GPU which
 * loads the library holds until the process exits. It calls no cudaMalloc, cudaFree or other
 * allocating routine.
 *   - Problems whose scratch need (dcnv2_workspace_size) exceeds the buffer are rejected with
 *     DCNV2_ERR_SCRATCH_LIMIT before anything is launched.
 *   - The first call on each device looks up the buffer's device address (cudaGetSymbolAddress
 *     with that device current); make that first call before any stream capture begins.
 *   - All calls on a device share the one buffer and it keeps the last call's contents (each call
 *     rewrites every byte it reads and clears the error word itself). Calls that overlap on the
 *     GPU — on different streams, or from different host threads — race on it; issue them on one
 *     stream, one after another. */
DCNV2_API dcnv2_status dcnv2_forward_static_scratch(const dcnv2_desc* desc, const void* x,
                                                   const void* offset, const void* mask,
                                                   const void* weight, const void* bias, void* y,
                                                   float x_scale, float w_scale,
                                                   dcnv2_stream_t stream);

/* Copies the device error word of the last dcnv2_forward_static_scratch call on the current device
 * (which lives in the static buffer, an address the caller never sees) to *code, after
 * synchronising `stream`: 0 = none, otherwise DCNV2_DEVERR_* bits, with DCNV2_ERR_DEVICE_TIMEOUT
 * returned. The word belongs to whichever call ran last on the device. Allocates nothing. No
 * counterpart in the reference plugin (it reports no device-side errors). */
DCNV2_API dcnv2_status dcnv2_read_static_scratch_error(dcnv2_stream_t stream, int32_t* code);

/* Copies the device error word of the last forward that used `workspace` to *code (0 = none;
 * otherwise DCNV2_DEVERR_* bits) after synchronising `stream`. Test and debug helper. */
DCNV2_API dcnv2_status dcnv2_read_device_error(const void* workspace, dcnv2_stream_t stream, int32_t* code);

/* Device error bits written by the kernels into the workspace error word. */
enum {
  DCNV2_DEVERR_TIMEOUT_PRODUCER = 1,
  DCNV2_DEVERR_TIMEOUT_MMA = 2,
  DCNV2_DEVERR_TIMEOUT_SAMPLER = 4,
  DCNV2_DEVERR_TIMEOUT_EPILOGUE = 8,
  DCNV2_DEVERR_TIMEOUT_DRAIN = 16
};

/* Which kernel family dcnv2_forward would launch: 1 = fused tcgen05 (tensor cores),
 * 2 = fused fp32-exact CUDA-core kernel, 0 = one-thread-per-output CUDA-core kernel. */
DCNV2_API int32_t dcnv2_uses_tensor_cores(const dcnv2_desc* desc);

/* Number of kernels dcnv2_forward launches for this desc. */
DCNV2_API int32_t dcnv2_launch_count(const dcnv2_desc* desc);

DCNV2_API const char* dcnv2_status_string(dcnv2_status status);

/* ---- Plugin object API (IPluginV3 + creator, without TensorRT types) ---- */

/* Plugin identity: "DCNv2", "1", namespace "" (src/dcn_plugin.cpp:22-23,56-58,216-218). */
DCNV2_API const char* dcnv2_plugin_name(void);
DCNV2_API const char* dcnv2_plugin_version(void);
DCNV2_API const char* dcnv2_plugin_namespace(void);

/* Attribute names in creator order: stride, padding, dilation, kernel, deformable_groups
 * (src/dcn_plugin.cpp:211). Returns the count; names[i] valid for the library's lifetime. */
DCNV2_API int32_t dcnv2_plugin_field_names(const char* const** names);

typedef struct dcnv2_plugin dcnv2_plugin;

/* DCNv2Creator::createPlugin (src/dcn_plugin.cpp:222-235): unknown names are ignored, missing
 * ones take the defaults stride=1 padding=1 dilation=1 kernel=3 deformable_groups=1, a field
 * with a NULL value reads as 0. Values are INT32. Returns NULL on out-of-memory. */
DCNV2_API dcnv2_plugin* dcnv2_plugin_create(const char* const* names, const int32_t* const* values,
                                  int32_t nb_fields);
/* DCNv2Plugin::clone (src/dcn_plugin.cpp:51-53) and attachToContext (:181). */
DCNV2_API dcnv2_plugin* dcnv2_plugin_clone(const dcnv2_plugin* p);
DCNV2_API void dcnv2_plugin_destroy(dcnv2_plugin* p);

/* DCNv2Plugin::getFieldsToSerialize (src/dcn_plugin.cpp:184-194): writes the five INT32 fields in
 * the order stride, padding, dilation, kernel, deformable_groups; names may be NULL. Returns 5. */
DCNV2_API int32_t dcnv2_plugin_serialize(const dcnv2_plugin* p, const char** names, int32_t values[5]);

/* PluginTensorDesc mirror: dims, type (dcnv2_dtype), format and quantisation scale. */
typedef struct {
  int32_t nb_dims;
  int64_t d[8];
  int32_t type;
  int32_t format;
  float scale;
} dcnv2_tensor_desc;

/* getNbOutputs (src/dcn_plugin.cpp:61). Always 1. */
DCNV2_API int32_t dcnv2_plugin_nb_outputs(const dcnv2_plugin* p);

/* getOutputDataTypes (src/dcn_plugin.cpp:64-68), with the INT8 case returning FLOAT so that it
 * agrees with supportsFormatCombination. */
DCNV2_API int32_t dcnv2_plugin_output_dtype(const dcnv2_plugin* p, int32_t x_type);

/* getOutputShapes (src/dcn_plugin.cpp:72-89) on concrete dims: in_dims = x dims, w_dims = weight
 * dims. Output d[0] = N, d[1] = weight.d[0], d[2..3] = floor((in + 2p - d(K-1) - 1)/s) + 1. */
DCNV2_API dcnv2_status dcnv2_plugin_output_shape(const dcnv2_plugin* p, const int64_t x_dims[4],
                                       const int64_t w_dims[4], int64_t out_dims[4]);

/* supportsFormatCombination (src/dcn_plugin.cpp:94-104) over 6 positions (5 inputs + output). */
DCNV2_API int32_t dcnv2_plugin_supports_format(const dcnv2_plugin* p, int32_t pos,
                                     const dcnv2_tensor_desc* in_out, int32_t nb_inputs,
                                     int32_t nb_outputs);

/* getWorkspaceSize (src/dcn_plugin.cpp:110-118) from the x and output descs. */
DCNV2_API size_t dcnv2_plugin_workspace_size(const dcnv2_plugin* p, const dcnv2_tensor_desc* inputs,
                                   int32_t nb_inputs, const dcnv2_tensor_desc* outputs,
                                   int32_t nb_outputs);

/* enqueue (src/dcn_plugin.cpp:122-176): reads N/C/H/W from in[0], O from in[3], the precision
 * from in[0].type and the INT8 scales from in[0].scale, in[3].scale. Returns 0 on success and
 * a dcnv2_status value otherwise (the reference always returned 0). */
DCNV2_API int32_t dcnv2_plugin_enqueue(const dcnv2_plugin* p, const dcnv2_tensor_desc* in_desc,
                             const dcnv2_tensor_desc* out_desc, const void* const* inputs,
                             void* const* outputs, void* workspace, size_t workspace_bytes,
                             dcnv2_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DCNV2_H_ */
