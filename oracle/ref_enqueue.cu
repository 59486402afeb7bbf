// ref_enqueue.cu — test harness around the reference's own kernels (src/dcn_kernel.cu of
// flairziv/tensorrt-dcnv2-plugin, compiled unchanged from the reference tree by oracle/Makefile).
// It replays the three precision branches of DCNv2Plugin::enqueue (src/dcn_plugin.cpp:135-174)
// with the same launcher and cuBLAS calls, once per image (the reference enqueue reads image 0
// only; the loop applies it to every image). deformable_groups is not supported by the reference
// kernels; callers use it with dg = 1 only. Test infrastructure: never linked into libdcnv2.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "dcn_kernel.h"

namespace {
int out_dim(int in, int k, int s, int p, int d) { return (in + 2 * p - d * (k - 1) - 1) / s + 1; }

// One cuBLAS handle per device, created on the first call and kept for the process, as the
// reference plugin creates its handle once, lazily, on its first enqueue
// (src/dcn_plugin.cpp:131) and keeps it until the plugin is destroyed.
constexpr int kMaxDev = 64;
cublasHandle_t g_handle[kMaxDev] = {};
std::mutex g_handle_mu;

cublasHandle_t handle_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lock(g_handle_mu);
  if (!g_handle[dev] && cublasCreate(&g_handle[dev]) != CUBLAS_STATUS_SUCCESS)
    g_handle[dev] = nullptr;
  return g_handle[dev];
}
}  // namespace

extern "C" {

// Bytes of workspace the reference asks for (getWorkspaceSize, src/dcn_plugin.cpp:110-118).
size_t ref_workspace_size(int Cin, int K, int Cout, int Ho, int Wo) {
  const size_t CKK = static_cast<size_t>(Cin) * K * K, HW = static_cast<size_t>(Ho) * Wo;
  return (CKK * HW + static_cast<size_t>(Cout) * CKK) * sizeof(float);
}

// dtype: 0 = fp32, 1 = fp16, 2 = int8 (x, weight int8; offset, mask, bias, y fp32).
// Returns 0 on success, 1 on a cuBLAS error, 2 on a CUDA error.
int ref_enqueue(int dtype, int N, int Cin, int H, int W, int Cout, int K, int stride, int pad,
                int dil, const void* x, const void* offset, const void* mask, const void* weight,
                const void* bias, void* y, void* workspace, float x_scale, float w_scale,
                void* stream) {
  const int Ho = out_dim(H, K, stride, pad, dil), Wo = out_dim(W, K, stride, pad, dil);
  const int CKK = Cin * K * K, HW = Ho * Wo;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cublasHandle_t h = handle_for_current_device();
  if (!h || cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS) return 1;
  const float one = 1.f, zero = 0.f;
  int rc = 0;
  for (int n = 0; n < N && rc == 0; ++n) {
    const size_t xo = static_cast<size_t>(n) * Cin * H * W;
    const size_t oo = static_cast<size_t>(n) * 2 * K * K * HW;
    const size_t mo = static_cast<size_t>(n) * K * K * HW;
    const size_t yo = static_cast<size_t>(n) * Cout * HW;
    if (dtype == 2) {
      float* cols = static_cast<float*>(workspace);
      float* wf = cols + static_cast<size_t>(CKK) * HW;
      deform_im2col_int8_launch(static_cast<const int8_t*>(x) + xo,
                                static_cast<const float*>(offset) + oo,
                                static_cast<const float*>(mask) + mo, cols, Cin, H, W, Ho, Wo, K,
                                stride, pad, dil, st);
      dequant_weight_launch(static_cast<const int8_t*>(weight), wf, Cout * CKK, st);
      if (cublasSgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, HW, Cout, CKK, &one, cols, HW, wf, CKK, &zero,
                      static_cast<float*>(y) + yo, HW) != CUBLAS_STATUS_SUCCESS)
        rc = 1;
      add_bias_scale_launch(static_cast<float*>(y) + yo, static_cast<const float*>(bias),
                            x_scale * w_scale, Cout, HW, st);
    } else if (dtype == 1) {
      __half* cols = static_cast<__half*>(workspace);
      deform_im2col_half_launch(static_cast<const __half*>(x) + xo,
                                static_cast<const __half*>(offset) + oo,
                                static_cast<const __half*>(mask) + mo, cols, Cin, H, W, Ho, Wo, K,
                                stride, pad, dil, st);
      if (cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, HW, Cout, CKK, &one, cols, CUDA_R_16F, HW,
                       static_cast<const __half*>(weight), CUDA_R_16F, CKK, &zero,
                       static_cast<__half*>(y) + yo, CUDA_R_16F, HW, CUBLAS_COMPUTE_32F,
                       CUBLAS_GEMM_DEFAULT_TENSOR_OP) != CUBLAS_STATUS_SUCCESS)
        rc = 1;
      add_bias_half_launch(static_cast<__half*>(y) + yo, static_cast<const __half*>(bias), Cout,
                           HW, st);
    } else {
      float* cols = static_cast<float*>(workspace);
      deform_im2col_launch(static_cast<const float*>(x) + xo,
                           static_cast<const float*>(offset) + oo,
                           static_cast<const float*>(mask) + mo, cols, Cin, H, W, Ho, Wo, K,
                           stride, pad, dil, st);
      if (cublasSgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, HW, Cout, CKK, &one, cols, HW,
                      static_cast<const float*>(weight), CKK, &zero, static_cast<float*>(y) + yo,
                      HW) != CUBLAS_STATUS_SUCCESS)
        rc = 1;
      add_bias_launch(static_cast<float*>(y) + yo, static_cast<const float*>(bias), Cout, HW, st);
    }
    if (cudaGetLastError() != cudaSuccess) rc = 2;
  }
  // Asynchronous like the reference enqueue: nothing waits for the stream here.
  return rc;
}

}  // extern "C"
