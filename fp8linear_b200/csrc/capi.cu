// capi.cu -- the extern "C" boundary (include/fp8linear_b200.h): argument checks that
// mirror the reference's TORCH_CHECKs, workspace carving for the fused op, and the
// thread-local error message. Only the peer-buffer set-up calls allocate (or map)
// device memory; every operator call works in the caller's buffers.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "fp8linear_b200.h"
#include "internal.h"

namespace fp8lin {

namespace {
thread_local std::string g_last_error;

int fail(int code, const std::string &msg) {
  set_error(msg);
  return code;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr size_t kWsAlign = 256;
size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

void set_error(const std::string &msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

bool current_device_info(DeviceInfo *info) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return false;
  }
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal out of range");
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].device != dev) {
    DeviceInfo d;
    d.device = dev;
    if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) !=
            cudaSuccess) {
      set_error(std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
      return false;
    }
    cache[dev] = d;
  }
  *info = cache[dev];
  return true;
}

namespace {

int check_gemm_args(const void *xq, const float *xs, const void *wq, const float *ws,
                    const void *bias, int bias_dtype, const void *out, int out_dtype, int64_t M,
                    int64_t N, int64_t K, const char *op) {
  const std::string o(op);
  if (M < 0 || N < 0 || K < 0) return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": negative size");
  if (out_dtype != kBF16 && out_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": out_dtype must be BF16 or F16");
  if (bias != nullptr && bias_dtype != kBF16 && bias_dtype != kF16 && bias_dtype != kF32)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": bias_dtype must be BF16, F16 or F32");
  if (K % 16 != 0 || K == 0)
    return fail(FP8LIN_ERR_UNSUPPORTED,
                o + ": K must be a positive multiple of 16 for FP8 matmul, got " +
                    std::to_string(K));
  if (M == 0 || N == 0) return FP8LIN_OK;
  if (!xq || !xs || !wq || !ws || !out)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": null pointer");
  if (!aligned(xq, 16) || !aligned(wq, 16))
    return fail(FP8LIN_ERR_UNSUPPORTED, o + ": xq and wq must be 16-byte aligned");
  if (!aligned(out, 2)) return fail(FP8LIN_ERR_UNSUPPORTED, o + ": out must be 2-byte aligned");
  return FP8LIN_OK;
}

}  // namespace
}  // namespace fp8lin

using namespace fp8lin;

extern "C" {

int fp8lin_abi_version(void) { return FP8LIN_ABI_VERSION; }

#define FP8LIN_STR2(x) #x
#define FP8LIN_STR(x) FP8LIN_STR2(x)
const char *fp8lin_build_info(void) {
  return "fp8linear_b200: sm_100a tcgen05 e4m3 GEMM (128x256x128 tiles, 4-stage TMA ring, "
         "fused dequant+bias epilogue), per-token quantizer; nvcc " FP8LIN_STR(
             __CUDACC_VER_MAJOR__) "." FP8LIN_STR(__CUDACC_VER_MINOR__);
}

const char *fp8lin_last_error(void) { return g_last_error.c_str(); }

int fp8lin_quantize_fp8(const void *x, int x_dtype, int64_t M, int64_t K, void *xq,
                        float *x_scale, void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_fp8: x must be fp16 or bf16");
  if (M < 0 || K < 0) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_fp8: negative size");
  if (M == 0) return FP8LIN_OK;
  if (K == 0) return fail(FP8LIN_ERR_UNSUPPORTED, "quantize_fp8: K must be positive");
  if (!x || !xq || !x_scale) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_fp8: null pointer");
  cudaError_t e = launch_quantize_rows(x, x_dtype, M, K, static_cast<uint8_t *>(xq), x_scale,
                                       static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("quantize_fp8: launch: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

size_t fp8lin_mx_scale_bytes(int64_t rows, int64_t K) {
  if (rows <= 0 || K <= 0) return 0;
  return static_cast<size_t>(mx_scale_bytes(rows, K));
}

int fp8lin_quantize_mxfp8(const void *x, int x_dtype, int64_t M, int64_t K, void *xq,
                          void *scales, void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_mxfp8: x must be fp16 or bf16");
  if (M < 0 || K < 0) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_mxfp8: negative size");
  if (K % 32 != 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "quantize_mxfp8: K must be a multiple of 32 for MXFP8, got " + std::to_string(K));
  if (M == 0) return FP8LIN_OK;
  if (K == 0) return fail(FP8LIN_ERR_UNSUPPORTED, "quantize_mxfp8: K must be positive");
  if (!x || !xq || !scales)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_mxfp8: null pointer");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(xq) % 8 ||
      reinterpret_cast<uintptr_t>(scales) % 4)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "quantize_mxfp8: x must be 16-byte, xq 8-byte and scales 4-byte aligned");
  cudaError_t e = launch_quantize_mx(x, x_dtype, M, K, static_cast<uint8_t *>(xq),
                                     static_cast<uint8_t *>(scales),
                                     static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("quantize_mxfp8: launch: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_quantize_weight(const void *w, int w_dtype, int64_t N, int64_t K, void *wq,
                           float *w_scale, void *stream) {
  clear_error();
  if (w_dtype != kBF16 && w_dtype != kF16 && w_dtype != kF32)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_weight: weight must be bf16, fp16 or fp32");
  if (N < 0 || K < 0) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_weight: negative size");
  if (N == 0) return FP8LIN_OK;
  if (!w || !wq || !w_scale)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_weight: null pointer");
  cudaError_t e = launch_quantize_weight(w, w_dtype, N, K, static_cast<uint8_t *>(wq), w_scale,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("quantize_weight: launch: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_fp8_gemm(const void *xq, const float *x_scale, const void *wq, const float *w_scale,
                    const void *bias, int bias_dtype, void *out, int out_dtype, int64_t M,
                    int64_t N, int64_t K, void *stream) {
  clear_error();
  int rc = check_gemm_args(xq, x_scale, wq, w_scale, bias, bias_dtype, out, out_dtype, M, N, K,
                           "fp8_gemm");
  if (rc != FP8LIN_OK || M == 0 || N == 0) return rc;
  GemmArgs a{static_cast<const uint8_t *>(xq), x_scale, static_cast<const uint8_t *>(wq),
             w_scale, bias, bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  return launch_gemm(a, static_cast<cudaStream_t>(stream), true);
}

size_t fp8lin_linear_workspace_size(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return round_up(static_cast<size_t>(M) * static_cast<size_t>(K), kWsAlign) +
         round_up(static_cast<size_t>(M) * sizeof(float), kWsAlign);
}

int fp8lin_fp8_linear(const void *x, int x_dtype, const void *wq, const float *w_scale,
                      const void *bias, int bias_dtype, void *out, int out_dtype, int64_t M,
                      int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                      void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear: x must be fp16 or bf16");
  int rc = check_gemm_args(reinterpret_cast<const void *>(16), w_scale, wq, w_scale, bias,
                           bias_dtype, out, out_dtype, M, N, K, "fp8_linear");
  if (rc != FP8LIN_OK || M == 0 || N == 0) return rc;
  if (!x) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear: null x");
  const size_t need = fp8lin_linear_workspace_size(M, K);
  if (!workspace || workspace_bytes < need)
    return fail(FP8LIN_ERR_WORKSPACE, "fp8_linear: workspace of " + std::to_string(need) +
                                          " bytes required, got " +
                                          std::to_string(workspace_bytes));
  if (!aligned(workspace, kWsAlign))
    return fail(FP8LIN_ERR_WORKSPACE, "fp8_linear: workspace must be 256-byte aligned");
  uint8_t *xq = static_cast<uint8_t *>(workspace);
  float *xs = reinterpret_cast<float *>(
      xq + round_up(static_cast<size_t>(M) * static_cast<size_t>(K), kWsAlign));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Few tokens (the GEMM streams the weight matrix once): the quantizer, which launches
  // while the kernel before it still runs, brings the weights into L2 on the way.
  L2Prefetch pf;
  if (M <= kFewTokenMaxM) {
    pf.ptr = wq;
    pf.bytes = N * K;
  }
  cudaError_t e = launch_quantize_rows(x, x_dtype, M, K, xq, xs, s, true, pf);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("fp8_linear: quantize launch: ") +
                                     cudaGetErrorString(e));
  GemmArgs a{xq, xs, static_cast<const uint8_t *>(wq), w_scale, bias,
             bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  a.weights_before_wait = true;  // the previous kernel is this call's quantizer
  return launch_gemm(a, s, true);
}

int fp8lin_mxfp8_gemm(const void *xq, const void *x_scales, const void *wq, const void *w_scales,
                      const void *bias, int bias_dtype, void *out, int out_dtype, int64_t M,
                      int64_t N, int64_t K, void *stream) {
  clear_error();
  const float *dummy = reinterpret_cast<const float *>(16);
  int rc = check_gemm_args(xq, dummy, wq, dummy, bias, bias_dtype, out, out_dtype, M, N, K,
                           "mxfp8_gemm");
  if (rc != FP8LIN_OK) return rc;
  if (K % 32 != 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "mxfp8_gemm: K must be a multiple of 32 for MXFP8, got " + std::to_string(K));
  if (M == 0 || N == 0) return FP8LIN_OK;
  if (!x_scales || !w_scales) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "mxfp8_gemm: null scales");
  if (!aligned(x_scales, 16) || !aligned(w_scales, 16))
    return fail(FP8LIN_ERR_UNSUPPORTED, "mxfp8_gemm: scale grids must be 16-byte aligned");
  GemmArgs a{static_cast<const uint8_t *>(xq), nullptr, static_cast<const uint8_t *>(wq),
             nullptr, bias, bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  a.mx = true;
  a.xsf = static_cast<const uint8_t *>(x_scales);
  a.wsf = static_cast<const uint8_t *>(w_scales);
  return launch_gemm(a, static_cast<cudaStream_t>(stream), true);
}

size_t fp8lin_mxfp8_linear_workspace_size(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return round_up(static_cast<size_t>(M) * static_cast<size_t>(K), kWsAlign) +
         round_up(static_cast<size_t>(mx_scale_bytes(M, K)), kWsAlign);
}

int fp8lin_mxfp8_linear(const void *x, int x_dtype, const void *wq, const void *w_scales,
                        const void *bias, int bias_dtype, void *out, int out_dtype, int64_t M,
                        int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                        void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "mxfp8_linear: x must be fp16 or bf16");
  const float *dummy = reinterpret_cast<const float *>(16);
  int rc = check_gemm_args(reinterpret_cast<const void *>(16), dummy, wq, dummy, bias, bias_dtype,
                           out, out_dtype, M, N, K, "mxfp8_linear");
  if (rc != FP8LIN_OK) return rc;
  if (K % 32 != 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "mxfp8_linear: K must be a multiple of 32 for MXFP8, got " + std::to_string(K));
  if (M == 0 || N == 0) return FP8LIN_OK;
  if (!x || !w_scales) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "mxfp8_linear: null pointer");
  if (!aligned(x, 16) || !aligned(w_scales, 16))
    return fail(FP8LIN_ERR_UNSUPPORTED, "mxfp8_linear: x and w_scales must be 16-byte aligned");
  const size_t need = fp8lin_mxfp8_linear_workspace_size(M, K);
  if (!workspace || workspace_bytes < need || !aligned(workspace, kWsAlign))
    return fail(FP8LIN_ERR_WORKSPACE, "mxfp8_linear: workspace of " + std::to_string(need) +
                                          " bytes (256-byte aligned) required, got " +
                                          std::to_string(workspace_bytes));
  uint8_t *xq = static_cast<uint8_t *>(workspace);
  uint8_t *xsf = xq + round_up(static_cast<size_t>(M) * static_cast<size_t>(K), kWsAlign);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_quantize_mx(x, x_dtype, M, K, xq, xsf, s, true);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("mxfp8_linear: quantize launch: ") +
                                     cudaGetErrorString(e));
  GemmArgs a{xq, nullptr, static_cast<const uint8_t *>(wq), nullptr, bias,
             bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  a.mx = true;
  a.xsf = xsf;
  a.wsf = static_cast<const uint8_t *>(w_scales);
  a.weights_before_wait = true;  // the previous kernel is this call's quantizer
  return launch_gemm(a, s, true);
}

size_t fp8lin_nv_scale_bytes(int64_t rows, int64_t K) {
  if (rows <= 0 || K <= 0) return 0;
  return static_cast<size_t>(nv_scale_bytes(rows, K));
}

int fp8lin_quantize_nvfp4(const void *x, int x_dtype, int64_t M, int64_t K, void *xq,
                          void *scales, void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_nvfp4: x must be fp16 or bf16");
  if (M < 0 || K < 0) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_nvfp4: negative size");
  if (K % 32 != 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "quantize_nvfp4: K must be a multiple of 32 for NVFP4, got " + std::to_string(K));
  if (M == 0) return FP8LIN_OK;
  if (K == 0) return fail(FP8LIN_ERR_UNSUPPORTED, "quantize_nvfp4: K must be positive");
  if (!x || !xq || !scales)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "quantize_nvfp4: null pointer");
  if (!aligned(x, 16) || !aligned(xq, 4) || !aligned(scales, 4))
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "quantize_nvfp4: x must be 16-byte, xq and scales 4-byte aligned");
  cudaError_t e = launch_quantize_nv(x, x_dtype, M, K, static_cast<uint8_t *>(xq),
                                     static_cast<uint8_t *>(scales),
                                     static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("quantize_nvfp4: launch: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_nvfp4_gemm(const void *xq, const void *x_scales, const void *wq, const void *w_scales,
                      const void *bias, int bias_dtype, void *out, int out_dtype, int64_t M,
                      int64_t N, int64_t K, void *stream) {
  clear_error();
  const float *dummy = reinterpret_cast<const float *>(16);
  int rc = check_gemm_args(xq, dummy, wq, dummy, bias, bias_dtype, out, out_dtype, M, N, K,
                           "nvfp4_gemm");
  if (rc != FP8LIN_OK) return rc;
  if (K % 32 != 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "nvfp4_gemm: K must be a multiple of 32 for NVFP4, got " + std::to_string(K));
  if (M == 0 || N == 0) return FP8LIN_OK;
  if (!x_scales || !w_scales) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "nvfp4_gemm: null scales");
  if (!aligned(x_scales, 16) || !aligned(w_scales, 16))
    return fail(FP8LIN_ERR_UNSUPPORTED, "nvfp4_gemm: scale grids must be 16-byte aligned");
  GemmArgs a{static_cast<const uint8_t *>(xq), nullptr, static_cast<const uint8_t *>(wq),
             nullptr, bias, bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  a.mx = true;
  a.nv = true;
  a.xsf = static_cast<const uint8_t *>(x_scales);
  a.wsf = static_cast<const uint8_t *>(w_scales);
  return launch_gemm(a, static_cast<cudaStream_t>(stream), true);
}

size_t fp8lin_nvfp4_linear_workspace_size(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return round_up(static_cast<size_t>(M) * static_cast<size_t>(K) / 2, kWsAlign) +
         round_up(static_cast<size_t>(nv_scale_bytes(M, K)), kWsAlign);
}

int fp8lin_nvfp4_linear(const void *x, int x_dtype, const void *wq, const void *w_scales,
                        const void *bias, int bias_dtype, void *out, int out_dtype, int64_t M,
                        int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                        void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "nvfp4_linear: x must be fp16 or bf16");
  const float *dummy = reinterpret_cast<const float *>(16);
  int rc = check_gemm_args(reinterpret_cast<const void *>(16), dummy, wq, dummy, bias, bias_dtype,
                           out, out_dtype, M, N, K, "nvfp4_linear");
  if (rc != FP8LIN_OK) return rc;
  if (K % 32 != 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                "nvfp4_linear: K must be a multiple of 32 for NVFP4, got " + std::to_string(K));
  if (M == 0 || N == 0) return FP8LIN_OK;
  if (!x || !w_scales) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "nvfp4_linear: null pointer");
  if (!aligned(x, 16) || !aligned(w_scales, 16))
    return fail(FP8LIN_ERR_UNSUPPORTED, "nvfp4_linear: x and w_scales must be 16-byte aligned");
  const size_t need = fp8lin_nvfp4_linear_workspace_size(M, K);
  if (!workspace || workspace_bytes < need || !aligned(workspace, kWsAlign))
    return fail(FP8LIN_ERR_WORKSPACE, "nvfp4_linear: workspace of " + std::to_string(need) +
                                          " bytes (256-byte aligned) required, got " +
                                          std::to_string(workspace_bytes));
  uint8_t *xq = static_cast<uint8_t *>(workspace);
  uint8_t *xsf = xq + round_up(static_cast<size_t>(M) * static_cast<size_t>(K) / 2, kWsAlign);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_quantize_nv(x, x_dtype, M, K, xq, xsf, s, true);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("nvfp4_linear: quantize launch: ") +
                                     cudaGetErrorString(e));
  GemmArgs a{xq, nullptr, static_cast<const uint8_t *>(wq), nullptr, bias,
             bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  a.mx = true;
  a.nv = true;
  a.xsf = xsf;
  a.wsf = static_cast<const uint8_t *>(w_scales);
  a.weights_before_wait = true;  // the previous kernel is this call's quantizer
  return launch_gemm(a, s, true);
}

static int check_modulation(const void *x, int x_dtype, int64_t M, int64_t K, int64_t batches,
                     const void *shift, const void *scale, float eps, const char *op) {
  const std::string o(op);
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": x must be fp16 or bf16");
  if (M < 0 || K < 0) return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": negative size");
  if (K % 8 != 0 || K == 0 || K > kLnMaxK)
    return fail(FP8LIN_ERR_UNSUPPORTED,
                o + ": K must be a positive multiple of 8 up to 8192, got " + std::to_string(K));
  if (batches <= 0 || (M > 0 && M % batches != 0))
    return fail(FP8LIN_ERR_INVALID_ARGUMENT,
                o + ": batches must be positive and divide M (rows " + std::to_string(M) +
                    ", batches " + std::to_string(batches) + ")");
  if (!(eps >= 0.0f)) return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": eps must be >= 0");
  if (M == 0) return FP8LIN_OK;
  if (!x || !shift || !scale) return fail(FP8LIN_ERR_INVALID_ARGUMENT, o + ": null pointer");
  if (!aligned(x, 16) || !aligned(shift, 16) || !aligned(scale, 16))
    return fail(FP8LIN_ERR_UNSUPPORTED, o + ": x, shift and scale must be 16-byte aligned");
  return FP8LIN_OK;
}

int fp8lin_layernorm_modulate_quantize_fp8(const void *x, int x_dtype, int64_t M, int64_t K,
                                           int64_t batches, const void *shift,
                                           const void *scale, float eps, void *xq,
                                           float *x_scale, void *stream) {
  clear_error();
  int rc = check_modulation(x, x_dtype, M, K, batches, shift, scale, eps,
                            "layernorm_modulate_quantize_fp8");
  if (rc != FP8LIN_OK || M == 0) return rc;
  if (!xq || !x_scale)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "layernorm_modulate_quantize_fp8: null output");
  if (!aligned(xq, 8) || !aligned(x_scale, 4))
    return fail(FP8LIN_ERR_UNSUPPORTED,
                "layernorm_modulate_quantize_fp8: xq must be 8-byte, x_scale 4-byte aligned");
  cudaError_t e = launch_ln_modulate_quantize(x, x_dtype, M, K, batches, shift, scale, eps,
                                              static_cast<uint8_t *>(xq), x_scale,
                                              static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("layernorm_modulate_quantize_fp8: launch: ") +
                                     cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_fp8_linear_modulated(const void *x, int x_dtype, int64_t M, int64_t K,
                                int64_t batches, const void *shift, const void *scale, float eps,
                                const void *wq, const float *w_scale, const void *bias,
                                int bias_dtype, void *out, int out_dtype, int64_t N,
                                void *workspace, size_t workspace_bytes, void *stream) {
  clear_error();
  int rc = check_modulation(x, x_dtype, M, K, batches, shift, scale, eps, "fp8_linear_modulated");
  if (rc != FP8LIN_OK) return rc;
  rc = check_gemm_args(reinterpret_cast<const void *>(16), w_scale, wq, w_scale, bias, bias_dtype,
                       out, out_dtype, M, N, K, "fp8_linear_modulated");
  if (rc != FP8LIN_OK || M == 0 || N == 0) return rc;
  const size_t need = fp8lin_linear_workspace_size(M, K);
  if (!workspace || workspace_bytes < need || !aligned(workspace, kWsAlign))
    return fail(FP8LIN_ERR_WORKSPACE, "fp8_linear_modulated: workspace of " +
                                          std::to_string(need) +
                                          " bytes (256-byte aligned) required, got " +
                                          std::to_string(workspace_bytes));
  uint8_t *xq = static_cast<uint8_t *>(workspace);
  float *xs = reinterpret_cast<float *>(
      xq + round_up(static_cast<size_t>(M) * static_cast<size_t>(K), kWsAlign));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_ln_modulate_quantize(x, x_dtype, M, K, batches, shift, scale, eps, xq, xs,
                                              s, true);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("fp8_linear_modulated: quantize launch: ") +
                                     cudaGetErrorString(e));
  GemmArgs a{xq, xs, static_cast<const uint8_t *>(wq), w_scale, bias,
             bias ? bias_dtype : kNone, out, out_dtype, M, N, K};
  a.weights_before_wait = true;  // the previous kernel is this call's quantizer
  return launch_gemm(a, s, true);
}

// ---------------------------------------------------------------- host-buffer linear
namespace {
constexpr int64_t kHostChunkRows = 512;

struct HostStreams {
  std::mutex enqueue;  // one call's copies, kernels and event records at a time
  bool ready = false;
  cudaError_t err = cudaSuccess;
  cudaStream_t up = nullptr, comp = nullptr, down = nullptr;
  cudaEvent_t start = nullptr, up_done[2] = {}, comp_done[2] = {}, down_done[2] = {};
  cudaEvent_t join[3] = {};  // error path: the caller's stream waits on all three streams
};

// The three streams and the events of the current device (created once, kept for the
// life of the process).
HostStreams *host_streams(std::string *why) {
  static std::mutex mu;
  static HostStreams hs[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  HostStreams &h = hs[dev & 63];
  if (!h.ready) {
    h.ready = true;
    const unsigned sf = cudaStreamNonBlocking;
    const unsigned ef = cudaEventDisableTiming;
    if ((h.err = cudaStreamCreateWithFlags(&h.up, sf)) == cudaSuccess &&
        (h.err = cudaStreamCreateWithFlags(&h.comp, sf)) == cudaSuccess &&
        (h.err = cudaStreamCreateWithFlags(&h.down, sf)) == cudaSuccess &&
        (h.err = cudaEventCreateWithFlags(&h.start, ef)) == cudaSuccess) {
      for (int i = 0; i < 3 && h.err == cudaSuccess; ++i)
        h.err = cudaEventCreateWithFlags(&h.join[i], ef);
      for (int i = 0; i < 2 && h.err == cudaSuccess; ++i)
        if ((h.err = cudaEventCreateWithFlags(&h.up_done[i], ef)) == cudaSuccess &&
            (h.err = cudaEventCreateWithFlags(&h.comp_done[i], ef)) == cudaSuccess)
          h.err = cudaEventCreateWithFlags(&h.down_done[i], ef);
    }
  }
  if (h.err != cudaSuccess) {
    *why = cudaGetErrorString(h.err);
    return nullptr;
  }
  return &h;
}

int64_t host_chunk_rows(int64_t M) { return M < kHostChunkRows ? M : kHostChunkRows; }
}  // namespace

size_t fp8lin_fp8_linear_host_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int64_t c = host_chunk_rows(M);
  // two x chunks (2 B per element), two out chunks (2 B), one quantizer workspace
  return 2 * round_up(static_cast<size_t>(c * K * 2), kWsAlign) +
         2 * round_up(static_cast<size_t>(c * N * 2), kWsAlign) + fp8lin_linear_workspace_size(c, K);
}

int fp8lin_fp8_linear_host(const void *x_host, int x_dtype, const void *wq, const float *w_scale,
                           const void *bias, int bias_dtype, void *out_host, int out_dtype,
                           int64_t M, int64_t N, int64_t K, void *workspace,
                           size_t workspace_bytes, void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear_host: x must be fp16 or bf16");
  int rc = check_gemm_args(reinterpret_cast<const void *>(16), w_scale, wq, w_scale, bias,
                           bias_dtype, reinterpret_cast<const void *>(16), out_dtype, M, N, K,
                           "fp8_linear_host");
  if (rc != FP8LIN_OK || M == 0 || N == 0) return rc;
  if (!x_host || !out_host) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear_host: null host buffer");
  const size_t need = fp8lin_fp8_linear_host_workspace_size(M, N, K);
  if (!workspace || workspace_bytes < need || !aligned(workspace, kWsAlign))
    return fail(FP8LIN_ERR_WORKSPACE, "fp8_linear_host: workspace of " + std::to_string(need) +
                                          " bytes (256-byte aligned) required, got " +
                                          std::to_string(workspace_bytes));
  std::string why;
  HostStreams *h = host_streams(&why);
  if (!h) return fail(FP8LIN_ERR_CUDA, "fp8_linear_host: stream setup: " + why);
  const int64_t rows = host_chunk_rows(M);
  const size_t xb = round_up(static_cast<size_t>(rows * K * 2), kWsAlign);
  const size_t ob = round_up(static_cast<size_t>(rows * N * 2), kWsAlign);
  uint8_t *base = static_cast<uint8_t *>(workspace);
  uint8_t *xbuf[2] = {base, base + xb};
  uint8_t *obuf[2] = {base + 2 * xb, base + 2 * xb + ob};
  uint8_t *xq = base + 2 * xb + 2 * ob;
  float *xs = reinterpret_cast<float *>(xq + round_up(static_cast<size_t>(rows * K), kWsAlign));
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  // Calls from several host threads share the device's streams and events: the event
  // records and waits of one call must not interleave with another's.
  std::lock_guard<std::mutex> serial(h->enqueue);
  const char *step = "ordering";
  cudaError_t e = cudaEventRecord(h->start, user);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(h->up, h->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(h->comp, h->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(h->down, h->start, 0);
  const int64_t chunks = (M + rows - 1) / rows;
  DeviceInfo dev;
  const int host_tile_n = current_device_info(&dev) ? pair_tile_n(M, N, dev.sm_count) : 256;
  rc = FP8LIN_OK;
  for (int64_t i = 0; i < chunks && e == cudaSuccess; ++i) {
    const int s = static_cast<int>(i & 1);
    const int64_t r0 = i * rows;
    const int64_t mr = M - r0 < rows ? M - r0 : rows;
    // upload chunk i once the kernels of chunk i-2 no longer read this x slot
    step = "upload";
    if (i >= 2) e = cudaStreamWaitEvent(h->up, h->comp_done[s], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(xbuf[s], static_cast<const uint8_t *>(x_host) + r0 * K * 2,
                          static_cast<size_t>(mr * K * 2), cudaMemcpyHostToDevice, h->up);
    if (e == cudaSuccess) e = cudaEventRecord(h->up_done[s], h->up);
    // kernels of chunk i once it has landed and chunk i-2's output has left this slot
    step = "kernels";
    if (e == cudaSuccess) e = cudaStreamWaitEvent(h->comp, h->up_done[s], 0);
    if (e == cudaSuccess && i >= 2) e = cudaStreamWaitEvent(h->comp, h->down_done[s], 0);
    if (e != cudaSuccess) break;
    e = launch_quantize_rows(xbuf[s], x_dtype, mr, K, xq, xs, h->comp, true);
    if (e != cudaSuccess) break;
    GemmArgs a{xq, xs, static_cast<const uint8_t *>(wq), w_scale, bias,
               bias ? bias_dtype : kNone, obuf[s], out_dtype, mr, N, K};
    // A ragged last chunk of a multi-chunk call takes the CTA-pair kernel like the full
    // chunks, so every row is summed in the order the whole-M call uses.
    a.pairs_only = chunks > 1;
    if (chunks > 1) a.tile_n = host_tile_n;  // the whole call's tile width, every chunk
    a.weights_before_wait = true;  // the previous kernel is this chunk's quantizer
    rc = launch_gemm(a, h->comp, true);
    if (rc != FP8LIN_OK) break;  // launch_gemm set the message
    e = cudaEventRecord(h->comp_done[s], h->comp);
    // download chunk i
    step = "download";
    if (e == cudaSuccess) e = cudaStreamWaitEvent(h->down, h->comp_done[s], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<uint8_t *>(out_host) + r0 * N * 2, obuf[s],
                          static_cast<size_t>(mr * N * 2), cudaMemcpyDeviceToHost, h->down);
    if (e == cudaSuccess) e = cudaEventRecord(h->down_done[s], h->down);
  }
  // the caller's stream continues once the last download is done (it follows every
  // earlier copy and kernel of the call)
  if (e == cudaSuccess && rc == FP8LIN_OK) {
    step = "ordering";
    e = cudaStreamWaitEvent(user, h->down_done[(chunks - 1) & 1], 0);
    if (e == cudaSuccess) return FP8LIN_OK;
  }
  // Failed part-way: copies and kernels of earlier chunks may still be queued on the
  // library's streams and still target the caller's host buffers and workspace. The
  // caller's stream waits for all three streams before the error is returned, so work
  // the caller orders after this call (a free, a reuse of out_host) follows them.
  const std::string msg = rc != FP8LIN_OK
                              ? std::string(g_last_error)
                              : std::string("fp8_linear_host: ") + step + ": " +
                                    cudaGetErrorString(e);
  cudaEvent_t joins[3] = {h->join[0], h->join[1], h->join[2]};
  cudaStream_t lanes[3] = {h->up, h->comp, h->down};
  bool joined = true;
  for (int j = 0; j < 3; ++j)
    joined = joined && cudaEventRecord(joins[j], lanes[j]) == cudaSuccess &&
             cudaStreamWaitEvent(user, joins[j], 0) == cudaSuccess;
  if (!joined) {
    // the event path itself failed: wait on the host instead
    for (int j = 0; j < 3; ++j) cudaStreamSynchronize(lanes[j]);
  }
  return fail(rc != FP8LIN_OK ? rc : FP8LIN_ERR_CUDA, msg);
}

int fp8lin_fp8_linear_allgather(const void *x, int x_dtype, const void *wq, const float *w_scale,
                                const void *bias, int bias_dtype, void *const *outs, int n_outs,
                                int out_dtype, int64_t M, int64_t N, int64_t K, int64_t ldo,
                                void *workspace, size_t workspace_bytes, void *stream) {
  clear_error();
  if (x_dtype != kBF16 && x_dtype != kF16)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear_allgather: x must be fp16 or bf16");
  if (!outs || n_outs < 1 || n_outs > 1 + kMaxPeers)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear_allgather: n_outs must be 1..8");
  if (ldo < N) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear_allgather: ldo < N");
  int rc = check_gemm_args(reinterpret_cast<const void *>(16), w_scale, wq, w_scale, bias,
                           bias_dtype, outs[0], out_dtype, M, N, K, "fp8_linear_allgather");
  if (rc != FP8LIN_OK || M == 0 || N == 0) return rc;
  if (N % 8 != 0 || ldo % 8 != 0)
    return fail(FP8LIN_ERR_UNSUPPORTED, "fp8_linear_allgather: N and ldo must be multiples of 8");
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i] || !aligned(outs[i], 16))
      return fail(FP8LIN_ERR_UNSUPPORTED,
                  "fp8_linear_allgather: every output pointer must be 16-byte aligned");
  if (!x) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "fp8_linear_allgather: null x");
  const size_t need = fp8lin_linear_workspace_size(M, K);
  if (!workspace || workspace_bytes < need || !aligned(workspace, kWsAlign))
    return fail(FP8LIN_ERR_WORKSPACE, "fp8_linear_allgather: workspace of " +
                                          std::to_string(need) +
                                          " bytes (256-byte aligned) required");
  uint8_t *xq = static_cast<uint8_t *>(workspace);
  float *xs = reinterpret_cast<float *>(
      xq + round_up(static_cast<size_t>(M) * static_cast<size_t>(K), kWsAlign));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_quantize_rows(x, x_dtype, M, K, xq, xs, s, true);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("fp8_linear_allgather: quantize launch: ") +
                                     cudaGetErrorString(e));
  GemmArgs a{xq, xs, static_cast<const uint8_t *>(wq), w_scale, bias,
             bias ? bias_dtype : kNone, outs[0], out_dtype, M, N, K};
  a.ldo = ldo;
  a.n_peers = n_outs - 1;
  a.peers = outs + 1;
  a.weights_before_wait = true;  // the previous kernel is this call's quantizer
  return launch_gemm(a, s, true);
}

static_assert(sizeof(cudaIpcMemHandle_t) == FP8LIN_PEER_HANDLE_BYTES,
              "CUDA IPC handle size differs from FP8LIN_PEER_HANDLE_BYTES");

int fp8lin_peer_buffer_alloc(size_t bytes, void **ptr, unsigned char *handle_out) {
  clear_error();
  if (!ptr || !handle_out || bytes == 0)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "peer_buffer_alloc: null pointer or zero size");
  *ptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("peer_buffer_alloc: cudaMalloc: ") +
                                     cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(FP8LIN_ERR_CUDA, std::string("peer_buffer_alloc: cudaIpcGetMemHandle: ") +
                                     cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return FP8LIN_OK;
}

int fp8lin_peer_buffer_open(const unsigned char *handle, void **ptr) {
  clear_error();
  if (!ptr || !handle) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "peer_buffer_open: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("peer_buffer_open: cudaIpcOpenMemHandle: ") +
                                     cudaGetErrorString(e));
  *ptr = p;
  return FP8LIN_OK;
}

int fp8lin_peer_buffer_close(void *ptr) {
  clear_error();
  if (!ptr) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "peer_buffer_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("peer_buffer_close: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_peer_buffer_free(void *ptr) {
  clear_error();
  if (!ptr) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "peer_buffer_free: null pointer");
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("peer_buffer_free: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_selftest_watchdog(unsigned int limit_us, unsigned int *status, void *stream) {
  clear_error();
  if (!status) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "selftest_watchdog: null status");
  if (limit_us == 0 || limit_us > 1000000u)
    return fail(FP8LIN_ERR_INVALID_ARGUMENT, "selftest_watchdog: limit must be 1..1000000 us");
  cudaError_t e = launch_watchdog_selftest(limit_us, status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("selftest_watchdog: ") + cudaGetErrorString(e));
  return FP8LIN_OK;
}

int fp8lin_device_status(unsigned int *status, int clear) {
  clear_error();
  if (!status) return fail(FP8LIN_ERR_INVALID_ARGUMENT, "device_status: null pointer");
  unsigned int q = 0, sm = 0;
  cudaError_t e = read_gemm_status(status, clear != 0);
  if (e == cudaSuccess) e = read_quant_status(&q, clear != 0);
  if (e == cudaSuccess) e = read_small_status(&sm, clear != 0);
  if (e != cudaSuccess)
    return fail(FP8LIN_ERR_CUDA, std::string("device_status: ") + cudaGetErrorString(e));
  *status |= q | sm;
  return FP8LIN_OK;
}

}  // extern "C"
