// noalloc.cu -- fp8lin_fp8_linear_noalloc: the fused FP8 linear for callers that
// cannot allocate device memory.
//
// fp8lin_fp8_linear needs a workspace for the activations' e4m3 codes and per-token
// scales, and asks the caller to provide it. Some callers cannot: a plugin or custom-op
// interface that hands the op only its input and output buffers and owns all other
// device memory through its own pool, or a latency-critical path where cudaMalloc's
// implicit device synchronisation is not acceptable. For them this entry point takes
// the workspace from a fixed array in device memory that is part of this library
// (FP8LIN_NOALLOC_SCRATCH_BYTES = 64 MiB; every GPU that loads the library keeps it
// until the process exits).
//
// Rules that follow from a single shared array:
//  * sizes whose workspace (fp8lin_linear_workspace_size(M, K)) exceeds the array
//    are rejected with FP8LIN_ERR_WORKSPACE;
//  * every call on a device uses the same array, so calls whose GPU work overlaps
//    (other streams, other host threads) race on it; serialise them;
//  * the array keeps the previous call's contents. Nothing in it needs to start at
//    zero: the quantizer writes every code and scale the GEMM then reads.
//  * the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that first
//    call before any stream capture.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "fp8linear_b200.h"
#include "internal.h"

namespace fp8lin {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FP8LIN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per
// device). The host-side symbol is only a handle, never a usable device pointer.
int scratch_on_current_device(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error(std::string("fp8_linear_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    return FP8LIN_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("fp8_linear_noalloc: device ordinal out of range");
    return FP8LIN_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      set_error(std::string("fp8_linear_noalloc: cudaGetSymbolAddress: ") +
                cudaGetErrorString(e));
      return FP8LIN_ERR_CUDA;
    }
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return FP8LIN_OK;
}

}  // namespace
}  // namespace fp8lin

extern "C" int fp8lin_fp8_linear_noalloc(const void *x, int x_dtype, const void *wq,
                                         const float *w_scale, const void *bias,
                                         int bias_dtype, void *out, int out_dtype, int64_t M,
                                         int64_t N, int64_t K, void *stream) {
  fp8lin::clear_error();
  if (M < 0 || K < 0) {
    fp8lin::set_error("fp8_linear_noalloc: negative size");
    return FP8LIN_ERR_INVALID_ARGUMENT;
  }
  const size_t need = fp8lin_linear_workspace_size(M, K);
  if (need > static_cast<size_t>(FP8LIN_NOALLOC_SCRATCH_BYTES)) {
    fp8lin::set_error("fp8_linear_noalloc: M=" + std::to_string(M) + ", K=" + std::to_string(K) +
                      " needs " + std::to_string(need) +
                      " bytes of scratch, more than the fixed " +
                      std::to_string(static_cast<size_t>(FP8LIN_NOALLOC_SCRATCH_BYTES)) +
                      " bytes; use fp8lin_fp8_linear with a caller-provided workspace");
    return FP8LIN_ERR_WORKSPACE;
  }
  void *scratch = nullptr;
  if (M > 0 && N > 0) {
    const int rc = fp8lin::scratch_on_current_device(&scratch);
    if (rc != FP8LIN_OK) return rc;
  }
  return fp8lin_fp8_linear(x, x_dtype, wq, w_scale, bias, bias_dtype, out, out_dtype, M, N, K,
                           scratch, static_cast<size_t>(FP8LIN_NOALLOC_SCRATCH_BYTES), stream);
}
