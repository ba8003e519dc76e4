// torch_binding.cpp -- TORCH_LIBRARY registration of the reference's op surface on
// top of the C ABI in libfp8linear_b200.so.
//
// Same schemas as the reference (torch-ext/torch_binding.cpp:7-27), registered for
// the CUDA dispatch key only, under the namespace `fp8linear_b200`. Host code here
// only checks arguments (the reference's TORCH_CHECKs, csrc/quantize.cu:200-204 and
// csrc/fp8_gemm.cu:144-160), allocates outputs with the caching allocator and calls
// the C ABI on the current stream of the tensors' device. There is no CPU path and
// no fallback: a failing kernel call raises.
//
// Output dtype: the reference's fp8_gemm/fp8_linear always return fp16
// (csrc/fp8_gemm.cu:163). Here fp8_linear returns x's dtype (bf16 for bf16 input,
// fp16 for fp16 input) and fp8_gemm returns bf16.
//
// The reference's MXFP8 and NVFP4 schemas (torch-ext/torch_binding.cpp:30-65) are
// implemented the same way (block-scaled tcgen05 GEMMs; mxfp8_gemm / nvfp4_gemm return
// bf16, mxfp8_linear / nvfp4_linear x's dtype).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>
#include <torch/torch.h>

#include <cstdlib>

#include "fp8linear_b200.h"

namespace {

at::Tensor mxfp8_linear(at::Tensor x, at::Tensor wq, at::Tensor w_scales,
                        std::optional<at::Tensor> bias);
at::Tensor nvfp4_linear(at::Tensor x, at::Tensor wq, at::Tensor w_scales,
                        std::optional<at::Tensor> bias);

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return FP8LIN_DTYPE_BF16;
    case at::kHalf: return FP8LIN_DTYPE_F16;
    case at::kFloat: return FP8LIN_DTYPE_F32;
    default: return -2;
  }
}

void check_rc(int rc, const char *op) {
  TORCH_CHECK(rc == FP8LIN_OK, op, " failed (status ", rc, "): ", fp8lin_last_error());
}

void *stream_of(const at::Tensor &t) {
  return static_cast<void *>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// A fresh allocation is 16-byte aligned; a view with an odd storage offset may not be.
at::Tensor aligned16(const at::Tensor &t) {
  auto c = t.contiguous();
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
  return c;
}

std::tuple<at::Tensor, at::Tensor> quantize_fp8(at::Tensor x) {
  TORCH_CHECK(x.is_cuda(), "x must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() == 2, "x must be 2D [M, K]");
  c10::cuda::CUDAGuard guard(x.device());
  auto xc = x.contiguous();
  const int64_t M = xc.size(0), K = xc.size(1);
  auto xq = at::empty_like(xc, xc.options().dtype(at::kFloat8_e4m3fn));
  auto scale = at::empty({M}, xc.options().dtype(at::kFloat));
  if (M == 0 || K == 0) {
    if (M > 0) scale.fill_(1e-12f);  // an empty row has amax 0 -> the scale floor
    return {xq, scale};
  }
  check_rc(fp8lin_quantize_fp8(xc.data_ptr(), dtype_code(xc.scalar_type()), M, K, xq.data_ptr(),
                               scale.data_ptr<float>(), stream_of(xc)),
           "quantize_fp8");
  return {xq, scale};
}

std::tuple<at::Tensor, at::Tensor> quantize_mxfp8(at::Tensor x);
std::tuple<at::Tensor, at::Tensor> quantize_nvfp4(at::Tensor x);

// Per-channel by default; on an sm_100 device FP8LINEAR_USE_NVFP4 selects NVFP4 weights
// and, failing that, FP8LINEAR_USE_MX selects MXFP8 (the reference's opt-ins, in that
// order, csrc/quantize.cu:344-357; fp32 weights go through bf16 first).
std::tuple<at::Tensor, at::Tensor> quantize_weight(at::Tensor weight) {
  TORCH_CHECK(weight.is_cuda() && weight.dim() == 2, "weight must be a 2D CUDA tensor");
  if (at::cuda::getCurrentDeviceProperties()->major >= 10) {
    auto w = weight.scalar_type() == at::kFloat ? weight.to(at::kBFloat16) : weight;
    if (std::getenv("FP8LINEAR_USE_NVFP4") != nullptr) return quantize_nvfp4(w);
    if (std::getenv("FP8LINEAR_USE_MX") != nullptr) return quantize_mxfp8(w);
  }
  const int code = dtype_code(weight.scalar_type());
  TORCH_CHECK(code >= 0, "weight must be bf16, fp16 or fp32");
  c10::cuda::CUDAGuard guard(weight.device());
  auto w = weight.detach().contiguous();
  const int64_t N = w.size(0), K = w.size(1);
  auto wq = at::empty({N, K}, w.options().dtype(at::kFloat8_e4m3fn));
  auto scale = at::empty({N}, w.options().dtype(at::kFloat));
  if (N == 0) return {wq, scale};
  if (K == 0) {
    scale.fill_(1e-12f);
    return {wq, scale};
  }
  check_rc(fp8lin_quantize_weight(w.data_ptr(), code, N, K, wq.data_ptr(),
                                  scale.data_ptr<float>(), stream_of(w)),
           "quantize_weight");
  return {wq, scale};
}

struct BiasArg {
  at::Tensor t;
  const void *ptr = nullptr;
  int dtype = FP8LIN_DTYPE_NONE;
};

BiasArg prep_bias(const std::optional<at::Tensor> &bias, int64_t N) {
  BiasArg b;
  if (!bias.has_value() || !bias->defined()) return b;
  TORCH_CHECK(bias->is_cuda(), "bias must be on CUDA");
  TORCH_CHECK(bias->numel() == N, "bias must have N entries");
  b.t = bias->contiguous();
  if (dtype_code(b.t.scalar_type()) < 0) b.t = b.t.to(at::kFloat);
  b.ptr = b.t.data_ptr();
  b.dtype = dtype_code(b.t.scalar_type());
  return b;
}

at::Tensor gemm_impl(const at::Tensor &xq, const at::Tensor &x_scale, const at::Tensor &wq,
                     const at::Tensor &w_scale, const std::optional<at::Tensor> &bias,
                     at::ScalarType out_dtype) {
  TORCH_CHECK(xq.is_cuda() && wq.is_cuda(), "inputs must be on CUDA");
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn,
              "xq and wq must be float8_e4m3fn");
  TORCH_CHECK(xq.dim() == 2 && wq.dim() == 2, "xq, wq must be 2D");
  TORCH_CHECK(xq.size(1) == wq.size(1), "K mismatch: xq[M,K], wq[N,K]");
  c10::cuda::CUDAGuard guard(xq.device());
  auto xqc = aligned16(xq);
  auto wqc = aligned16(wq);
  const int64_t M = xqc.size(0), K = xqc.size(1), N = wqc.size(0);
  TORCH_CHECK(K % 16 == 0, "K must be a multiple of 16 for FP8 matmul, got ", K);
  auto xs = x_scale.contiguous();
  auto ws = w_scale.contiguous();
  TORCH_CHECK(xs.scalar_type() == at::kFloat && ws.scalar_type() == at::kFloat,
              "scales must be fp32");
  TORCH_CHECK(xs.numel() == M, "x_scale must have M entries (per-token)");
  TORCH_CHECK(ws.numel() == N, "w_scale must have N entries (per-channel)");
  TORCH_CHECK(xs.is_cuda() && ws.is_cuda(), "scales must be on CUDA");
  auto out = at::empty({M, N}, xqc.options().dtype(out_dtype));
  if (M == 0 || N == 0) return out;
  TORCH_CHECK(K > 0, "K must be positive");
  BiasArg b = prep_bias(bias, N);
  check_rc(fp8lin_fp8_gemm(xqc.data_ptr(), xs.data_ptr<float>(), wqc.data_ptr(),
                           ws.data_ptr<float>(), b.ptr, b.dtype, out.data_ptr(),
                           dtype_code(out_dtype), M, N, K, stream_of(xqc)),
           "fp8_gemm");
  return out;
}

at::Tensor fp8_gemm(at::Tensor xq, at::Tensor x_scale, at::Tensor wq, at::Tensor w_scale,
                    std::optional<at::Tensor> bias) {
  return gemm_impl(xq, x_scale, wq, w_scale, bias, at::kBFloat16);
}

at::Tensor fp8_linear(at::Tensor x, at::Tensor wq, at::Tensor w_scale,
                      std::optional<at::Tensor> bias) {
  TORCH_CHECK(x.is_cuda() && wq.is_cuda(), "inputs must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() >= 1, "x must have at least one dimension");
  // Dispatch on the weight format, as csrc/fp8_gemm.cu:203-216: uint8 scales with a packed
  // uint8 weight are NVFP4, with an e4m3 weight MXFP8.
  if (w_scale.scalar_type() == at::kByte) {
    if (wq.scalar_type() == at::kByte) return nvfp4_linear(x, wq, w_scale, bias);
    return mxfp8_linear(x, wq, w_scale, bias);
  }
  TORCH_CHECK(wq.scalar_type() == at::kFloat8_e4m3fn, "wq must be float8_e4m3fn");
  TORCH_CHECK(wq.dim() == 2, "wq must be 2D [N, K]");
  TORCH_CHECK(w_scale.scalar_type() == at::kFloat, "w_scale must be fp32");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t K = x.size(-1);
  TORCH_CHECK(wq.size(1) == K, "K mismatch: x[..., K], wq[N, K]");
  auto x2d = aligned16(x.reshape({-1, K}));
  auto wqc = aligned16(wq);
  const int64_t M = x2d.size(0), N = wqc.size(0);
  TORCH_CHECK(K % 16 == 0, "K must be a multiple of 16 for FP8 matmul, got ", K);
  auto ws = w_scale.contiguous();
  TORCH_CHECK(ws.numel() == N, "w_scale must have N entries (per-channel)");
  auto out_shape = x.sizes().vec();
  out_shape.back() = N;
  auto out = at::empty({M, N}, x2d.options());
  if (M > 0 && N > 0) {
    TORCH_CHECK(K > 0, "K must be positive");
    BiasArg b = prep_bias(bias, N);
    const size_t ws_bytes = fp8lin_linear_workspace_size(M, K);
    auto workspace = at::empty({static_cast<int64_t>(ws_bytes)}, x2d.options().dtype(at::kByte));
    check_rc(fp8lin_fp8_linear(x2d.data_ptr(), dtype_code(x2d.scalar_type()), wqc.data_ptr(),
                               ws.data_ptr<float>(), b.ptr, b.dtype, out.data_ptr(),
                               dtype_code(x2d.scalar_type()), M, N, K, workspace.data_ptr(),
                               ws_bytes, stream_of(x2d)),
             "fp8_linear");
  }
  return out.reshape(out_shape);
}

// quantize_mxfp8 (csrc/quantize.cu:239-285): same checks and outputs; the scale grid is
// written whole by the kernel (padding included), so it is allocated uninitialised
// instead of being prefilled with 127 as the reference does.
std::tuple<at::Tensor, at::Tensor> quantize_mxfp8(at::Tensor x) {
  TORCH_CHECK(x.is_cuda(), "x must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() == 2, "x must be 2D [M, K]");
  c10::cuda::CUDAGuard guard(x.device());
  auto xc = aligned16(x);
  const int64_t M = xc.size(0), K = xc.size(1);
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32 for MXFP8, got ", K);
  auto xq = at::empty_like(xc, xc.options().dtype(at::kFloat8_e4m3fn));
  const int64_t sf_bytes = (M + 127) / 128 * ((K / 32 + 3) / 4) * 512;
  if (M == 0 || K == 0) {
    return {xq, at::full({sf_bytes}, 127, xc.options().dtype(at::kByte))};
  }
  auto scales = at::empty({sf_bytes}, xc.options().dtype(at::kByte));
  check_rc(fp8lin_quantize_mxfp8(xc.data_ptr(), dtype_code(xc.scalar_type()), M, K,
                                 xq.data_ptr(), scales.data_ptr(), stream_of(xc)),
           "quantize_mxfp8");
  return {xq, scales};
}
int64_t mx_scale_bytes(int64_t rows, int64_t K) {
  return (rows + 127) / 128 * ((K / 32 + 3) / 4) * 512;
}

// mxfp8_gemm (csrc/fp8_gemm.cu:233-333): the reference's checks; bf16 out (the reference
// writes fp16).
at::Tensor mxfp8_gemm(at::Tensor xq, at::Tensor x_scales, at::Tensor wq, at::Tensor w_scales,
                      std::optional<at::Tensor> bias) {
  TORCH_CHECK(xq.is_cuda() && wq.is_cuda(), "inputs must be on CUDA");
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn,
              "xq and wq must be float8_e4m3fn");
  TORCH_CHECK(xq.dim() == 2 && wq.dim() == 2, "xq, wq must be 2D");
  TORCH_CHECK(xq.size(1) == wq.size(1), "K mismatch: xq[M,K], wq[N,K]");
  c10::cuda::CUDAGuard guard(xq.device());
  auto xqc = aligned16(xq);
  auto wqc = aligned16(wq);
  const int64_t M = xqc.size(0), K = xqc.size(1), N = wqc.size(0);
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32 for MXFP8, got ", K);
  TORCH_CHECK(x_scales.scalar_type() == at::kByte && w_scales.scalar_type() == at::kByte,
              "MX scales must be uint8 (e8m0)");
  auto xs = aligned16(x_scales);
  auto ws = aligned16(w_scales);
  TORCH_CHECK(xs.numel() == mx_scale_bytes(M, K),
              "x_scales has wrong size for tiled MX layout (expected ", mx_scale_bytes(M, K),
              ", got ", xs.numel(), ")");
  TORCH_CHECK(ws.numel() == mx_scale_bytes(N, K),
              "w_scales has wrong size for tiled MX layout (expected ", mx_scale_bytes(N, K),
              ", got ", ws.numel(), ")");
  auto out = at::empty({M, N}, xqc.options().dtype(at::kBFloat16));
  if (M == 0 || N == 0) return out;
  TORCH_CHECK(K > 0, "K must be positive");
  BiasArg b = prep_bias(bias, N);
  check_rc(fp8lin_mxfp8_gemm(xqc.data_ptr(), xs.data_ptr(), wqc.data_ptr(), ws.data_ptr(), b.ptr,
                             b.dtype, out.data_ptr(), FP8LIN_DTYPE_BF16, M, N, K, stream_of(xqc)),
           "mxfp8_gemm");
  return out;
}

// mxfp8_linear (csrc/fp8_gemm.cu:335-345): x [..., K] -> [..., N] in x.dtype.
at::Tensor mxfp8_linear(at::Tensor x, at::Tensor wq, at::Tensor w_scales,
                        std::optional<at::Tensor> bias) {
  TORCH_CHECK(x.is_cuda() && wq.is_cuda(), "inputs must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() >= 1, "x must have at least one dimension");
  TORCH_CHECK(wq.scalar_type() == at::kFloat8_e4m3fn, "wq must be float8_e4m3fn");
  TORCH_CHECK(wq.dim() == 2, "wq must be 2D [N, K]");
  TORCH_CHECK(w_scales.scalar_type() == at::kByte, "MX scales must be uint8 (e8m0)");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t K = x.size(-1);
  TORCH_CHECK(wq.size(1) == K, "K mismatch: x[..., K], wq[N, K]");
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32 for MXFP8, got ", K);
  auto x2d = aligned16(x.reshape({-1, K}));
  auto wqc = aligned16(wq);
  auto ws = aligned16(w_scales);
  const int64_t M = x2d.size(0), N = wqc.size(0);
  TORCH_CHECK(ws.numel() == mx_scale_bytes(N, K),
              "w_scales has wrong size for tiled MX layout (expected ", mx_scale_bytes(N, K),
              ", got ", ws.numel(), ")");
  auto out_shape = x.sizes().vec();
  out_shape.back() = N;
  auto out = at::empty({M, N}, x2d.options());
  if (M > 0 && N > 0) {
    TORCH_CHECK(K > 0, "K must be positive");
    BiasArg b = prep_bias(bias, N);
    const size_t ws_bytes = fp8lin_mxfp8_linear_workspace_size(M, K);
    auto workspace = at::empty({static_cast<int64_t>(ws_bytes)}, x2d.options().dtype(at::kByte));
    check_rc(fp8lin_mxfp8_linear(x2d.data_ptr(), dtype_code(x2d.scalar_type()), wqc.data_ptr(),
                                 ws.data_ptr(), b.ptr, b.dtype, out.data_ptr(),
                                 dtype_code(x2d.scalar_type()), M, N, K, workspace.data_ptr(),
                                 ws_bytes, stream_of(x2d)),
             "mxfp8_linear");
  }
  return out.reshape(out_shape);
}
int64_t nv_scale_bytes(int64_t rows, int64_t K) {
  return (rows + 127) / 128 * ((K / 16 + 3) / 4) * 512;
}

// quantize_nvfp4 (csrc/quantize.cu:290-334): xq [M, K/2] packed e2m1, the ue4m3 scale grid
// written whole by the kernel (the reference prefills it with 0x38).
std::tuple<at::Tensor, at::Tensor> quantize_nvfp4(at::Tensor x) {
  TORCH_CHECK(x.is_cuda(), "x must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() == 2, "x must be 2D [M, K]");
  c10::cuda::CUDAGuard guard(x.device());
  auto xc = aligned16(x);
  const int64_t M = xc.size(0), K = xc.size(1);
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32 for NVFP4, got ", K);
  auto xq = at::empty({M, K / 2}, xc.options().dtype(at::kByte));
  const int64_t sf_bytes = nv_scale_bytes(M, K);
  if (M == 0 || K == 0) {
    return {xq, at::full({sf_bytes}, 0x38, xc.options().dtype(at::kByte))};
  }
  auto scales = at::empty({sf_bytes}, xc.options().dtype(at::kByte));
  check_rc(fp8lin_quantize_nvfp4(xc.data_ptr(), dtype_code(xc.scalar_type()), M, K,
                                 xq.data_ptr(), scales.data_ptr(), stream_of(xc)),
           "quantize_nvfp4");
  return {xq, scales};
}

// nvfp4_gemm (csrc/fp8_gemm.cu:352-445): the reference's checks; bf16 out (the reference
// writes fp16).
at::Tensor nvfp4_gemm(at::Tensor xq, at::Tensor x_scales, at::Tensor wq, at::Tensor w_scales,
                      std::optional<at::Tensor> bias) {
  TORCH_CHECK(xq.is_cuda() && wq.is_cuda(), "inputs must be on CUDA");
  TORCH_CHECK(xq.scalar_type() == at::kByte && wq.scalar_type() == at::kByte,
              "xq and wq must be packed uint8 (two e2m1 per byte)");
  TORCH_CHECK(xq.dim() == 2 && wq.dim() == 2, "xq, wq must be 2D");
  c10::cuda::CUDAGuard guard(xq.device());
  auto xqc = aligned16(xq);
  auto wqc = aligned16(wq);
  const int64_t M = xqc.size(0), K = xqc.size(1) * 2, N = wqc.size(0);
  TORCH_CHECK(wqc.size(1) * 2 == K, "K mismatch: xq[M,K/2], wq[N,K/2]");
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32 for NVFP4, got ", K);
  TORCH_CHECK(x_scales.scalar_type() == at::kByte && w_scales.scalar_type() == at::kByte,
              "NVFP4 scales must be uint8 (e4m3)");
  auto xs = aligned16(x_scales);
  auto ws = aligned16(w_scales);
  TORCH_CHECK(xs.numel() == nv_scale_bytes(M, K),
              "x_scales has wrong size for tiled NVFP4 layout (expected ", nv_scale_bytes(M, K),
              ", got ", xs.numel(), ")");
  TORCH_CHECK(ws.numel() == nv_scale_bytes(N, K),
              "w_scales has wrong size for tiled NVFP4 layout (expected ", nv_scale_bytes(N, K),
              ", got ", ws.numel(), ")");
  auto out = at::empty({M, N}, xqc.options().dtype(at::kBFloat16));
  if (M == 0 || N == 0) return out;
  TORCH_CHECK(K > 0, "K must be positive");
  BiasArg b = prep_bias(bias, N);
  check_rc(fp8lin_nvfp4_gemm(xqc.data_ptr(), xs.data_ptr(), wqc.data_ptr(), ws.data_ptr(), b.ptr,
                             b.dtype, out.data_ptr(), FP8LIN_DTYPE_BF16, M, N, K, stream_of(xqc)),
           "nvfp4_gemm");
  return out;
}

// nvfp4_linear (csrc/fp8_gemm.cu:447-457): x [..., K] -> [..., N] in x.dtype; wq [N, K/2].
at::Tensor nvfp4_linear(at::Tensor x, at::Tensor wq, at::Tensor w_scales,
                        std::optional<at::Tensor> bias) {
  TORCH_CHECK(x.is_cuda() && wq.is_cuda(), "inputs must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() >= 1, "x must have at least one dimension");
  TORCH_CHECK(wq.scalar_type() == at::kByte, "wq must be packed uint8 (two e2m1 per byte)");
  TORCH_CHECK(wq.dim() == 2, "wq must be 2D [N, K/2]");
  TORCH_CHECK(w_scales.scalar_type() == at::kByte, "NVFP4 scales must be uint8 (e4m3)");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t K = x.size(-1);
  TORCH_CHECK(wq.size(1) * 2 == K, "K mismatch: x[..., K], wq[N, K/2]");
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32 for NVFP4, got ", K);
  auto x2d = aligned16(x.reshape({-1, K}));
  auto wqc = aligned16(wq);
  auto ws = aligned16(w_scales);
  const int64_t M = x2d.size(0), N = wqc.size(0);
  TORCH_CHECK(ws.numel() == nv_scale_bytes(N, K),
              "w_scales has wrong size for tiled NVFP4 layout (expected ", nv_scale_bytes(N, K),
              ", got ", ws.numel(), ")");
  auto out_shape = x.sizes().vec();
  out_shape.back() = N;
  auto out = at::empty({M, N}, x2d.options());
  if (M > 0 && N > 0) {
    TORCH_CHECK(K > 0, "K must be positive");
    BiasArg b = prep_bias(bias, N);
    const size_t ws_bytes = fp8lin_nvfp4_linear_workspace_size(M, K);
    auto workspace = at::empty({static_cast<int64_t>(ws_bytes)}, x2d.options().dtype(at::kByte));
    check_rc(fp8lin_nvfp4_linear(x2d.data_ptr(), dtype_code(x2d.scalar_type()), wqc.data_ptr(),
                                 ws.data_ptr(), b.ptr, b.dtype, out.data_ptr(),
                                 dtype_code(x2d.scalar_type()), M, N, K, workspace.data_ptr(),
                                 ws_bytes, stream_of(x2d)),
             "nvfp4_linear");
  }
  return out.reshape(out_shape);
}

// Modulated input (no reference op; it fuses the chain that feeds Fp8Linear in a FLUX
// block): x [B, T, K] or [M, K], shift and scale [B, K] of x's dtype (B divides M).
struct ModArgs {
  at::Tensor x2d, shift, scale;
  int64_t M = 0, K = 0, B = 0;
};

ModArgs prep_modulation(const at::Tensor &x, const at::Tensor &shift, const at::Tensor &scale,
                        const char *op) {
  TORCH_CHECK(x.is_cuda() && shift.is_cuda() && scale.is_cuda(), op, ": inputs must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kHalf || x.scalar_type() == at::kBFloat16,
              op, ": x must be fp16 or bf16");
  TORCH_CHECK(shift.scalar_type() == x.scalar_type() && scale.scalar_type() == x.scalar_type(),
              op, ": shift and scale must have x's dtype");
  TORCH_CHECK(x.dim() == 2 || x.dim() == 3, op, ": x must be [M, K] or [B, T, K]");
  TORCH_CHECK(shift.dim() == 2 && scale.dim() == 2 && shift.sizes() == scale.sizes(),
              op, ": shift and scale must be [B, K]");
  ModArgs a;
  a.K = x.size(-1);
  a.B = shift.size(0);
  TORCH_CHECK(shift.size(1) == a.K, op, ": shift/scale width must equal x's last dim");
  if (x.dim() == 3) TORCH_CHECK(x.size(0) == a.B, op, ": x [B, T, K] needs shift/scale [B, K]");
  a.x2d = aligned16(x.reshape({-1, a.K}));
  a.M = a.x2d.size(0);
  TORCH_CHECK(a.B > 0 && a.M % a.B == 0, op, ": the batch count must divide the rows");
  TORCH_CHECK(a.K % 8 == 0 && a.K > 0 && a.K <= 8192, op,
              ": K must be a positive multiple of 8 up to 8192, got ", a.K);
  a.shift = aligned16(shift);
  a.scale = aligned16(scale);
  return a;
}

std::tuple<at::Tensor, at::Tensor> layernorm_modulate_quantize_fp8(at::Tensor x, at::Tensor shift,
                                                                   at::Tensor scale, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  ModArgs a = prep_modulation(x, shift, scale, "layernorm_modulate_quantize_fp8");
  auto xq = at::empty({a.M, a.K}, a.x2d.options().dtype(at::kFloat8_e4m3fn));
  auto xs = at::empty({a.M}, a.x2d.options().dtype(at::kFloat));
  if (a.M == 0) return {xq, xs};
  check_rc(fp8lin_layernorm_modulate_quantize_fp8(
               a.x2d.data_ptr(), dtype_code(a.x2d.scalar_type()), a.M, a.K, a.B,
               a.shift.data_ptr(), a.scale.data_ptr(), static_cast<float>(eps), xq.data_ptr(),
               xs.data_ptr<float>(), stream_of(a.x2d)),
           "layernorm_modulate_quantize_fp8");
  return {xq, xs};
}

at::Tensor fp8_linear_modulated(at::Tensor x, at::Tensor shift, at::Tensor scale, at::Tensor wq,
                                at::Tensor w_scale, std::optional<at::Tensor> bias, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  ModArgs a = prep_modulation(x, shift, scale, "fp8_linear_modulated");
  TORCH_CHECK(wq.is_cuda() && wq.scalar_type() == at::kFloat8_e4m3fn && wq.dim() == 2,
              "fp8_linear_modulated: wq must be a 2D float8_e4m3fn CUDA tensor");
  TORCH_CHECK(wq.size(1) == a.K, "K mismatch: x[..., K], wq[N, K]");
  TORCH_CHECK(w_scale.scalar_type() == at::kFloat, "w_scale must be fp32");
  auto wqc = aligned16(wq);
  auto ws = w_scale.contiguous();
  const int64_t N = wqc.size(0);
  TORCH_CHECK(ws.numel() == N, "w_scale must have N entries (per-channel)");
  auto out_shape = x.sizes().vec();
  out_shape.back() = N;
  auto out = at::empty({a.M, N}, a.x2d.options());
  if (a.M > 0 && N > 0) {
    BiasArg b = prep_bias(bias, N);
    const size_t ws_bytes = fp8lin_linear_workspace_size(a.M, a.K);
    auto workspace =
        at::empty({static_cast<int64_t>(ws_bytes)}, a.x2d.options().dtype(at::kByte));
    check_rc(fp8lin_fp8_linear_modulated(
                 a.x2d.data_ptr(), dtype_code(a.x2d.scalar_type()), a.M, a.K, a.B,
                 a.shift.data_ptr(), a.scale.data_ptr(), static_cast<float>(eps), wqc.data_ptr(),
                 ws.data_ptr<float>(), b.ptr, b.dtype, out.data_ptr(),
                 dtype_code(a.x2d.scalar_type()), N, workspace.data_ptr(), ws_bytes,
                 stream_of(a.x2d)),
             "fp8_linear_modulated");
  }
  return out.reshape(out_shape);
}

}  // namespace

TORCH_LIBRARY(fp8linear_b200, m) {
  m.def("quantize_fp8(Tensor x) -> (Tensor, Tensor)");
  m.def("quantize_weight(Tensor weight) -> (Tensor, Tensor)");
  m.def("fp8_gemm(Tensor xq, Tensor x_scale, Tensor wq, Tensor w_scale, Tensor? bias) -> Tensor");
  m.def("fp8_linear(Tensor x, Tensor wq, Tensor w_scale, Tensor? bias) -> Tensor");
  m.def("quantize_mxfp8(Tensor x) -> (Tensor, Tensor)");
  m.def("mxfp8_gemm(Tensor xq, Tensor x_scales, Tensor wq, Tensor w_scales, Tensor? bias) -> Tensor");
  m.def("mxfp8_linear(Tensor x, Tensor wq, Tensor w_scales, Tensor? bias) -> Tensor");
  m.def("quantize_nvfp4(Tensor x) -> (Tensor, Tensor)");
  m.def("nvfp4_gemm(Tensor xq, Tensor x_scales, Tensor wq, Tensor w_scales, Tensor? bias) -> Tensor");
  m.def("nvfp4_linear(Tensor x, Tensor wq, Tensor w_scales, Tensor? bias) -> Tensor");
  m.def("layernorm_modulate_quantize_fp8(Tensor x, Tensor shift, Tensor scale, float eps=1e-06) "
        "-> (Tensor, Tensor)");
  m.def("fp8_linear_modulated(Tensor x, Tensor shift, Tensor scale, Tensor wq, Tensor w_scale, "
        "Tensor? bias, float eps=1e-06) -> Tensor");
}

TORCH_LIBRARY_IMPL(fp8linear_b200, CUDA, m) {
  m.impl("quantize_fp8", &quantize_fp8);
  m.impl("quantize_weight", &quantize_weight);
  m.impl("fp8_gemm", &fp8_gemm);
  m.impl("fp8_linear", &fp8_linear);
  m.impl("quantize_mxfp8", &quantize_mxfp8);
  m.impl("mxfp8_gemm", &mxfp8_gemm);
  m.impl("mxfp8_linear", &mxfp8_linear);
  m.impl("quantize_nvfp4", &quantize_nvfp4);
  m.impl("nvfp4_gemm", &nvfp4_gemm);
  m.impl("nvfp4_linear", &nvfp4_linear);
  m.impl("layernorm_modulate_quantize_fp8", &layernorm_modulate_quantize_fp8);
  m.impl("fp8_linear_modulated", &fp8_linear_modulated);
}
