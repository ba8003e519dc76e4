// quantize.cu -- per-token e4m3 activation quantizer and per-channel weight quantizer
// for sm_100a.
//
// Activation path (replaces quant_rowwise_kernel, csrc/quantize.cu:45-73 of the
// reference): each row is read from HBM exactly once with 128-bit loads and held in
// registers; its absmax is reduced with warp shuffles (plus one shared-memory step
// when a row spans several warps); the codes are written as packed 8-byte stores.
// Arithmetic is the reference's, operation for operation, so codes and scales are
// bit-identical:
//   amax = fmaxf-reduce |x|           (NaN inputs ignored, as fmaxf does)
//   sc   = fmaxf(amax / 448, 1e-12)   (IEEE divide)
//   inv  = 1 / sc                     (IEEE divide)
//   q    = e4m3_rn_satfinite(fminf(fmaxf(x * inv, -448), 448))
// Max-reduction over non-negative values is order independent, so the different
// reduction tree does not change the result.
//
// Weight path (replaces the ATen ops of quantize_weight, csrc/quantize.cu:359-365):
// same shape of kernel, with ATen's CUDA semantics: NaN propagates through amax and
// both clamps, the scalar divide by 448 is a multiply by the fp32 reciprocal, and the
// per-element divide is a true IEEE divide.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "ptx.cuh"

namespace fp8lin {
namespace {

constexpr int kRowsBlock = 256;  // threads per CTA target for the vector kernel

template <typename T>
struct In;

template <>
struct In<__nv_bfloat16> {
  // 8 bf16 in a uint4 -> 8 floats (exact)
  __device__ __forceinline__ static void unpack8(const uint4 &v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __device__ __forceinline__ static float load1(const void *p, int64_t i) {
    const uint16_t b = reinterpret_cast<const uint16_t *>(p)[i];
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
  }
};

template <>
struct In<__half> {
  __device__ __forceinline__ static void unpack8(const uint4 &v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ __forceinline__ static float load1(const void *p, int64_t i) {
    return __half2float(reinterpret_cast<const __half *>(p)[i]);
  }
};

template <>
struct In<float> {
  __device__ __forceinline__ static float load1(const void *p, int64_t i) {
    return reinterpret_cast<const float *>(p)[i];
  }
};

__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float quant_clamp(float x, float inv) {
  const float v = __fmul_rn(x, inv);
  return fminf(fmaxf(v, -kE4M3Max), kE4M3Max);
}

// Vector kernel: TPR threads per row (multiple of 32), VPT 16-byte vectors per
// thread, rows_per_cta = blockDim.x / TPR rows per CTA. Row r's vector j
// (8 elements) is held by thread (j % TPR) as its (j / TPR)-th register vector.
template <typename T, int VPT>
__global__ void __launch_bounds__(1024) quant_rows_vec_kernel(const T *__restrict__ x,
                                                              uint8_t *__restrict__ xq,
                                                              float *__restrict__ scale,
                                                              int64_t M, int K, int tpr,
                                                              int trigger) {
  if (trigger) ptx::grid_launch_dependents();
  __shared__ float red[32];
  const int t_in_row = threadIdx.x % tpr;
  const int row_in_cta = threadIdx.x / tpr;
  const int rows_per_cta = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_cta + row_in_cta;
  const bool row_ok = row < M;
  const int nvec = K >> 3;
  const T *xr = x + (row_ok ? row : 0) * static_cast<int64_t>(K);

  uint4 v[VPT];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int j = t_in_row + i * tpr;
    if (row_ok && j < nvec) {
      v[i] = ld_stream_v4(xr + static_cast<int64_t>(j) * 8);
      float f[8];
      In<T>::unpack8(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    }
  }
  amax = warp_max(amax);
  const int warps_per_row = tpr >> 5;
  if (warps_per_row > 1) {
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    const int base = row_in_cta * warps_per_row;
    amax = red[base];
    for (int w = 1; w < warps_per_row; ++w) amax = fmaxf(amax, red[base + w]);
  }
  if (!row_ok) return;

  const float sc = fmaxf(__fdiv_rn(amax, kE4M3Max), kScaleFloor);
  const float inv = __fdiv_rn(1.0f, sc);
  if (t_in_row == 0) scale[row] = sc;

  uint8_t *qr = xq + row * static_cast<int64_t>(K);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int j = t_in_row + i * tpr;
    if (j < nvec) {
      float f[8];
      In<T>::unpack8(v[i], f);
      uint2 o;
      o.x = static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[0], inv), quant_clamp(f[1], inv))) |
            (static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[2], inv), quant_clamp(f[3], inv)))
             << 16);
      o.y = static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[4], inv), quant_clamp(f[5], inv))) |
            (static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[6], inv), quant_clamp(f[7], inv)))
             << 16);
      *reinterpret_cast<uint2 *>(qr + static_cast<int64_t>(j) * 8) = o;
    }
  }
}

// Generic kernel for any K / alignment: one CTA per row, two passes over the row
// (the second mostly from L2), scalar 2-byte loads. Same arithmetic.
template <typename T>
__global__ void __launch_bounds__(256) quant_rows_generic_kernel(const T *__restrict__ x,
                                                                 uint8_t *__restrict__ xq,
                                                                 float *__restrict__ scale,
                                                                 int64_t M, int64_t K,
                                                                 int trigger) {
  if (trigger) ptx::grid_launch_dependents();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const T *xr = x + row * K;
  float amax = 0.0f;
  for (int64_t j = threadIdx.x; j < K; j += blockDim.x)
    amax = fmaxf(amax, fabsf(In<T>::load1(xr, j)));
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
  for (int w = 1; w < (blockDim.x >> 5); ++w) amax = fmaxf(amax, red[w]);
  const float sc = fmaxf(__fdiv_rn(amax, kE4M3Max), kScaleFloor);
  const float inv = __fdiv_rn(1.0f, sc);
  if (threadIdx.x == 0) scale[row] = sc;
  uint8_t *qr = xq + row * K;
  for (int64_t j = threadIdx.x; j < K; j += blockDim.x) {
    const float c = quant_clamp(In<T>::load1(xr, j), inv);
    qr[j] = static_cast<uint8_t>(ptx::cvt_e4m3x2(c, 0.0f) & 0xFFu);
  }
}

// ---------------------------------------------------------------- weight path

// NaN-propagating clamp (ATen clamp / clamp_min semantics).
__device__ __forceinline__ float aten_clamp(float v, float lo, float hi) {
  return isnan(v) ? v : fminf(fmaxf(v, lo), hi);
}

template <typename T>
__global__ void __launch_bounds__(256) quant_weight_kernel(const T *__restrict__ w,
                                                           uint8_t *__restrict__ wq,
                                                           float *__restrict__ scale,
                                                           int64_t N, int64_t K) {
  __shared__ float red[8];
  __shared__ int red_nan[8];
  const int64_t row = blockIdx.x;
  const T *wr = w + row * K;
  float amax = 0.0f;
  int has_nan = 0;
  for (int64_t j = threadIdx.x; j < K; j += blockDim.x) {
    const float a = fabsf(In<T>::load1(wr, j));
    if (isnan(a)) has_nan = 1;
    else amax = fmaxf(amax, a);
  }
  amax = warp_max(amax);
  has_nan = __any_sync(0xffffffffu, has_nan);
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = amax;
    red_nan[threadIdx.x >> 5] = has_nan;
  }
  __syncthreads();
  amax = red[0];
  has_nan = red_nan[0];
  for (int i = 1; i < (blockDim.x >> 5); ++i) {
    amax = fmaxf(amax, red[i]);
    has_nan |= red_nan[i];
  }
  // ATen on CUDA: tensor / python-scalar multiplies by the fp32 reciprocal.
  constexpr float kInv448 = 1.0f / kE4M3Max;
  const float s = has_nan ? __int_as_float(0x7fffffff) : __fmul_rn(amax, kInv448);
  const float sc = isnan(s) ? s : fmaxf(s, kScaleFloor);
  if (threadIdx.x == 0) scale[row] = sc;
  uint8_t *qr = wq + row * K;
  for (int64_t j = threadIdx.x; j < K; j += blockDim.x) {
    const float q = __fdiv_rn(In<T>::load1(wr, j), sc);
    const float c = aten_clamp(q, -kE4M3Max, kE4M3Max);
    // In range after the clamp, so RN-satfinite equals ATen's non-saturating cast;
    // NaN encodes as 0x7F in both.
    qr[j] = static_cast<uint8_t>(ptx::cvt_e4m3x2(c, 0.0f) & 0xFFu);
  }
}

template <typename T>
cudaError_t launch_rows_typed(const void *x, int64_t M, int64_t K, uint8_t *xq, float *scale,
                              cudaStream_t stream, bool trigger) {
  const T *xp = reinterpret_cast<const T *>(x);
  const int64_t nvec = K / 8;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(xq) % 8 == 0);
  int vpt = nvec >= 256 ? 8 : nvec >= 128 ? 4 : nvec >= 64 ? 2 : 1;
  int64_t tpr = ((nvec + vpt - 1) / vpt + 31) / 32 * 32;
  if (K % 8 == 0 && aligned && tpr <= 1024) {
    const int rows_per_cta = tpr >= kRowsBlock ? 1 : static_cast<int>(kRowsBlock / tpr);
    const int threads = static_cast<int>(tpr) * rows_per_cta;
    const int64_t blocks = (M + rows_per_cta - 1) / rows_per_cta;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>(blocks));
    const int ik = static_cast<int>(K), it = static_cast<int>(tpr), trig = trigger ? 1 : 0;
    switch (vpt) {
      case 8: quant_rows_vec_kernel<T, 8><<<grid, threads, 0, stream>>>(xp, xq, scale, M, ik, it, trig); break;
      case 4: quant_rows_vec_kernel<T, 4><<<grid, threads, 0, stream>>>(xp, xq, scale, M, ik, it, trig); break;
      case 2: quant_rows_vec_kernel<T, 2><<<grid, threads, 0, stream>>>(xp, xq, scale, M, ik, it, trig); break;
      default: quant_rows_vec_kernel<T, 1><<<grid, threads, 0, stream>>>(xp, xq, scale, M, ik, it, trig); break;
    }
  } else {
    if (M > 0x7fffffffLL) return cudaErrorInvalidValue;
    quant_rows_generic_kernel<T><<<static_cast<unsigned>(M), 256, 0, stream>>>(
        xp, xq, scale, M, K, trigger ? 1 : 0);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quantize_rows(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                                 float *scale, cudaStream_t stream, bool trigger_dependents) {
  if (M == 0) return cudaSuccess;
  if (dtype == kBF16)
    return launch_rows_typed<__nv_bfloat16>(x, M, K, xq, scale, stream, trigger_dependents);
  return launch_rows_typed<__half>(x, M, K, xq, scale, stream, trigger_dependents);
}

cudaError_t launch_quantize_weight(const void *w, int dtype, int64_t N, int64_t K, uint8_t *wq,
                                   float *scale, cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  if (N > 0x7fffffffLL) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(N));
  switch (dtype) {
    case kBF16:
      quant_weight_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          reinterpret_cast<const __nv_bfloat16 *>(w), wq, scale, N, K);
      break;
    case kF16:
      quant_weight_kernel<__half><<<grid, 256, 0, stream>>>(reinterpret_cast<const __half *>(w),
                                                            wq, scale, N, K);
      break;
    default:
      quant_weight_kernel<float><<<grid, 256, 0, stream>>>(reinterpret_cast<const float *>(w),
                                                           wq, scale, N, K);
      break;
  }
  return cudaGetLastError();
}

}  // namespace fp8lin
