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

#include <algorithm>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace fp8lin {

__device__ unsigned int g_quant_status;  // watchdog bit 8: a quantizer wait ran out

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

// ---------------------------------------------------------------- fast row path
//
// Rows whose values are all finite (the normal case) take a cheaper path that gives the
// same bits as the reference arithmetic:
//  * amax: with the sign bits cleared, finite bf16/fp16 values order like their bit
//    patterns read as unsigned integers, so a packed integer max (max.u16x2) over the
//    magnitudes' bits, converted back exactly, equals fmaxf-reduce over |x|. The same
//    max exposes a non-finite value in the row (bits above the largest finite pattern).
//  * q = cvt_satfinite(x * inv): x and inv are finite, so no product is NaN, and the
//    saturating convert maps anything beyond +-448 to +-448 exactly as the clamp
//    fminf(fmaxf(v, -448), 448) before it would. x * inv uses packed IEEE multiplies.
// Rows holding inf or NaN fall back to the literal clamp path (reference NaN/inf
// semantics: NaN is ignored by the amax and clamps to -448; an inf amax gives inv = 0).
template <typename T>
struct Bits;
template <>
struct Bits<__nv_bfloat16> {
  static constexpr uint32_t kMaxFinite = 0x7F7Fu;  // largest finite |bf16| pattern
  __device__ __forceinline__ static float to_float(uint32_t b) { return __uint_as_float(b << 16); }
};
template <>
struct Bits<__half> {
  static constexpr uint32_t kMaxFinite = 0x7BFFu;  // largest finite |fp16| pattern
  __device__ __forceinline__ static float to_float(uint32_t b) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
  }
};

// running max of the magnitude bit patterns of two packed 16-bit values
__device__ __forceinline__ uint32_t mag_max2(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("{.reg .b32 t;\n\tand.b32 t, %2, 0x7fff7fff;\n\tmax.u16x2 %0, %1, t;}"
      : "=r"(r)
      : "r"(acc), "r"(w));
  return r;
}

__device__ __forceinline__ uint32_t mag_max8(uint32_t acc, const uint4 &v) {
  acc = mag_max2(acc, v.x);
  acc = mag_max2(acc, v.y);
  acc = mag_max2(acc, v.z);
  return mag_max2(acc, v.w);
}

__device__ __forceinline__ uint32_t fold_halves(uint32_t acc) {
  const uint32_t lo = acc & 0xFFFFu, hi = acc >> 16;
  return lo > hi ? lo : hi;
}

// (a, b) * inv with one packed IEEE round-to-nearest multiply
__device__ __forceinline__ void mul2(float &a, float &b, float inv) {
  asm("{.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %4};\n\t"
      "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;}"
      : "=f"(a), "=f"(b)
      : "f"(a), "f"(b), "f"(inv));
}

// 8 finite values -> 8 e4m3 codes (fast path)
template <typename T>
__device__ __forceinline__ uint2 quant8_fast(const uint4 &v, float inv) {
  float f[8];
  In<T>::unpack8(v, f);
#pragma unroll
  for (int i = 0; i < 8; i += 2) mul2(f[i], f[i + 1], inv);
  uint2 o;
  o.x = static_cast<uint32_t>(ptx::cvt_e4m3x2(f[0], f[1])) |
        (static_cast<uint32_t>(ptx::cvt_e4m3x2(f[2], f[3])) << 16);
  o.y = static_cast<uint32_t>(ptx::cvt_e4m3x2(f[4], f[5])) |
        (static_cast<uint32_t>(ptx::cvt_e4m3x2(f[6], f[7])) << 16);
  return o;
}

// 8 values -> 8 e4m3 codes with the reference's literal clamp (any input)
template <typename T>
__device__ __forceinline__ uint2 quant8_clamp(const uint4 &v, float inv) {
  float f[8];
  In<T>::unpack8(v, f);
  uint2 o;
  o.x = static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[0], inv), quant_clamp(f[1], inv))) |
        (static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[2], inv), quant_clamp(f[3], inv)))
         << 16);
  o.y = static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[4], inv), quant_clamp(f[5], inv))) |
        (static_cast<uint32_t>(ptx::cvt_e4m3x2(quant_clamp(f[6], inv), quant_clamp(f[7], inv)))
         << 16);
  return o;
}

// fmaxf-reduce of |x| over 8 values (NaN ignored), the slow-path amax
template <typename T>
__device__ __forceinline__ float amax8_float(float amax, const uint4 &v) {
  float f[8];
  In<T>::unpack8(v, f);
#pragma unroll
  for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
  return amax;
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
  // trigger bit 0: let the dependent grid launch now; bit 1: this grid is itself a
  // programmatic dependent and waits for its prerequisite before touching memory
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  __shared__ uint32_t red[32];
  const int t_in_row = threadIdx.x % tpr;
  const int row_in_cta = threadIdx.x / tpr;
  const int rows_per_cta = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_cta + row_in_cta;
  const bool row_ok = row < M;
  const int nvec = K >> 3;
  const T *xr = x + (row_ok ? row : 0) * static_cast<int64_t>(K);

  uint4 v[VPT];
  uint32_t mb = 0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int j = t_in_row + i * tpr;
    if (row_ok && j < nvec) {
      v[i] = ld_stream_v4(xr + static_cast<int64_t>(j) * 8);
      mb = mag_max8(mb, v[i]);
    }
  }
  mb = __reduce_max_sync(0xffffffffu, fold_halves(mb));
  const int warps_per_row = tpr >> 5;
  bool finite;
  if (warps_per_row > 1) {
    // Rows span several warps: exchange the per-warp maxima. The fast/slow decision is
    // made for the whole CTA (any non-finite row -> every row takes the clamp path,
    // which is exact for all rows), so the slow path's barriers stay CTA-uniform.
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mb;
    __syncthreads();
    const int base = row_in_cta * warps_per_row;
    uint32_t rmb = 0, any_nonfinite = 0;
    for (int w = 0; w < warps_per_row; ++w) rmb = rmb > red[base + w] ? rmb : red[base + w];
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w)
      any_nonfinite |= red[w] > Bits<T>::kMaxFinite ? 1u : 0u;
    mb = rmb;
    finite = any_nonfinite == 0;
  } else {
    finite = mb <= Bits<T>::kMaxFinite;  // warp == row: warp-uniform
  }
  float amax;
  if (finite) {
    amax = Bits<T>::to_float(mb);
  } else {
    amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = t_in_row + i * tpr;
      if (row_ok && j < nvec) amax = amax8_float<T>(amax, v[i]);
    }
    amax = warp_max(amax);
    if (warps_per_row > 1) {
      __shared__ float redf[32];
      if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = amax;
      __syncthreads();
      const int base = row_in_cta * warps_per_row;
      amax = redf[base];
      for (int w = 1; w < warps_per_row; ++w) amax = fmaxf(amax, redf[base + w]);
    }
  }
  if (!row_ok) return;

  const float sc = fmaxf(__fdiv_rn(amax, kE4M3Max), kScaleFloor);
  const float inv = __fdiv_rn(1.0f, sc);
  if (t_in_row == 0) scale[row] = sc;

  uint8_t *qr = xq + row * static_cast<int64_t>(K);
  if (finite) {  // CTA-uniform: one conversion per value, not both and a select
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = t_in_row + i * tpr;
      if (j < nvec)
        *reinterpret_cast<uint2 *>(qr + static_cast<int64_t>(j) * 8) = quant8_fast<T>(v[i], inv);
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = t_in_row + i * tpr;
      if (j < nvec)
        *reinterpret_cast<uint2 *>(qr + static_cast<int64_t>(j) * 8) = quant8_clamp<T>(v[i], inv);
    }
  }
}

// ---------------------------------------------------------------- pipelined kernel
//
// Persistent and row-pipelined: a group of WPR warps owns rows g, g + G, g + 2G, ... (G
// groups in the grid) and keeps two rows in registers: the 16-byte loads of its next row
// are issued before the current row is reduced, converted and stored, so every group
// has a row in flight while it works and the grid never drains between waves. Thread t
// of a group holds vectors t + i * 32 * WPR (i < VPL) of a row: each warp load covers
// 512 contiguous bytes. The amax of a row spanning several warps is exchanged through
// shared memory under a named barrier of the group's threads (one barrier per row; the
// exchange slots alternate by row so a slot is rewritten only after every warp of the
// group has passed the next row's barrier). The fast/slow (non-finite) decision is made
// per row from the group's maximum, so the slow path's barriers stay group-uniform.
template <typename T, int VPL>
__device__ __forceinline__ void pipe_load(uint4 (&v)[VPL], const T *x, int64_t row, int64_t M,
                                          int K, int t, int stride) {
  if (row >= M) return;
  const T *xr = x + row * static_cast<int64_t>(K);
  const int nvec = K >> 3;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int j = t + i * stride;
    if (j < nvec) v[i] = ld_stream_v4(xr + static_cast<int64_t>(j) * 8);
  }
}

template <typename T, int VPL, int WPR>
__device__ __forceinline__ void pipe_row(const uint4 (&v)[VPL], uint8_t *xq, float *scale,
                                         int64_t row, int K, int t, int stride, int group,
                                         int parity, uint32_t (*redu)[WPR], float (*redf)[WPR]) {
  const int nvec = K >> 3;
  const int lane = t & 31, wi = t >> 5;
  uint32_t mb = 0;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (t + i * stride < nvec) mb = mag_max8(mb, v[i]);
  mb = __reduce_max_sync(0xffffffffu, fold_halves(mb));
  if constexpr (WPR > 1) {
    uint32_t *slot = redu[2 * group + parity];
    if (lane == 0) slot[wi] = mb;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(32 * WPR) : "memory");
#pragma unroll
    for (int w = 0; w < WPR; ++w) mb = mb > slot[w] ? mb : slot[w];
  }
  const bool finite = mb <= Bits<T>::kMaxFinite;  // group-uniform
  float amax;
  if (finite) {
    amax = Bits<T>::to_float(mb);
  } else {
    amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (t + i * stride < nvec) amax = amax8_float<T>(amax, v[i]);
    amax = warp_max(amax);
    if constexpr (WPR > 1) {
      float *slot = redf[2 * group + parity];
      if (lane == 0) slot[wi] = amax;
      asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(32 * WPR) : "memory");
      amax = slot[0];
#pragma unroll
      for (int w = 1; w < WPR; ++w) amax = fmaxf(amax, slot[w]);
    }
  }
  const float sc = fmaxf(__fdiv_rn(amax, kE4M3Max), kScaleFloor);
  const float inv = __fdiv_rn(1.0f, sc);
  if (t == 0) scale[row] = sc;
  uint8_t *qr = xq + row * static_cast<int64_t>(K);
  // two loops behind one warp-uniform branch: a select between the two conversions
  // inside one loop would evaluate both
  if (finite) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int j = t + i * stride;
      if (j < nvec)
        *reinterpret_cast<uint2 *>(qr + static_cast<int64_t>(j) * 8) = quant8_fast<T>(v[i], inv);
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int j = t + i * stride;
      if (j < nvec)
        *reinterpret_cast<uint2 *>(qr + static_cast<int64_t>(j) * 8) = quant8_clamp<T>(v[i], inv);
    }
  }
}

constexpr int kPipeThreads = 512;

// Two row buffers in registers, written out as two explicit halves of the loop body.
template <typename T, int VPL, int WPR>
__global__ void __launch_bounds__(kPipeThreads)
    quant_rows_pipe_kernel(const T *__restrict__ x, uint8_t *__restrict__ xq,
                           float *__restrict__ scale, int64_t M, int K, int trigger) {
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  // per group and row parity: one slot of WPR integer maxima and one of float maxima
  __shared__ uint32_t redu[2 * (kPipeThreads / 32)][WPR];
  __shared__ float redf[2 * (kPipeThreads / 32)][WPR];
  const int warp = threadIdx.x >> 5;
  const int group = warp / WPR;
  const int t = (warp % WPR) * 32 + (threadIdx.x & 31);
  const int stride = 32 * WPR;
  const int groups_per_cta = static_cast<int>(blockDim.x >> 5) / WPR;
  const int64_t G = static_cast<int64_t>(gridDim.x) * groups_per_cta;
  int64_t row = static_cast<int64_t>(blockIdx.x) * groups_per_cta + group;
  uint4 a[VPL], b[VPL];
  pipe_load<T, VPL>(a, x, row, M, K, t, stride);
  int parity = 0;
  while (row < M) {
    const int64_t r1 = row + G;
    pipe_load<T, VPL>(b, x, r1, M, K, t, stride);
    pipe_row<T, VPL, WPR>(a, xq, scale, row, K, t, stride, group, parity, redu, redf);
    parity ^= 1;
    if (r1 >= M) break;
    const int64_t r2 = r1 + G;
    pipe_load<T, VPL>(a, x, r2, M, K, t, stride);
    pipe_row<T, VPL, WPR>(b, xq, scale, r1, K, t, stride, group, parity, redu, redf);
    parity ^= 1;
    row = r2;
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// NB rows in flight per group through shared memory: each thread copies its own 16-byte
// vectors of a row with cp.async into its slots (stage[slot][i][thread], so a warp's
// copies and reads cover 512 contiguous bytes) and reads back only what it copied
// itself, so the data needs no barrier, only the thread's own cp.async.wait_group. One
// commit group per row (empty past M) keeps the group count uniform: after committing
// row r + (NB - 1) G, waiting until NB - 1 groups remain pending means row r has landed.
// `pf` / `pf_bytes`: a range the kernel launched after this one will read (the fused
// linear's weight matrix), brought into L2 before this grid's own dependency wait, one
// slice per CTA; L2 is where every SM's accesses to device memory meet, so this is safe
// even while the kernel before still writes the range.
template <typename T, int VPL, int WPR, int NB>
__global__ void __launch_bounds__(kPipeThreads)
    quant_rows_pipe_async_kernel(const T *__restrict__ x, uint8_t *__restrict__ xq,
                                 float *__restrict__ scale, int64_t M, int K, int trigger,
                                 const uint8_t *pf, int64_t pf_bytes) {
  if (pf_bytes > 0 && threadIdx.x == 0) {
    const int64_t slice = ((pf_bytes + gridDim.x - 1) / gridDim.x + 15) & ~int64_t{15};
    const int64_t off = static_cast<int64_t>(blockIdx.x) * slice;
    if (off < pf_bytes)
      ptx::bulk_prefetch_l2(pf + off, static_cast<uint32_t>(min(slice, pf_bytes - off)));
  }
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  extern __shared__ __align__(16) uint4 stage[];  // [NB][VPL][blockDim.x]
  __shared__ uint32_t redu[2 * (kPipeThreads / 32)][WPR];
  __shared__ float redf[2 * (kPipeThreads / 32)][WPR];
  const int warp = threadIdx.x >> 5;
  const int group = warp / WPR;
  const int t = (warp % WPR) * 32 + (threadIdx.x & 31);
  const int stride = 32 * WPR;
  const int nthr = static_cast<int>(blockDim.x);
  const int nvec = K >> 3;
  const int groups_per_cta = nthr / 32 / WPR;
  const int64_t G = static_cast<int64_t>(gridDim.x) * groups_per_cta;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * groups_per_cta + group;
  const uint32_t sbase = ptx::smem_u32(stage) + 16u * threadIdx.x;
  auto issue = [&](int64_t r, int slot) {
    if (r < M) {
      const T *xr = x + r * static_cast<int64_t>(K);
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int j = t + i * stride;
        if (j < nvec)
          cp_async16(sbase + 16u * static_cast<uint32_t>((slot * VPL + i) * nthr),
                     xr + static_cast<int64_t>(j) * 8);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < NB - 1; ++k) issue(row0 + k * G, k);
  int parity = 0, slot = 0;
  for (int64_t r = row0; r < M; r += G) {
    issue(r + (NB - 1) * G, slot == 0 ? NB - 1 : slot - 1);
    cp_async_wait<NB - 1>();
    uint4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (t + i * stride < nvec) v[i] = stage[(slot * VPL + i) * nthr + threadIdx.x];
    pipe_row<T, VPL, WPR>(v, xq, scale, r, K, t, stride, group, parity, redu, redf);
    parity ^= 1;
    slot = slot + 1 == NB ? 0 : slot + 1;
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------- streaming kernel
//
// Persistent: two CTAs per SM, each owning a contiguous block of rows. One producer
// thread per CTA streams whole rows into a ring of row slots in shared memory with 1-D
// bulk async copies (one cp.async.bulk per row, tracked by an mbarrier per slot), so an
// SM keeps up to ~200 KB of x in flight with almost no registers. Up to 8 consumer
// warps per CTA take one row each: amax over the row in shared memory, then the conversion
// (same arithmetic as above) with coalesced 8-byte stores, then the slot is released.
// Row j lives in slot j % nslot and is consumed by warp j % nwarps, with nwarps dividing
// nslot: every use of a slot is consumed by the same warp, in order, so a warp never
// waits on a later phase of a slot while an earlier phase of the same parity is live.
constexpr int kBulkWarps = 8;
constexpr int kBulkThreads = 32 * (kBulkWarps + 1);  // + the producer warp
constexpr uint32_t kBulkRing = 100 * 1024;  // per CTA; two CTAs per SM
constexpr int kBulkCtasPerSm = 2;
// Inputs below this size stream better through the register kernel (one short wave).
constexpr int64_t kBulkMinBytes = 48ll << 20;
constexpr int kBulkMaxSlots = 64;
constexpr uint64_t kQuantWaitNs = 2000000000ull;  // 2 s: far above any legitimate wait

template <typename T>
__global__ void __launch_bounds__(kBulkThreads, 1)
    quant_rows_bulk_kernel(const T *__restrict__ x, uint8_t *__restrict__ xq,
                           float *__restrict__ scale, int64_t M, int K, int nslot, int nwarps,
                           int trigger) {
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  extern __shared__ __align__(128) uint8_t qsm[];
  const uint32_t row_bytes = static_cast<uint32_t>(K) * 2u;
  const uint32_t sbase = ptx::smem_u32(qsm);
  const uint32_t bar_full = sbase + static_cast<uint32_t>(nslot) * row_bytes;  // 16B aligned
  const uint32_t bar_empty = bar_full + 8u * static_cast<uint32_t>(nslot);
  volatile int *abort = reinterpret_cast<volatile int *>(qsm + (bar_empty - sbase) + 8 * nslot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int64_t per_cta = (M + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * per_cta;
  const int64_t r1 = r0 + per_cta < M ? r0 + per_cta : M;
  const int n = r1 > r0 ? static_cast<int>(r1 - r0) : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nslot; ++i) {
      ptx::mbar_init(bar_full + 8 * i, 1);
      ptx::mbar_init(bar_empty + 8 * i, 1);
    }
    *abort = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  if (warp == kBulkWarps) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % nslot;
        const uint32_t ph = static_cast<uint32_t>(j / nslot) & 1u;
        if (!ptx::mbar_wait_bounded(bar_empty + 8 * s, ph ^ 1u, abort, kQuantWaitNs)) {
          if (!*abort) {
            atomicOr(&g_quant_status, 8u);
            *abort = 1;
          }
          break;
        }
        ptx::mbar_arrive_expect_tx(bar_full + 8 * s, row_bytes);
        ptx::bulk_load_1d(sbase + static_cast<uint32_t>(s) * row_bytes,
                          x + (r0 + j) * static_cast<int64_t>(K), row_bytes, bar_full + 8 * s);
        ++issued;
      }
      // Drain: every issued row has been consumed (or the bounded wait gave up).
      for (int j = issued - 1; j >= 0 && j >= issued - nslot; --j)
        ptx::mbar_wait_timeout(bar_empty + 8 * (j % nslot),
                               static_cast<uint32_t>(j / nslot) & 1u, kQuantWaitNs);
    }
  } else {
    // ---------------------------------------------------------------- consumers
    const int nchunk = K >> 3;  // 16-byte chunks (8 elements) per row
    for (int j = warp; j < n && warp < nwarps; j += nwarps) {
      const int s = j % nslot;
      const uint32_t ph = static_cast<uint32_t>(j / nslot) & 1u;
      if (!ptx::mbar_wait_bounded(bar_full + 8 * s, ph, abort, kQuantWaitNs)) {
        if (lane == 0 && !*abort) {
          atomicOr(&g_quant_status, 8u);
          *abort = 1;
        }
        break;
      }
      const uint4 *row = reinterpret_cast<const uint4 *>(qsm + static_cast<uint32_t>(s) * row_bytes);
      uint32_t mb = 0;
      for (int c = lane; c < nchunk; c += 32) mb = mag_max8(mb, row[c]);
      mb = __reduce_max_sync(0xffffffffu, fold_halves(mb));
      const bool finite = mb <= Bits<T>::kMaxFinite;  // warp-uniform
      float amax;
      if (finite) {
        amax = Bits<T>::to_float(mb);
      } else {
        amax = 0.0f;
        for (int c = lane; c < nchunk; c += 32) amax = amax8_float<T>(amax, row[c]);
        amax = warp_max(amax);
      }
      const float sc = fmaxf(__fdiv_rn(amax, kE4M3Max), kScaleFloor);
      const float inv = __fdiv_rn(1.0f, sc);
      const int64_t grow = r0 + j;
      if (lane == 0) scale[grow] = sc;
      uint2 *qrow = reinterpret_cast<uint2 *>(xq + grow * static_cast<int64_t>(K));
      if (finite) {
        for (int c = lane; c < nchunk; c += 32) qrow[c] = quant8_fast<T>(row[c], inv);
      } else {
        for (int c = lane; c < nchunk; c += 32) qrow[c] = quant8_clamp<T>(row[c], inv);
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);  // slot reusable
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
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
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
cudaError_t launch_rows_bulk(const T *xp, int64_t M, int64_t K, uint8_t *xq, float *scale,
                             cudaStream_t stream, bool trigger, const DeviceInfo &dev) {
  const uint32_t row_bytes = static_cast<uint32_t>(K) * 2u;
  const int64_t max_ctas = static_cast<int64_t>(kBulkCtasPerSm) * dev.sm_count;
  const int64_t grid = M < max_ctas ? M : max_ctas;
  const int64_t per_cta = (M + grid - 1) / grid;
  int64_t nslot = kBulkRing / row_bytes;
  if (nslot > kBulkMaxSlots) nslot = kBulkMaxSlots;
  if (nslot > per_cta) nslot = per_cta;
  // consumer warps: at most kBulkWarps and a divisor of the slot count (slot ownership)
  const int64_t nwarps = nslot < kBulkWarps ? nslot : kBulkWarps;
  nslot -= nslot % nwarps;
  // slots + a full and an empty barrier per slot + the abort word
  const size_t smem = static_cast<size_t>(nslot) * row_bytes + 16 * static_cast<size_t>(nslot) + 16;
  static std::once_flag once[64];
  cudaError_t e = cudaSuccess;
  std::call_once(once[dev.device & 63], [&] {
    e = cudaFuncSetAttribute(quant_rows_bulk_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kBulkRing + 16 * kBulkMaxSlots + 16));
  });
  if (e != cudaSuccess) return e;
  quant_rows_bulk_kernel<T><<<static_cast<unsigned>(grid), kBulkThreads, smem, stream>>>(
      xp, xq, scale, M, static_cast<int>(K), static_cast<int>(nslot), static_cast<int>(nwarps),
      trigger ? 1 : 0);
  return cudaGetLastError();
}

// Launch as a programmatic dependent of the previous kernel on the stream: the grid may
// be scheduled while that kernel finishes, and waits for it (griddepcontrol.wait, trigger
// bit 1) before touching memory, so only the launch latency overlaps.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*k)(KArgs...), unsigned grid, unsigned block, size_t smem,
                             cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// CTAs of `Kernel` one SM holds at a block size and dynamic shared memory, per device
// (one cache per kernel instantiation; the first query also sets the kernel's dynamic
// shared memory limit).
template <auto Kernel>
int blocks_per_sm(int device, int threads, size_t smem, cudaError_t *err) {
  static std::mutex mu;
  static int cache[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  int &c = cache[device & 63];
  if (c == 0) {
    *err = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
    if (*err == cudaSuccess)
      *err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c, Kernel, threads, smem);
    if (*err == cudaSuccess && c < 1) *err = cudaErrorInvalidConfiguration;
    if (*err != cudaSuccess) c = 0;
  }
  return c;
}

constexpr int kPipeBlock = 256;                   // threads per CTA of the pipelined kernels
constexpr int64_t kPipeRegMinBytes = 256ll << 20;  // register form from this input size up

// Pipelined per-token quantizer for K % 8 == 0, K <= 16384 (16-byte aligned rows): a
// persistent grid of every CTA the SMs hold (capped at one group per row). Inputs below
// kPipeRegMinBytes stream through cp.async slots (two rows in flight per group), larger
// ones through the two register buffers; both measured on B200 as the faster form at
// their sizes.
template <typename T, int VPL, int WPR>
cudaError_t launch_rows_pipe(const T *xp, int64_t M, int64_t K, uint8_t *xq, float *scale,
                             cudaStream_t stream, int trig, const DeviceInfo &dev,
                             const L2Prefetch &pf) {
  cudaError_t e = cudaSuccess;
  const int gpc = kPipeBlock / 32 / WPR;
  const int64_t need = (M + gpc - 1) / gpc;
  if (M * K * 2 >= kPipeRegMinBytes) {
    auto k = quant_rows_pipe_kernel<T, VPL, WPR>;
    const int occ = blocks_per_sm<quant_rows_pipe_kernel<T, VPL, WPR>>(dev.device, kPipeBlock, 0, &e);
    if (e != cudaSuccess) return e;
    const int64_t grid = std::min<int64_t>(need, static_cast<int64_t>(occ) * dev.sm_count);
    return launch_dependent(k, static_cast<unsigned>(grid), kPipeBlock, 0, stream, xp, xq, scale,
                            M, static_cast<int>(K), trig);
  }
  auto k = quant_rows_pipe_async_kernel<T, VPL, WPR, 2>;
  const size_t smem = static_cast<size_t>(2) * VPL * kPipeBlock * 16;
  const int occ =
      blocks_per_sm<quant_rows_pipe_async_kernel<T, VPL, WPR, 2>>(dev.device, kPipeBlock, smem, &e);
  if (e != cudaSuccess) return e;
  const int64_t resident = static_cast<int64_t>(occ) * dev.sm_count;
  int64_t grid = std::min<int64_t>(need, resident);
  // with a prefetch, enough CTAs (rowless ones only prefetch) for ~64 KB slices
  if (pf.bytes > 0) grid = std::max(grid, std::min<int64_t>(resident, (pf.bytes + 65535) / 65536));
  return launch_dependent(k, static_cast<unsigned>(grid), kPipeBlock, smem, stream, xp, xq, scale,
                          M, static_cast<int>(K), trig,
                          static_cast<const uint8_t *>(pf.bytes > 0 ? pf.ptr : nullptr),
                          pf.bytes > 0 ? pf.bytes : int64_t{0});
}

// Rows of nvec 16-byte vectors: twice the fewest warps per row that keep a thread at
// <= 8 vectors (at most 8 warps), then the vectors per thread that covers the row.
template <typename T>
bool launch_rows_pipe_any(const T *xp, int64_t M, int64_t K, uint8_t *xq, float *scale,
                          cudaStream_t stream, int trig, const DeviceInfo &dev, cudaError_t *e,
                          const L2Prefetch &pf) {
  const int64_t nvec = K / 8;
  int wpr = 1;
  while ((nvec + 32 * wpr - 1) / (32 * wpr) > 8 && wpr < 8) wpr *= 2;
  wpr = wpr * 2 > 8 ? 8 : wpr * 2;
  const int64_t per = (nvec + 32 * wpr - 1) / (32 * wpr);
  if (per > 8) return false;
  const int vpl = per <= 2 ? 2 : per <= 4 ? 4 : per <= 6 ? 6 : 8;
#define FP8LIN_PIPE_CASE(V, W)                                                     \
  if (vpl == V && wpr == W) {                                                       \
    *e = launch_rows_pipe<T, V, W>(xp, M, K, xq, scale, stream, trig, dev, pf);     \
    return true;                                                                    \
  }
  FP8LIN_PIPE_CASE(2, 2) FP8LIN_PIPE_CASE(4, 2) FP8LIN_PIPE_CASE(2, 4) FP8LIN_PIPE_CASE(4, 4)
  FP8LIN_PIPE_CASE(2, 8) FP8LIN_PIPE_CASE(4, 8) FP8LIN_PIPE_CASE(6, 8) FP8LIN_PIPE_CASE(8, 8)
#undef FP8LIN_PIPE_CASE
  return false;
}

template <typename T>
cudaError_t launch_rows_typed(const void *x, int64_t M, int64_t K, uint8_t *xq, float *scale,
                              cudaStream_t stream, bool trigger, const L2Prefetch &pf) {
  const T *xp = reinterpret_cast<const T *>(x);
  const int64_t nvec = K / 8;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(xq) % 8 == 0);
  DeviceInfo dev;
  // 16-byte rows up to K = 16384: the pipelined kernels, launched as programmatic
  // dependents; streaming kernel for larger inputs of wider rows that fit the ring
  // twice; the register kernel below for the rest.
  if (K % 8 == 0 && aligned && current_device_info(&dev)) {
    cudaError_t e = cudaSuccess;
    if (launch_rows_pipe_any<T>(xp, M, K, xq, scale, stream, (trigger ? 1 : 0) | 2, dev, &e, pf))
      return e;
    if (2 * K * 2 <= static_cast<int64_t>(kBulkRing) && M * K * 2 >= kBulkMinBytes)
      return launch_rows_bulk<T>(xp, M, K, xq, scale, stream, trigger, dev);
  }
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

// ---------------------------------------------------------------- MXFP8 block quantizer
//
// Replaces quant_mxfp8_kernel (csrc/quantize.cu:92-131 of the reference): per 32-element
// block of a row, a power-of-two (e8m0) scale and e4m3 codes, the scales written in
// the tiled block-scale layout the block-scaled tensor-core GEMM reads (512-byte tiles
// of 128 rows x 4 scale columns; scale (r, c) at tile (r / 128, c / 4), byte
// (r % 32) * 16 + ((r % 128) / 32) * 4 + c % 4; tiles ordered K-major).
//   amax  = max |x| over the block, NaN ignored (an all-NaN block counts as 0)
//   e8    = 127 for amax 0; 254 for an infinite amax; otherwise
//           clamp(exponent(amax) + 119, 0, 254) with exponent(amax) = floor(log2(amax)),
//           read exactly from the magnitude's bits (the reference's floorf(log2f(amax))
//           agrees with it for every bf16 and fp16 amax)
//   q     = e4m3_satfinite(fminf(fmaxf(x * 2^(127 - e8), -448), 448))
// One warp owns a 1024-element segment of a row: lane l holds elements (32 i + l) * 8 ..
// +7 of vector i (i = 0..3), so each block is 4 consecutive lanes (amax by two
// shuffles) and each 4-block group of scales (4 consecutive bytes of the layout) is one
// 32-bit store by lane 0 or 16. Warps past row M, and blocks past K/32 inside the last
// 4-block group of a row, write the padding value 127 (e8m0 1.0), so the whole padded
// grid is written and needs no prefill.
template <typename T>
struct MxBits;
template <>
struct MxBits<__nv_bfloat16> {
  static constexpr uint32_t kInf = 0x7F80u;
  // floor(log2(value)) of a nonzero finite magnitude bit pattern
  __device__ __forceinline__ static int exponent(uint32_t mag) {
    const uint32_t f = mag >> 7;
    return f ? static_cast<int>(f) - 127 : (31 - __clz(static_cast<int>(mag & 0x7Fu))) - 133;
  }
};
template <>
struct MxBits<__half> {
  static constexpr uint32_t kInf = 0x7C00u;
  __device__ __forceinline__ static int exponent(uint32_t mag) {
    const uint32_t f = mag >> 10;
    return f ? static_cast<int>(f) - 15 : (31 - __clz(static_cast<int>(mag & 0x3FFu))) - 24;
  }
};

template <typename T>
__device__ __forceinline__ uint32_t mx_mag_max8(const uint4 &v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t mx = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = w[i] & 0x7FFFu, hi = (w[i] >> 16) & 0x7FFFu;
    mx = max(mx, lo > MxBits<T>::kInf ? 0u : lo);  // NaN patterns count as 0
    mx = max(mx, hi > MxBits<T>::kInf ? 0u : hi);
  }
  return mx;
}

template <typename T>
__device__ __forceinline__ uint32_t mx_block_e8(uint32_t mag) {
  if (mag == 0) return 127u;
  if (mag == MxBits<T>::kInf) return 254u;
  const int e8 = MxBits<T>::exponent(mag) + 119;
  return static_cast<uint32_t>(e8 < 0 ? 0 : (e8 > 254 ? 254 : e8));
}

// 2^(127 - e8) for e8 in 0..254, exactly (2^-127 is a subnormal float)
__device__ __forceinline__ float mx_inv(uint32_t e8) {
  const int e = 127 - static_cast<int>(e8);
  return e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23)
                   : __uint_as_float(0x00400000u);
}

constexpr int kMxWarps = 8;
constexpr int kMxVecs = 4;                       // 16-byte vectors per lane
constexpr int kMxSeg = 32 * kMxVecs * 8;         // elements per warp segment (1024)

template <typename T>
__global__ void __launch_bounds__(32 * kMxWarps) quant_mx_kernel(
    const T *__restrict__ x, uint8_t *__restrict__ xq, uint8_t *__restrict__ sf, int64_t M,
    int K, int64_t rows_pad, int segs, int ncb, int trigger) {
  // trigger bits as the per-token kernels': 1 = release the dependents, 2 = wait first
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * kMxWarps + (threadIdx.x >> 5);
  const int64_t row = wid / segs;
  if (row >= rows_pad) return;  // warp-uniform
  const int seg = static_cast<int>(wid - row * segs);
  const int nblk = K >> 5;
  const bool row_live = row < M;
  const int e0 = seg * kMxSeg;
  const T *xr = x + (row_live ? row : 0) * static_cast<int64_t>(K);
  uint4 v[kMxVecs];
#pragma unroll
  for (int i = 0; i < kMxVecs; ++i) {
    const int el = e0 + (i * 32 + lane) * 8;
    v[i] = (row_live && el < K) ? ld_stream_v4(xr + el) : make_uint4(0u, 0u, 0u, 0u);
  }
  const int64_t sf_row = (row >> 7) * static_cast<int64_t>(ncb) * 512 + (row & 31) * 16 +
                         ((row & 127) >> 5) * 4;
  // Magnitude maxima of this lane's 8-element groups with packed integer maxima (exact
  // for finite and infinite values, which order like their bits); a maximum above the
  // infinity pattern means the group holds a NaN. Segments without NaN (the normal
  // case, warp-uniform) keep these maxima and convert with a multiply and the saturating
  // convert: x * 2^(127 - e8) is below 512 for every finite x of a block, and an inf
  // saturates to 448 exactly as the reference's clamp makes it. A segment with a NaN
  // recomputes the maxima ignoring NaN and takes the literal clamp (NaN -> -448).
  uint32_t m8[kMxVecs];
  bool nan = false;
#pragma unroll
  for (int i = 0; i < kMxVecs; ++i) {
    m8[i] = fold_halves(mag_max8(0u, v[i]));
    nan |= m8[i] > MxBits<T>::kInf;
  }
  const bool any_nan = __any_sync(0xffffffffu, nan);
  if (any_nan) {
#pragma unroll
    for (int i = 0; i < kMxVecs; ++i) m8[i] = mx_mag_max8<T>(v[i]);
  }
  float inv[kMxVecs];
#pragma unroll
  for (int i = 0; i < kMxVecs; ++i) {
    const int el = e0 + (i * 32 + lane) * 8;
    const int g = el >> 5;  // this lane's block
    const bool live = row_live && g < nblk;
    uint32_t mag = live ? m8[i] : 0u;
    mag = max(mag, __shfl_xor_sync(0xffffffffu, mag, 1));
    mag = max(mag, __shfl_xor_sync(0xffffffffu, mag, 2));
    const uint32_t e8 = live ? mx_block_e8<T>(mag) : 127u;
    inv[i] = mx_inv(e8);
    // the scales of blocks g .. g+3 from lanes l, l+4, l+8, l+12 (l = 0, 16)
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, e8, 4);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, e8, 8);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, e8, 12);
    const int grp = g >> 2;
    if ((lane & 15) == 0 && grp < ncb)
      *reinterpret_cast<uint32_t *>(sf + sf_row + static_cast<int64_t>(grp) * 512) =
          e8 | (b1 << 8) | (b2 << 16) | (b3 << 24);
  }
  uint8_t *qr = xq + row * static_cast<int64_t>(K);
  // two loops behind the warp-uniform branch, so each value is converted once
  if (!any_nan) {
#pragma unroll
    for (int i = 0; i < kMxVecs; ++i) {
      const int el = e0 + (i * 32 + lane) * 8;
      if (row_live && el < K) *reinterpret_cast<uint2 *>(qr + el) = quant8_fast<T>(v[i], inv[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < kMxVecs; ++i) {
      const int el = e0 + (i * 32 + lane) * 8;
      if (row_live && el < K) *reinterpret_cast<uint2 *>(qr + el) = quant8_clamp<T>(v[i], inv[i]);
    }
  }
}

// ---------------------------------------------------------------- NVFP4 block quantizer
//
// Replaces quant_nvfp4_kernel (csrc/quantize.cu:157-194 of the reference): per 16-element
// block, an e4m3 scale and e2m1 codes packed two per byte (element 2j in the low nibble),
// the scales in the same tiled layout (K/16 scale columns).
//   amax  = fmaxf-reduce |x| over the block (NaN ignored unless all NaN)
//   s     = fminf(amax * fl(1/6), 448); s8 = e4m3_satfinite(s); sdec = value of s8
//   x_inv = sdec > 0 ? 1 / sdec : 0   (IEEE divide)
//   code  = e2m1(fminf(fmaxf(x * x_inv, -6), 6)): sign bit 8 when negative, magnitude by
//           the thresholds 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5 (ties go up)
// Lane l holds 8 consecutive elements of vector i (16 bytes): a block is 2 lanes, a
// 4-block group of scales (one 32-bit word of the layout) is 8 lanes. Padding scales are
// 0x38 (e4m3 1.0), written by the kernel.
// The magnitude code of |v| <= 6 by the thresholds above. Each threshold has at most two
// mantissa bits, so a >= t exactly when (exponent, top two mantissa bits) of a are >= those of
// t: the code is a function of bits 21-30 of a. From 0.25 (exponent 125) upwards those index
// a table of 19 3-bit codes; below 0.25 the code is 0. (Checked against the threshold form
// for every float in [0, 6].)
constexpr uint64_t kE2m1Lut = 0x01fed6c8da489249ull;  // codes 1,1,1,1,1,1,2,2,2,3,3,4,4,5,5,6,6,7,7
__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const uint32_t sgn = v < 0.0f ? 8u : 0u;
  const int idx = static_cast<int>((__float_as_uint(v) & 0x7FFFFFFFu) >> 21) - (125 << 2);
  const uint32_t c = idx < 0 ? 0u : static_cast<uint32_t>(kE2m1Lut >> (3 * idx)) & 7u;
  return sgn | c;
}

// value of a non-negative e4m3 code (exact)
__device__ __forceinline__ float e4m3_pos_value(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  return e ? __uint_as_float(((e + 120u) << 23) | (m << 20))
           : __fmul_rn(static_cast<float>(m), 0.001953125f);  // m * 2^-9
}

template <typename T>
__global__ void __launch_bounds__(32 * kMxWarps) quant_nv_kernel(
    const T *__restrict__ x, uint8_t *__restrict__ xq, uint8_t *__restrict__ sf, int64_t M,
    int K, int64_t rows_pad, int segs, int ncb, int trigger) {
  // trigger bits as the per-token kernels': 1 = release the dependents, 2 = wait first
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * kMxWarps + (threadIdx.x >> 5);
  const int64_t row = wid / segs;
  if (row >= rows_pad) return;  // warp-uniform
  const int seg = static_cast<int>(wid - row * segs);
  const int nblk = K >> 4;
  const bool row_live = row < M;
  const int e0 = seg * kMxSeg;
  const T *xr = x + (row_live ? row : 0) * static_cast<int64_t>(K);
  uint4 v[kMxVecs];
#pragma unroll
  for (int i = 0; i < kMxVecs; ++i) {
    const int el = e0 + (i * 32 + lane) * 8;
    v[i] = (row_live && el < K) ? ld_stream_v4(xr + el) : make_uint4(0u, 0u, 0u, 0u);
  }
  const int64_t sf_row = (row >> 7) * static_cast<int64_t>(ncb) * 512 + (row & 31) * 16 +
                         ((row & 127) >> 5) * 4;
  const float inv6 = 1.0f / 6.0f;
#pragma unroll
  for (int i = 0; i < kMxVecs; ++i) {
    const int el = e0 + (i * 32 + lane) * 8;
    const int g = el >> 4;  // this lane's 16-element block
    const bool live = row_live && g < nblk;
    float f[8];
    In<T>::unpack8(v[i], f);
    float amax = fabsf(f[0]);
#pragma unroll
    for (int e = 1; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float sc = fminf(__fmul_rn(amax, inv6), kE4M3Max);
    const uint32_t s8 = live ? static_cast<uint32_t>(ptx::cvt_e4m3x2(sc, 0.0f) & 0xFFu) : 0x38u;
    // the scales of blocks g .. g+3 from lanes l, l+2, l+4, l+6 (l = 0, 8, 16, 24)
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, s8, 2);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, s8, 4);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, s8, 6);
    const int grp = g >> 2;
    if ((lane & 7) == 0 && grp < ncb)
      *reinterpret_cast<uint32_t *>(sf + sf_row + static_cast<int64_t>(grp) * 512) =
          s8 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    if (live) {
      const float sdec = e4m3_pos_value(s8);
      const float x_inv = sdec > 0.0f ? __fdiv_rn(1.0f, sdec) : 0.0f;
      uint32_t packed = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float q = fminf(fmaxf(__fmul_rn(f[e], x_inv), -6.0f), 6.0f);
        packed |= e2m1_code(q) << (4 * e);
      }
      *reinterpret_cast<uint32_t *>(xq + (row * static_cast<int64_t>(K) + el) / 2) = packed;
    }
  }
}

template <typename T>
cudaError_t launch_nv_typed(const void *x, int64_t M, int64_t K, uint8_t *xq, uint8_t *sf,
                            cudaStream_t stream, bool trigger) {
  const int64_t rows_pad = (M + 127) / 128 * 128;
  const int segs = static_cast<int>((K + kMxSeg - 1) / kMxSeg);
  const int ncb = static_cast<int>((K / 16 + 3) / 4);
  const int64_t warps = rows_pad * segs;
  const int64_t blocks = (warps + kMxWarps - 1) / kMxWarps;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  // a programmatic dependent of the kernel before it, as the per-token quantizer
  return launch_dependent(quant_nv_kernel<T>, static_cast<unsigned>(blocks), 32 * kMxWarps, 0, stream,
                          reinterpret_cast<const T *>(x), xq, sf, M, static_cast<int>(K),
                          rows_pad, segs, ncb, (trigger ? 1 : 0) | 2);
}

template <typename T>
cudaError_t launch_mx_typed(const void *x, int64_t M, int64_t K, uint8_t *xq, uint8_t *sf,
                            cudaStream_t stream, bool trigger) {
  const int64_t rows_pad = (M + 127) / 128 * 128;
  const int segs = static_cast<int>((K + kMxSeg - 1) / kMxSeg);
  const int ncb = static_cast<int>((K / 32 + 3) / 4);
  const int64_t warps = rows_pad * segs;
  const int64_t blocks = (warps + kMxWarps - 1) / kMxWarps;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  // a programmatic dependent of the kernel before it, as the per-token quantizer
  return launch_dependent(quant_mx_kernel<T>, static_cast<unsigned>(blocks), 32 * kMxWarps, 0, stream,
                          reinterpret_cast<const T *>(x), xq, sf, M, static_cast<int>(K),
                          rows_pad, segs, ncb, (trigger ? 1 : 0) | 2);
}

// ---------------------------------------------------------------- LayerNorm + modulation
//
// The quantizer fused into the op that precedes the linear in a FLUX / DiT block
// (AdaLayerNormZero: y = LayerNorm(x) * (1 + scale[b]) + shift[b], LayerNorm without
// affine parameters), so that the modulated activations never go to HBM in bf16: the
// kernel reads x and writes the e4m3 codes and per-token scales the GEMM consumes.
// y is rounded to x's type after each step exactly as the unfused bf16 torch ops round it
//   ln = T((x - mean) * rstd); m1 = T(1 + scale); t = T(ln * m1); y = T(t + shift)
// and is then quantized with the reference's per-token rule (quant8_clamp, the literal
// clamp arithmetic of csrc/quantize.cu:52-72). mean and the variance are fp32 sums in a
// fixed order -- lane l adds the elements of its 8-element chunks l, l + 32, ... in
// sequence, then a butterfly over xor offsets 16, 8, 4, 2, 1 -- and
// rstd = 1 / sqrt(var + eps) with IEEE square root and divides, so the result is
// reproducible exactly on the CPU.
// One warp per row holding the row in registers (K <= 8192, K % 8 == 0); 8 rows per CTA.
constexpr int kLnThreads = 256;

// Pairs of values: IEEE fp32 add / multiply of two lanes at once, and rounding of a pair to
// T (round-to-nearest-even, one convert) with the rounded values read back exactly.
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 r;
  asm("{.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "add.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 mul2v(float2 a, float2 b) {
  float2 r;
  asm("{.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// add / mul of two packed pairs of T with one rounding (IEEE, subnormals kept). For two
// values of T they equal the fp32 operation followed by the rounding to T that a torch
// elementwise op applies: a product of two 8- (11-) bit significands is exact in fp32, and
// a sum is inexact in fp32 only when one operand is below 2^-16 (2^-13) of the other,
// where the sum is too far from a midpoint of T's grid for the second rounding to differ.
template <typename T>
struct Rnd;
template <>
struct Rnd<__nv_bfloat16> {
  static constexpr uint32_t kOne2 = 0x3F803F80u;  // (1, 1)
  __device__ __forceinline__ static uint32_t pack(float2 v) { return ptx::pack_bf16x2(v.x, v.y); }
  __device__ __forceinline__ static float2 unpack(uint32_t b) {
    return make_float2(__uint_as_float(b << 16), __uint_as_float(b & 0xFFFF0000u));
  }
  __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
};
template <>
struct Rnd<__half> {
  static constexpr uint32_t kOne2 = 0x3C003C00u;
  __device__ __forceinline__ static uint32_t pack(float2 v) { return ptx::pack_f16x2(v.x, v.y); }
  __device__ __forceinline__ static float2 unpack(uint32_t b) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&b));
  }
  __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
};

__device__ __forceinline__ float warp_sum_xor(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <typename T, int CPL>
__global__ void __launch_bounds__(kLnThreads) ln_mod_quant_kernel(
    const T *__restrict__ x, const T *__restrict__ shift, const T *__restrict__ scale, int64_t M,
    int K, int64_t rows_per_batch, float eps, uint8_t *__restrict__ xq, float *__restrict__ xs,
    int trigger) {
  // trigger bits as the per-token kernels': 1 = release the dependents, 2 = wait first
  if (trigger & 2) ptx::grid_dependency_wait();
  if (trigger & 1) ptx::grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kLnThreads / 32) + (threadIdx.x >> 5);
  if (row >= M) return;  // warp-uniform
  const int nch = K >> 3;
  const T *xr = x + row * static_cast<int64_t>(K);
  uint4 v[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < nch ? ld_stream_v4(xr + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
  }
  const float kf = static_cast<float>(K);
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    if (lane + 32 * i < nch) {
      float f[8];
      In<T>::unpack8(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum = __fadd_rn(sum, f[e]);
    }
  }
  const float mean = __fdiv_rn(warp_sum_xor(sum), kf);
  // (x - mean)^2 two elements at a time (x - mean is x + (-mean): the same IEEE result),
  // accumulated in element order
  const float2 nmean = make_float2(-mean, -mean);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    if (lane + 32 * i < nch) {
      const uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 d = add2(Rnd<T>::unpack(xw[p]), nmean);
        const float2 dd = mul2v(d, d);
        sq = __fadd_rn(sq, dd.x);
        sq = __fadd_rn(sq, dd.y);
      }
    }
  }
  const float var = __fdiv_rn(warp_sum_xor(sq), kf);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const int64_t boff = (row / rows_per_batch) * static_cast<int64_t>(K);
  // y, two elements at a time: ln in fp32 and rounded, then m1, t and y as packed T ops
  const float2 rs2 = make_float2(rstd, rstd);
  uint32_t mag = 0;  // packed max of |y| bit patterns (the amax of finite rows)
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) {
      const uint4 sv = __ldg(reinterpret_cast<const uint4 *>(scale + boff + 8 * c));
      const uint4 hv = __ldg(reinterpret_cast<const uint4 *>(shift + boff + 8 * c));
      const uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
      const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
      uint32_t w[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t ln = Rnd<T>::pack(mul2v(add2(Rnd<T>::unpack(xw[p]), nmean), rs2));
        const uint32_t m1 = Rnd<T>::add(Rnd<T>::kOne2, sw[p]);
        w[p] = Rnd<T>::add(Rnd<T>::mul(ln, m1), hw[p]);
        mag = mag_max2(mag, w[p]);
      }
      v[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  // quantize_fp8's rule on y: the packed-integer amax and the fast conversion when the row
  // is finite, the float amax (NaN ignored) and the literal clamp otherwise
  const uint32_t mmax = fold_halves(mag);
  const bool finite = __all_sync(0xffffffffu, mmax <= Bits<T>::kMaxFinite);
  float amax;
  if (finite) {
    amax = warp_max(Bits<T>::to_float(mmax));
  } else {
    amax = 0.0f;
#pragma unroll
    for (int i = 0; i < CPL; ++i)
      if (lane + 32 * i < nch) amax = amax8_float<T>(amax, v[i]);
    amax = warp_max(amax);
  }
  const float sc = fmaxf(__fdiv_rn(amax, kE4M3Max), kScaleFloor);
  const float inv = __fdiv_rn(1.0f, sc);
  if (lane == 0) xs[row] = sc;
  uint8_t *qr = xq + row * static_cast<int64_t>(K);
  if (finite) {  // warp-uniform: one conversion per value, not both and a select
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) *reinterpret_cast<uint2 *>(qr + 8 * c) = quant8_fast<T>(v[i], inv);
    }
  } else {
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) *reinterpret_cast<uint2 *>(qr + 8 * c) = quant8_clamp<T>(v[i], inv);
    }
  }
}

template <typename T, int CPL>
cudaError_t launch_ln_cpl(const void *x, const void *shift, const void *scale, int64_t M, int K,
                          int64_t rows_per_batch, float eps, uint8_t *xq, float *xs,
                          cudaStream_t stream, bool trigger) {
  const int64_t blocks = (M + kLnThreads / 32 - 1) / (kLnThreads / 32);
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  // a programmatic dependent of the kernel before it, as the per-token quantizer
  return launch_dependent(ln_mod_quant_kernel<T, CPL>, static_cast<unsigned>(blocks), kLnThreads,
                          0, stream, reinterpret_cast<const T *>(x),
                          reinterpret_cast<const T *>(shift), reinterpret_cast<const T *>(scale),
                          M, K, rows_per_batch, eps, xq, xs, (trigger ? 1 : 0) | 2);
}

template <typename T>
cudaError_t launch_ln_typed(const void *x, const void *shift, const void *scale, int64_t M,
                            int K, int64_t rows_per_batch, float eps, uint8_t *xq, float *xs,
                            cudaStream_t stream, bool trigger) {
  const int per_lane = (K / 8 + 31) / 32;  // 16-byte chunks per lane
  if (per_lane <= 4)
    return launch_ln_cpl<T, 4>(x, shift, scale, M, K, rows_per_batch, eps, xq, xs, stream, trigger);
  if (per_lane <= 8)
    return launch_ln_cpl<T, 8>(x, shift, scale, M, K, rows_per_batch, eps, xq, xs, stream, trigger);
  if (per_lane <= 12)
    return launch_ln_cpl<T, 12>(x, shift, scale, M, K, rows_per_batch, eps, xq, xs, stream, trigger);
  if (per_lane <= 16)
    return launch_ln_cpl<T, 16>(x, shift, scale, M, K, rows_per_batch, eps, xq, xs, stream, trigger);
  if (per_lane <= 24)
    return launch_ln_cpl<T, 24>(x, shift, scale, M, K, rows_per_batch, eps, xq, xs, stream, trigger);
  return launch_ln_cpl<T, 32>(x, shift, scale, M, K, rows_per_batch, eps, xq, xs, stream, trigger);
}

}  // namespace

cudaError_t launch_quantize_rows(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                                 float *scale, cudaStream_t stream, bool trigger_dependents,
                                 const L2Prefetch &prefetch) {
  if (M == 0) return cudaSuccess;
  if (dtype == kBF16)
    return launch_rows_typed<__nv_bfloat16>(x, M, K, xq, scale, stream, trigger_dependents,
                                            prefetch);
  return launch_rows_typed<__half>(x, M, K, xq, scale, stream, trigger_dependents, prefetch);
}

cudaError_t launch_quantize_mx(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                               uint8_t *scales, cudaStream_t stream, bool trigger_dependents) {
  if (M == 0) return cudaSuccess;
  if (dtype == kBF16)
    return launch_mx_typed<__nv_bfloat16>(x, M, K, xq, scales, stream, trigger_dependents);
  return launch_mx_typed<__half>(x, M, K, xq, scales, stream, trigger_dependents);
}

cudaError_t launch_quantize_nv(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                               uint8_t *scales, cudaStream_t stream, bool trigger_dependents) {
  if (M == 0) return cudaSuccess;
  if (dtype == kBF16)
    return launch_nv_typed<__nv_bfloat16>(x, M, K, xq, scales, stream, trigger_dependents);
  return launch_nv_typed<__half>(x, M, K, xq, scales, stream, trigger_dependents);
}

cudaError_t launch_ln_modulate_quantize(const void *x, int dtype, int64_t M, int64_t K,
                                        int64_t batches, const void *shift, const void *scale,
                                        float eps, uint8_t *xq, float *x_scale,
                                        cudaStream_t stream, bool trigger_dependents) {
  if (M == 0) return cudaSuccess;
  if (K <= 0 || K > kLnMaxK || K % 8 != 0 || batches <= 0 || M % batches != 0)
    return cudaErrorInvalidValue;
  const int64_t rpb = M / batches;
  if (dtype == kBF16)
    return launch_ln_typed<__nv_bfloat16>(x, shift, scale, M, static_cast<int>(K), rpb, eps, xq,
                                          x_scale, stream, trigger_dependents);
  return launch_ln_typed<__half>(x, shift, scale, M, static_cast<int>(K), rpb, eps, xq, x_scale,
                                 stream, trigger_dependents);
}

cudaError_t read_quant_status(unsigned int *bits, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(bits, g_quant_status, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_quant_status, &zero, sizeof(unsigned int));
  }
  return e;
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
