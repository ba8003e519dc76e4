// gemm_sm100.cu -- persistent, warp-specialised tcgen05 e4m3 GEMM for sm_100a with the
// per-token x per-channel dequant and the bias fused into its epilogue.
//
// Replaces the reference's cuBLASLt matmul into an fp32 [M,N] buffer
// (csrc/fp8_gemm.cu:109-131, 180-184) plus its separate dequant_bias_kernel pass
// (csrc/fp8_gemm.cu:65-80): here the fp32 accumulator never leaves the SM.
//
//   out[m,n] = fma(acc[m,n] * x_scale[m], w_scale[n], bias[n])    -> bf16 (or fp16)
//   acc[m,n] = sum_k e4m3(xq[m,k]) * e4m3(wq[n,k])                 (fp32, tensor cores)
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles of BM x BN = 128 x 256:
//   warp 0     TMA producer: A (xq) and B (wq) K-blocks of 128 bytes into a STAGES-deep
//              shared-memory ring (128-byte swizzle), one mbarrier pair per stage.
//   warp 1     MMA issuer: one thread issues tcgen05.mma.kind::f8f6f4 (M=128, N=256,
//              K=32) into one of two TMEM accumulators (2 x 256 fp32 columns), and
//              tcgen05.commit frees smem stages / publishes finished accumulators.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time from the warp's TMEM lane
//              quarter, apply scales + bias, pack to bf16, stage in swizzled smem and
//              TMA-store 32x32 boxes. Double-buffered TMEM lets the epilogue of tile i
//              overlap the main loop of tile i+1.
// Every mbarrier wait is bounded (see kWaitLimitNs); a wait that runs out records a bit
// in g_gemm_status, tells the other roles to stop, drains its in-flight copies and the
// CTA frees its TMEM and returns.
// No TMA multicast is used anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>

#include "internal.h"
#include "ptx.cuh"

namespace fp8lin {

__device__ unsigned int g_gemm_status;  // watchdog bits (1 producer, 2 mma, 4 epilogue)

namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes == e4m3 elements per K-block (one 128B swizzle row)
constexpr int UMMA_K = 32;
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int EPI_COLS = 32;
constexpr int TMEM_COLS = 2 * BN;
constexpr uint32_t A_STAGE = BM * BK;  // 16 KB
constexpr uint32_t B_STAGE = BN * BK;  // 32 KB
constexpr uint32_t EPI_BUF = 32 * EPI_COLS * 2;  // 2 KB: 32 rows x 32 cols x 2 B

constexpr uint32_t PAR_BYTES = 2 * BN * 4;        // per epilogue warp: w_scale + bias of a tile

constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_B = OFF_A + STAGES * A_STAGE;
constexpr uint32_t OFF_EPI = OFF_B + STAGES * B_STAGE;
constexpr uint32_t OFF_PAR = OFF_EPI + EPI_WARPS * 2 * EPI_BUF;
constexpr uint32_t OFF_BAR = OFF_PAR + EPI_WARPS * PAR_BYTES;
constexpr uint32_t NUM_BARS = 2 * STAGES + 5;  // full, empty, tmem full x2, tmem empty x2, drain
constexpr uint32_t OFF_TMEM_SLOT = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t OFF_ABORT = OFF_TMEM_SLOT + 4;
constexpr uint32_t SMEM_USED = OFF_ABORT + 4;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;  // slack to align the base to 1024 B

static_assert(SMEM_BYTES <= 232448, "shared memory budget");
static_assert(OFF_B % 1024 == 0 && OFF_EPI % 1024 == 0, "swizzle atoms need 1024 B alignment");

constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s: far above any legitimate wait
constexpr uint64_t kDrainLimitNs = 1000000000ull;  // 1 s for in-flight copies on exit

constexpr uint32_t IDESC = ptx::idesc_e4m3_f32(BM, BN);

struct Params {
  const float *xs;
  const float *ws;
  const void *bias;
  int bias_dtype;
  int out_dtype;
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int pdl;
};

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int &mt, int &nt) {
  // M-fastest order: the CTAs running at the same time share one or two B tiles and
  // stream the A tiles from L2.
  mt = t % m_tiles;
  nt = t / m_tiles;
}

__device__ __forceinline__ void record_timeout(unsigned bit, volatile int *abort) {
  atomicOr(&g_gemm_status, bit);
  *abort = 1;
}

__device__ __forceinline__ float load_bias(const void *bias, int dtype, int n) {
  switch (dtype) {
    case kBF16: {
      const uint16_t b = __ldg(reinterpret_cast<const unsigned short *>(bias) + n);
      return __uint_as_float(static_cast<uint32_t>(b) << 16);
    }
    case kF16: return __half2float(__ldg(reinterpret_cast<const __half *>(bias) + n));
    case kF32: return __ldg(reinterpret_cast<const float *>(bias) + n);
    default: return 0.0f;
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_out, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar_full = sbase + OFF_BAR;             // STAGES barriers
  const uint32_t bar_empty = bar_full + STAGES * 8;      // STAGES barriers
  const uint32_t bar_tfull = bar_empty + STAGES * 8;     // 2 barriers
  const uint32_t bar_tempty = bar_tfull + 2 * 8;         // 2 barriers
  const uint32_t bar_drain = bar_tempty + 2 * 8;         // MMA drain on the way out
  volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + OFF_TMEM_SLOT);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + OFF_ABORT);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_out);
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(bar_tfull + 8 * a, 1);
      ptx::mbar_init(bar_tempty + 8 * a, EPI_WARPS);
    }
    ptx::mbar_init(bar_drain, 1);
    *abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(sbase + OFF_TMEM_SLOT, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Everything above overlaps the previous kernel when launched as a PDL dependent;
  // nothing produced by it is read before this point.
  if (p.pdl) ptx::grid_dependency_wait();

  const int num_tiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, p.m_tiles, mt, nt);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ptx::mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1u, abort, kWaitLimitNs)) {
            if (!*abort) record_timeout(1u, abort);
            ok = false;
            break;
          }
          const uint32_t fb = bar_full + 8 * stage;
          ptx::mbar_arrive_expect_tx(fb, A_STAGE + B_STAGE);
          ptx::tma_load_2d(sbase + OFF_A + stage * A_STAGE, &tmap_a, kb * BK, mt * BM, fb);
          ptx::tma_load_2d(sbase + OFF_B + stage * B_STAGE, &tmap_b, kb * BK, nt * BN, fb);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: the last min(issued, STAGES) loads are the final use of their stages;
      // wait (bounded) until their bytes have landed before the CTA can exit.
      const uint32_t n_drain = issued < STAGES ? issued : STAGES;
      for (uint32_t i = 0; i < n_drain; ++i) {
        if (stage == 0) {
          stage = STAGES - 1;
          phase ^= 1u;
        } else {
          --stage;
        }
        ptx::mbar_wait_timeout(bar_full + 8 * stage, phase, kDrainLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!ptx::mbar_wait_bounded(bar_tempty + 8 * acc, acc_phase ^ 1u, abort, kWaitLimitNs)) {
          if (!*abort) record_timeout(2u, abort);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ptx::mbar_wait_bounded(bar_full + 8 * stage, phase, abort, kWaitLimitNs)) {
            if (!*abort) record_timeout(2u, abort);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint64_t adesc = ptx::sw128_kmajor_desc(sbase + OFF_A + stage * A_STAGE);
          const uint64_t bdesc = ptx::sw128_kmajor_desc(sbase + OFF_B + stage * B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // advance the start address by kk*32 bytes inside the swizzle atom
            const uint64_t koff = static_cast<uint64_t>((kk * UMMA_K) >> 4);
            ptx::mma_f8f6f4(d_tmem, adesc + koff, bdesc + koff, IDESC,
                            (kb | kk) != 0 ? 1u : 0u);
          }
          ptx::mma_commit(bar_empty + 8 * stage);  // stage reusable once these MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::mma_commit(bar_tfull + 8 * acc);  // accumulator complete
      }
      // No MMA may still be writing TMEM when the CTA frees it: commit everything
      // issued so far to the drain barrier and wait (bounded) for it. On the normal
      // path the last tile's MMAs are the only ones that can still be running.
      ptx::mma_commit(bar_drain);
      ptx::mbar_wait_timeout(bar_drain, 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int ew = warp - 2;
    const uint32_t buf0 = sbase + OFF_EPI + static_cast<uint32_t>(ew) * 2 * EPI_BUF;
    uint8_t *buf0_ptr = smem + OFF_EPI + ew * 2 * EPI_BUF;
    float *par_ws = reinterpret_cast<float *>(smem + OFF_PAR + ew * PAR_BYTES);
    float *par_b = par_ws + BN;
    uint32_t st_cnt = 0;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      int mt, nt;
      tile_coords(t, p.m_tiles, mt, nt);
      // Stage this tile's per-column w_scale and bias (as fp32) in the warp's own
      // smem slice while the main loop runs; columns past N read as 0.
      __syncwarp();
      for (int i = lane; i < BN; i += 32) {
        const int n = nt * BN + i;
        const bool in = n < p.N;
        par_ws[i] = in ? __ldg(p.ws + n) : 0.0f;
        par_b[i] = in ? load_bias(p.bias, p.bias_dtype, n) : 0.0f;
      }
      __syncwarp();
      if (!ptx::mbar_wait_bounded(bar_tfull + 8 * acc, acc_phase, abort, kWaitLimitNs)) {
        if (lane == 0 && !*abort) record_timeout(4u, abort);
        break;
      }
      ptx::tc_fence_after();
      const int row0 = mt * BM + quarter * 32;
      const int row = row0 + lane;
      const float xs = row < p.M ? __ldg(p.xs + row) : 0.0f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      const bool rows_live = row0 < p.M;  // a quarter wholly below M stores nothing
#pragma unroll 1
      for (int c = 0; c < BN / EPI_COLS; ++c) {
        const int n0 = nt * BN + c * EPI_COLS;
        if (n0 >= p.N || !rows_live) break;  // warp-uniform
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * EPI_COLS), r);
        ptx::tmem_wait_ld();
        uint32_t packed[16];
        const float4 *w4 = reinterpret_cast<const float4 *>(par_ws + c * EPI_COLS);
        const float4 *b4 = reinterpret_cast<const float4 *>(par_b + c * EPI_COLS);
#pragma unroll
        for (int j4 = 0; j4 < EPI_COLS / 4; ++j4) {
          const float4 w = w4[j4];
          const float4 bb = b4[j4];
          const float v0 = fmaf(__uint_as_float(r[4 * j4 + 0]) * xs, w.x, bb.x);
          const float v1 = fmaf(__uint_as_float(r[4 * j4 + 1]) * xs, w.y, bb.y);
          const float v2 = fmaf(__uint_as_float(r[4 * j4 + 2]) * xs, w.z, bb.z);
          const float v3 = fmaf(__uint_as_float(r[4 * j4 + 3]) * xs, w.w, bb.w);
          if (p.out_dtype == kF16) {
            packed[2 * j4] = ptx::pack_f16x2(v0, v1);
            packed[2 * j4 + 1] = ptx::pack_f16x2(v2, v3);
          } else {
            packed[2 * j4] = ptx::pack_bf16x2(v0, v1);
            packed[2 * j4 + 1] = ptx::pack_bf16x2(v2, v3);
          }
        }
        // Reuse a staging buffer only after the store issued two boxes ago has read it.
        if (lane == 0) ptx::bulk_wait_group_read<1>();
        __syncwarp();
        const uint32_t b = st_cnt & 1u;
        uint8_t *dst = buf0_ptr + b * EPI_BUF + lane * 64;
        const int sw = (lane >> 1) & 3;  // 64-byte swizzle: 16B chunk ^= offset bits 7..8
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          *reinterpret_cast<uint4 *>(dst + ((q ^ sw) << 4)) = v;
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_2d(&tmap_out, buf0 + b * EPI_BUF, n0, row0);
          ptx::bulk_commit_group();
        }
        ++st_cnt;
      }
      // All TMEM reads of this accumulator are complete (wait::ld above): release it.
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_tempty + 8 * acc);
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  __syncwarp();  // role loops ran on single lanes: reconverge before the CTA barrier
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool make_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle, std::string *err) {
  auto fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is unavailable (driver entry point query failed)";
    return false;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

}  // namespace gemm

int launch_gemm(const GemmArgs &a, cudaStream_t stream, bool pdl) {
  using namespace gemm;
  if (a.M == 0 || a.N == 0) return 0;
  DeviceInfo dev;
  if (!current_device_info(&dev)) return 5;
  if (dev.cc_major != 10) {
    set_error("fp8_gemm needs an sm_100 (B200-class) device; current device is sm_" +
              std::to_string(dev.cc_major) + std::to_string(dev.cc_minor));
    return 5;
  }
  if (a.M > 0x7fffffffLL || a.N > 0x7fffffffLL || a.K > 0x7fffffffLL) {
    set_error("fp8_gemm: dimensions must fit in int32");
    return 2;
  }
  std::string err;
  CUtensorMap ta, tb, tout;
  if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.xq, a.K, a.M, a.K, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B, &err) ||
      !make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wq, a.K, a.N, a.K, BK, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B, &err) ||
      !make_tmap_2d(&tout,
                    a.out_dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                    a.out, a.N, a.M, a.N * 2, EPI_COLS, 32, CU_TENSOR_MAP_SWIZZLE_64B, &err)) {
    set_error("fp8_gemm: " + err);
    return 4;
  }
  Params p;
  p.xs = a.xs;
  p.ws = a.ws;
  p.bias = a.bias;
  p.bias_dtype = a.bias ? a.bias_dtype : kNone;
  p.out_dtype = a.out_dtype;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.m_tiles = static_cast<int>((a.M + BM - 1) / BM);
  p.n_tiles = static_cast<int>((a.N + BN - 1) / BN);
  p.k_blocks = static_cast<int>((a.K + BK - 1) / BK);
  p.pdl = pdl ? 1 : 0;
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  if (tiles > 0x7fffffffLL) {
    set_error("fp8_gemm: too many output tiles");
    return 2;
  }
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.sm_count));

  static std::once_flag attr_once[64];
  cudaError_t ce = cudaSuccess;
  std::call_once(attr_once[dev.device & 63], [&] {
    ce = cudaFuncSetAttribute(fp8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(SMEM_BYTES));
  });
  if (ce != cudaSuccess) {
    set_error(std::string("fp8_gemm: cudaFuncSetAttribute: ") + cudaGetErrorString(ce));
    return 4;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ce = cudaLaunchKernelEx(&cfg, fp8_gemm_kernel, ta, tb, tout, p);
  if (ce != cudaSuccess) {
    set_error(std::string("fp8_gemm: launch failed: ") + cudaGetErrorString(ce));
    return 4;
  }
  return 0;
}

cudaError_t read_gemm_status(unsigned int *bits, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(bits, g_gemm_status, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(unsigned int));
  }
  return e;
}

}  // namespace fp8lin
