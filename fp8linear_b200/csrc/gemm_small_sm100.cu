// gemm_small_sm100.cu -- the FP8 GEMM + fused dequant/bias epilogue for few tokens
// (M <= 128, and M <= 256 where it gets a K-split), where the work is streaming the weight
// matrix once. Tokens go in blocks of 128 (grid y); each (weight tile, token block) pair
// is one cluster. Per-token e4m3 operands with at most 16 tokens, and MXFP8 with at most 8
// (K % 128 == 0), go to the warp-level kernel at the end of this file instead (whole
// weight rows per CTA, no cluster).
//
// Same result as fp8_gemm_kernel (out[m,n] = fma(acc * x_scale[m], w_scale[n], bias[n]),
// acc = e4m3 dot products accumulated in fp32), organised for a weight-bandwidth-bound
// shape:
//  * swap-AB: the MMA computes D^T = W . X^T, so 128 weight rows fill the tensor core's
//    M = 128 and the tokens (padded to a multiple of 16) are its N, instead of 127 of 128
//    MMA rows multiplying zero padding;
//  * split-K over a thread-block cluster of S CTAs (grid = ceil(N/128) x S, about one
//    CTA per SM): CTA r of a cluster streams K-blocks [r*kps, (r+1)*kps) of a 128-row
//    weight tile, so every SM pulls a slice of the weights;
//  * the S partial tiles meet in distributed shared memory: each CTA parks its fp32
//    partial [tokens x 128] in its own shared memory, and after a cluster barrier CTA r
//    reduces rows [r*R, (r+1)*R) of the tile over all S CTAs (fixed order, so the result
//    is deterministic), applies the scales and bias and writes bf16 (or fp16).
// Warp roles as in the large kernel: warp 0 TMA producer, warp 1 MMA issuer (+ TMEM
// owner), warps 2-5 move the accumulator from TMEM to shared memory; all warps reduce.
// Every mbarrier wait is bounded; a wait that runs out sets bit 16 of this file's
// watchdog word (read with the others by fp8lin_device_status) and the CTA winds down.
//
// The block-scaled forms (template parameter F: MXFP8, e4m3 codes with an e8m0 scale per
// 32 K-elements; NVFP4, e2m1 codes two per byte with a ue4m3 scale per 16) keep the same
// tiling, byte for byte along K (a K-block is 128 bytes of a row), and add to each stage
// the K-block's scale tiles in the quantizers' tiled layout (512-byte tiles of 128 rows x
// 4 scales): 1 (MX) or 4 (NV) tiles of the weight tile's 128 rows and as many of token
// rows 0-127. Before the K-block's MMAs they are copied into TMEM after the accumulator
// (tcgen05.cp .32x128b.warpx4, 4 columns per tile; weight scales are the MMA's scale A,
// token scales its scale B, of which an MMA with N = padded tokens reads rows 0..N-1). The
// scales are inside the accumulator, so the reduction adds only the bias.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "internal.h"
#include "ptx.cuh"

namespace fp8lin {

__device__ unsigned int g_small_status;  // watchdog bits (16 = small-M GEMM wait ran out)

namespace small {

constexpr int WN = 128;        // weight rows per CTA = MMA M
constexpr int BK = 128;        // bytes (= e4m3 elements) per K-block
constexpr int UMMA_K = 32;
constexpr int MAX_TOK = 128;   // tokens per launch (MMA N after padding)
constexpr int STAGES = 4;
constexpr int NUM_THREADS = 192;
constexpr uint32_t W_STAGE = WN * BK;                     // 16 KB
constexpr uint32_t X_STAGE_MAX = MAX_TOK * BK;            // 16 KB
constexpr uint32_t PART_MAX = MAX_TOK * WN * 4;           // fp32 partial tile, 64 KB
// the reduction's operands that do not depend on the partials: x_scale of every token,
// w_scale and bias of this CTA's rows (staged before the cluster barrier)
constexpr uint32_t EPI_BYTES = (MAX_TOK + 2 * WN) * 4;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint64_t kDrainLimitNs = 1000000000ull;

// Operand formats, numbered as the large kernel's.
enum : int { kFmtE4M3 = 0, kFmtMX = 1, kFmtNV = 2 };

template <int F>
struct Cfg {
  static constexpr bool BS = F != kFmtE4M3;  // block-scaled
  static constexpr bool NV = F == kFmtNV;
  static constexpr int SF_TILES = NV ? 4 : BS ? 1 : 0;   // scale tiles per K-block and operand
  static constexpr uint32_t SF_STAGE = 512u * SF_TILES;
  // stage: [weight 16 KB][tokens mpad x 128 B][weight scales][token scales]
  static constexpr uint32_t STAGE_MAX = W_STAGE + X_STAGE_MAX + 2 * SF_STAGE;
  static constexpr uint32_t OFF_PART = STAGES * STAGE_MAX;  // 128 / 136 / 160 KB
  static constexpr uint32_t OFF_EPI = OFF_PART + PART_MAX;
  static constexpr uint32_t OFF_BAR = OFF_EPI + EPI_BYTES;
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + (2 * STAGES + 2) * 8 + 16 + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(SF_STAGE % 512 == 0 && (2 * SF_STAGE) % 1024 == 0, "stages stay 1 KB aligned");
};

struct Params {
  const float *xs;
  const float *ws;
  const void *bias;
  int bias_dtype;
  void *out;
  int out_dtype;
  int M, N, K, ldo;
  int mpad;          // tokens padded to a multiple of 16 (MMA N)
  int k_blocks;
  int split;         // cluster size = K-splits per weight tile
  int kps;           // K-blocks per split
  uint32_t idesc;
  uint32_t tmem_cols;
  uint32_t sf_col;   // block-scaled: TMEM column of the weight scales (token scales follow)
  int pdl;
  int pre_w;         // weight boxes may be issued before the dependency wait
};

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

template <int F>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fp8_gemm_small_kernel(const __grid_constant__ CUtensorMap tmap_w,
                          const __grid_constant__ CUtensorMap tmap_x,
                          const __grid_constant__ CUtensorMap tmap_wsf,
                          const __grid_constant__ CUtensorMap tmap_xsf, const Params p) {
  using C = Cfg<F>;
  constexpr uint32_t OFF_PART = C::OFF_PART, OFF_EPI = C::OFF_EPI, OFF_BAR = C::OFF_BAR;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t x_stage = static_cast<uint32_t>(p.mpad) * BK;
  const uint32_t sf_off = W_STAGE + x_stage;  // weight scale tiles; token tiles follow
  const uint32_t stage_bytes = sf_off + 2 * C::SF_STAGE;  // multiple of 1 KB
  const uint32_t bar_full = sbase + OFF_BAR;
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_acc = bar_empty + 8 * STAGES;
  const uint32_t bar_drain = bar_acc + 8;
  volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + OFF_BAR +
                                                                       (2 * STAGES + 2) * 8);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + OFF_BAR + (2 * STAGES + 2) * 8 + 4);
  float *part = reinterpret_cast<float *>(smem + OFF_PART);  // [mpad][WN]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();  // K-split index
  const int tile = blockIdx.x / p.split;         // 128-row weight tile
  const int mb = blockIdx.y;                     // block of MAX_TOK tokens
  const int tok0 = mb * MAX_TOK;
  const int mrows = min(MAX_TOK, p.M - tok0);    // tokens of this block
  const int kb0 = static_cast<int>(rank) * p.kps;
  const int kb1 = min(p.k_blocks, kb0 + p.kps);
  const int nkb = kb1 - kb0;  // >= 1 (host guarantees)

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
    if constexpr (C::BS) {
      ptx::prefetch_tmap(&tmap_wsf);
      ptx::prefetch_tmap(&tmap_xsf);
    }
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);
    }
    ptx::mbar_init(bar_acc, 1);
    ptx::mbar_init(bar_drain, 1);
    *abort = 0;
    ptx::fence_mbar_init();
  }
  // The first stages' weight boxes (and weight scale tiles) go into shared memory at once
  // (each stage's barrier armed for all its boxes; the token boxes follow in the producer
  // loop), the rest of this CTA's K-range into L2. When the weights cannot depend on the
  // kernel this one overlaps (pre_w: that kernel is this call's quantizer), this happens
  // before the dependency wait, so the weight stream overlaps it. Otherwise the whole
  // K-range of the weight tile is prefetched into L2 before the wait (safe: writes of the
  // kernel before land in the same L2 lines) and the first stages are loaded after it.
  // (The first fill is unrolled over the compile-time ring, predicated on this CTA's
  // K-blocks: issued from runtime loops, copies took about twice as long to go out.)
  auto issue_weights = [&]() {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      if (i < nkb) {
        const uint32_t fb = bar_full + 8 * i;
        const uint32_t dst = sbase + static_cast<uint32_t>(i) * stage_bytes;
        ptx::mbar_arrive_expect_tx(fb, stage_bytes);
        ptx::tma_load_2d(dst, &tmap_w, (kb0 + i) * BK, tile * WN, fb);
        if constexpr (C::BS)
          ptx::tma_load_3d(dst + sf_off, &tmap_wsf, 0, (kb0 + i) * C::SF_TILES, tile, fb);
      }
    }
  };
  if (threadIdx.x == 0) {
    if (p.pre_w) issue_weights();
    for (int i = p.pre_w ? STAGES : 0; i < nkb; ++i)
      ptx::tma_prefetch_2d(&tmap_w, (kb0 + i) * BK, tile * WN);
  }
  if (warp == 1) {
    ptx::tmem_alloc<1>(ptx::smem_u32(const_cast<uint32_t *>(tmem_slot)), p.tmem_cols);
    ptx::tmem_relinquish<1>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (p.pdl) ptx::grid_dependency_wait();
  // Everything before this kernel has completed: its dependents may launch (they wait for
  // it in turn before touching memory).
  ptx::grid_launch_dependents();
  if (threadIdx.x == 0 && !p.pre_w) issue_weights();

  // The reduction's operands that do not depend on the partials (x_scale of this block's
  // tokens, w_scale and bias of the rows this CTA reduces), staged in shared memory by the
  // epilogue warps while the main loop runs.
  const int R = ((WN + p.split - 1) / p.split + 3) & ~3;
  const int r0 = static_cast<int>(rank) * R;
  const int r1 = min(WN, r0 + R);
  const int quads = r1 > r0 ? (r1 - r0) >> 2 : 0;
  float *e_xs = reinterpret_cast<float *>(smem + OFF_EPI);  // [MAX_TOK]
  float *e_ws = e_xs + MAX_TOK;                              // [WN]: rows r0.. of the tile
  float *e_b = e_ws + WN;
  if (warp >= 2) {
    const int et = threadIdx.x - 64;  // 0 .. 127
    // block-scaled: the scales are inside the accumulator, out = fma(acc * 1, 1, bias)
    for (int i = et; i < mrows; i += NUM_THREADS - 64)
      e_xs[i] = C::BS ? 1.0f : __ldg(p.xs + tok0 + i);
    for (int i = et; i < r1 - r0; i += NUM_THREADS - 64) {
      const int n = tile * WN + r0 + i;
      const bool in = n < p.N;
      e_ws[i] = in ? (C::BS ? 1.0f : __ldg(p.ws + n)) : 0.0f;
      e_b[i] = in && p.bias_dtype != kNone ? load_bias(p.bias, p.bias_dtype, n) : 0.0f;
    }
  }

  if (warp == 0) {
    if (lane == 0) {
      // the first fill's token boxes (its stages are armed and their weight boxes issued)
#pragma unroll
      for (int i = 0; i < STAGES; ++i) {
        if (i < nkb) {
          const uint32_t fb = bar_full + 8 * i;
          const uint32_t dst = sbase + static_cast<uint32_t>(i) * stage_bytes;
          ptx::tma_load_2d(dst + W_STAGE, &tmap_x, (kb0 + i) * BK, tok0, fb);
          if constexpr (C::BS)
            ptx::tma_load_3d(dst + sf_off + C::SF_STAGE, &tmap_xsf, 0, (kb0 + i) * C::SF_TILES,
                             mb, fb);
        }
      }
      int issued = nkb < STAGES ? nkb : STAGES;
      // refills: a stage is rewritten once the MMAs reading it have completed
      for (int i = STAGES; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t fb = bar_full + 8 * s;
        const uint32_t dst = sbase + static_cast<uint32_t>(s) * stage_bytes;
        const uint32_t ph = static_cast<uint32_t>(i / STAGES) & 1u;
        if (!ptx::mbar_wait_bounded(bar_empty + 8 * s, ph ^ 1u, abort, kWaitLimitNs)) {
          if (!*abort) {
            atomicOr(&g_small_status, 16u);
            *abort = 1;
          }
          break;
        }
        ptx::mbar_arrive_expect_tx(fb, stage_bytes);
        ptx::tma_load_2d(dst, &tmap_w, (kb0 + i) * BK, tile * WN, fb);
        if constexpr (C::BS)
          ptx::tma_load_3d(dst + sf_off, &tmap_wsf, 0, (kb0 + i) * C::SF_TILES, tile, fb);
        ptx::tma_load_2d(dst + W_STAGE, &tmap_x, (kb0 + i) * BK, tok0, fb);
        if constexpr (C::BS)
          ptx::tma_load_3d(dst + sf_off + C::SF_STAGE, &tmap_xsf, 0, (kb0 + i) * C::SF_TILES, mb,
                           fb);
        ++issued;
      }
      for (int i = issued - 1; i >= 0 && i >= issued - STAGES; --i)
        ptx::mbar_wait_timeout(bar_empty + 8 * (i % STAGES),
                               static_cast<uint32_t>(i / STAGES) & 1u, kDrainLimitNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = static_cast<uint32_t>(i / STAGES) & 1u;
        if (!ptx::mbar_wait_bounded(bar_full + 8 * s, ph, abort, kWaitLimitNs)) {
          if (!*abort) {
            atomicOr(&g_small_status, 16u);
            *abort = 1;
          }
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t st = sbase + static_cast<uint32_t>(s) * stage_bytes;
        const uint64_t adesc = ptx::sw128_kmajor_desc(st);
        const uint64_t bdesc = ptx::sw128_kmajor_desc(st + W_STAGE);
        const uint32_t sfa = tmem + p.sf_col;               // weight scales (scale A)
        const uint32_t sfb = sfa + 4u * C::SF_TILES;        // token scales (scale B)
        if constexpr (C::BS) {
          // this K-block's scale tiles into TMEM, ahead of its MMAs in the same pipe
#pragma unroll
          for (int j = 0; j < C::SF_TILES; ++j) {
            ptx::tmem_cp_32x128b_x4<1>(sfa + 4 * j, ptx::sf_block_desc(st + sf_off + 512 * j));
            ptx::tmem_cp_32x128b_x4<1>(
                sfb + 4 * j, ptx::sf_block_desc(st + sf_off + C::SF_STAGE + 512 * j));
          }
        }
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          const uint64_t koff = static_cast<uint64_t>((kk * UMMA_K) >> 4);
          const uint32_t accumulate = (i | kk) != 0 ? 1u : 0u;
          if constexpr (C::NV) {
            // 64 elements = the four 16-element scales of word kk of each row
            ptx::mma_nvf4<1>(tmem, adesc + koff, bdesc + koff, p.idesc, sfa + 4 * kk,
                             sfb + 4 * kk, accumulate);
          } else if constexpr (C::BS) {
            // scale byte kk of each row's word: the kk-th 32-element block
            const uint32_t sfid = static_cast<uint32_t>(kk) << 30;
            ptx::mma_mxf8f6f4<1>(tmem, adesc + koff, bdesc + koff,
                                 p.idesc | ptx::idesc_mx_e4m3(0, 0, kk), sfa | sfid,
                                 sfb | sfid, accumulate);
          } else {
            ptx::mma_f8f6f4(tmem, adesc + koff, bdesc + koff, p.idesc, accumulate);
          }
        }
        ptx::mma_commit(bar_empty + 8 * s);
      }
      if (ok) ptx::mma_commit(bar_acc);
      ptx::mma_commit(bar_drain);
      ptx::mbar_wait_timeout(bar_drain, 0, kDrainLimitNs);
    }
  } else {
    // TMEM (lane = weight row, column = token) -> part[token][row], fp32
    const int quarter = warp & 3;
    const bool ok = ptx::mbar_wait_bounded(bar_acc, 0, abort, kWaitLimitNs);
    if (!ok && lane == 0 && !*abort) {
      atomicOr(&g_small_status, 16u);
      *abort = 1;
    }
    ptx::tc_fence_after();
    const int row = quarter * 32 + lane;
    for (int c = 0; c < p.mpad; c += 16) {
      uint32_t r[16];
      if (ok) {
        ptx::tmem_ld_32x32b_x16(tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
                                    static_cast<uint32_t>(c),
                                r);
        ptx::tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(c + j) * WN + row] = __uint_as_float(r[j]);
    }
    ptx::tc_fence_before();
  }

  // CTA `rank` reduces tile rows [r0, r1) (a multiple of 4 wide) over the cluster's
  // partials and writes out.
  __syncwarp();
  __syncthreads();
  ptx::cluster_sync();  // every CTA's partial tile is in its shared memory

  // Each task is 4 consecutive rows of one token: the loads from all ranks' shared memory
  // are issued together, then summed in rank order.
  const uint32_t part_base = ptx::smem_u32(part);
  for (int idx = threadIdx.x; idx < mrows * quads; idx += NUM_THREADS) {
    const int m = idx / quads;
    const int nl = r0 + 4 * (idx - m * quads);
    const uint32_t off = static_cast<uint32_t>(m * WN + nl) * 4u;
    float4 v[8];
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2)
      if (s2 < p.split) v[s2] = ptx::ld_shared_cluster_v4(ptx::map_shared_rank(part_base + off, s2));
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2)
      if (s2 < p.split) {
        acc[0] += v[s2].x;
        acc[1] += v[s2].y;
        acc[2] += v[s2].z;
        acc[3] += v[s2].w;
      }
    const float xs = e_xs[m];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = tile * WN + nl + e;
      if (n >= p.N) break;
      const float val = fmaf(acc[e] * xs, e_ws[nl - r0 + e], e_b[nl - r0 + e]);
      const int64_t o = static_cast<int64_t>(tok0 + m) * p.ldo + n;
      if (p.out_dtype == kF16)
        reinterpret_cast<__half *>(p.out)[o] = __float2half_rn(val);
      else
        reinterpret_cast<__nv_bfloat16 *>(p.out)[o] = __float2bfloat16_rn(val);
    }
  }

  ptx::cluster_sync();  // peers may still be reading this CTA's partial tile
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<1>(tmem, p.tmem_cols);
  }
}

}  // namespace small

bool make_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                     uint32_t box_inner, uint32_t box_outer, std::string *err);
bool make_tmap_sf(CUtensorMap *map, const void *base, uint64_t rows, uint64_t ncb,
                  uint32_t tiles_per_box, std::string *err);
bool make_tmap_sf_box(CUtensorMap *map, const void *base, uint64_t rows, uint64_t ncb,
                      uint32_t box_words, uint32_t tiles_per_box, std::string *err);

namespace small {

template <int F>
int launch(const GemmArgs &a, const DeviceInfo &dev, cudaStream_t stream, bool pdl) {
  using C = Cfg<F>;
  const char *name = C::NV ? "nvfp4_gemm: " : C::BS ? "mxfp8_gemm: " : "fp8_gemm: ";
  std::string err;
  // tokens per block padded to a multiple of 16 (MMA N); blocks of MAX_TOK tokens
  const int mpad = a.M > MAX_TOK ? MAX_TOK : static_cast<int>((a.M + 15) / 16 * 16);
  const int nblk = static_cast<int>((a.M + MAX_TOK - 1) / MAX_TOK);
  // bytes of a row of codes (NV: two e2m1 codes per byte) and scale tiles per 128-row
  // block (4 scales of 32 (MX) or 16 (NV) elements per tile)
  const int64_t kbytes = C::NV ? a.K / 2 : a.K;
  const int64_t ncb = C::NV ? (a.K / 16 + 3) / 4 : (a.K / 32 + 3) / 4;
  CUtensorMap tw, tx, twsf, txsf;
  if (!make_tmap_2d_u8(&tw, a.wq, kbytes, a.N, BK, WN, &err) ||
      !make_tmap_2d_u8(&tx, a.xq, kbytes, a.M, BK, mpad, &err)) {
    set_error(name + err);
    return 4;
  }
  if constexpr (C::BS) {
    if (!make_tmap_sf(&twsf, a.wsf, a.N, ncb, C::SF_TILES, &err) ||
        !make_tmap_sf(&txsf, a.xsf, a.M, ncb, C::SF_TILES, &err)) {
      set_error(name + err);
      return 4;
    }
  } else {  // unused by the kernel: any valid map
    twsf = tw;
    txsf = tw;
  }
  Params p;
  p.xs = a.xs;
  p.ws = a.ws;
  p.bias = a.bias;
  p.bias_dtype = a.bias ? a.bias_dtype : kNone;
  p.out = a.out;
  p.out_dtype = a.out_dtype;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.ldo = static_cast<int>(a.ldo > 0 ? a.ldo : a.N);
  p.mpad = mpad;
  p.k_blocks = static_cast<int>((kbytes + BK - 1) / BK);
  const int tiles = static_cast<int>((a.N + WN - 1) / WN);

  static std::once_flag once[64];
  static cudaError_t setup_err[64];
  static int max_clusters[64][9];  // co-resident clusters per cluster size, per device
  const int d = dev.device & 63;
  std::call_once(once[d], [&] {
    cudaError_t ce = cudaFuncSetAttribute(fp8_gemm_small_kernel<F>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(C::SMEM_BYTES));
    for (int c = 1; c <= 8 && ce == cudaSuccess; ++c) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(c);
      q.blockDim = dim3(NUM_THREADS);
      q.dynamicSmemBytes = C::SMEM_BYTES;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = c;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      q.attrs = at;
      q.numAttrs = 1;
      int n = 0;
      ce = cudaOccupancyMaxActiveClusters(&n, fp8_gemm_small_kernel<F>, &q);
      max_clusters[d][c] = n;
    }
    setup_err[d] = ce;
  });
  if (setup_err[d] != cudaSuccess) {
    set_error(std::string(name) + "small kernel setup: " + cudaGetErrorString(setup_err[d]));
    return 4;
  }
  // K-splits (= cluster size): the largest, at most 8, whose co-resident clusters hold
  // every (weight tile, token block) pair in one wave; each split at least one K-block.
  int split = 1;
  for (int c = std::min(8, p.k_blocks); c >= 1; --c)
    if (max_clusters[d][c] >= tiles * nblk) {
      split = c;
      break;
    }
  // Above one token block, a launch without a K-split loses to the CTA-pair kernel.
  if (nblk > 1 && split < 2) return kSmallDeclined;
  p.kps = (p.k_blocks + split - 1) / split;
  split = (p.k_blocks + p.kps - 1) / p.kps;
  p.split = split;
  p.idesc = C::NV   ? ptx::idesc_nv_e2m1(WN, mpad)
            : C::BS ? ptx::idesc_mx_e4m3(WN, mpad, 0)
                    : ptx::idesc_e4m3_f32(WN, mpad);
  // accumulator in columns [0, mpad), then the scale tiles: 4 columns per tile and operand
  p.sf_col = static_cast<uint32_t>(mpad);
  const uint32_t used = p.sf_col + 8u * C::SF_TILES;
  uint32_t cols = 32;
  while (cols < used) cols <<= 1;
  p.tmem_cols = cols;
  p.pdl = pdl ? 1 : 0;
  p.pre_w = pdl && a.weights_before_wait ? 1 : 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * split, nblk);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int n = 1;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t ce =
      cudaLaunchKernelEx(&cfg, fp8_gemm_small_kernel<F>, tw, tx, twsf, txsf, p);
  if (ce != cudaSuccess) {
    set_error(std::string(name) + "small kernel launch failed: " + cudaGetErrorString(ce));
    return 4;
  }
  return 0;
}

}  // namespace small

// ---------------------------------------------------------------------------------------
// At most 16 tokens (e4m3): warp-level MMAs over whole weight rows, no K-split across CTAs.
//
// With 16 or fewer tokens the 128-row tcgen05 tile spreads the weight matrix over the SMs
// only by splitting K across a cluster, whose partial tiles then cross distributed shared
// memory (~20 GB/s per SM) between two cluster barriers. Here a CTA owns 16 whole weight
// rows (grid = ceil(N / 16), two CTAs per SM), so the weights still stream through every
// SM and the only reduction is between the CTA's own warps:
//  * warp 8 (one thread) streams K in stages of 1024 bytes through a ring of 3: per stage
//    and operand one TMA copy of a chunk view of the matrix (8 chunks of 128 bytes x 16
//    weight rows, or x 8 / 16 token rows; K % 128 == 0), else one 2-D box per chunk;
//    128-byte swizzle; rows past N or M and bytes past K arrive as zeros. The ring's first
//    fill is unrolled over its compile-time shape: issued from runtime loops, the copies
//    took about twice as long to go out. The weight rows are also prefetched into L2
//    before the dependency wait (L2 is where every SM's accesses meet, so this is safe
//    even while the kernel before writes them);
//  * warp w (0-7) takes chunk w of every stage: per 32-byte K-step one ldmatrix.x4 of the
//    weights (rows 0-7 / 8-15 x bytes 0-15 / 16-31 of the step) and one ldmatrix of the
//    tokens (8 tokens per fragment), the codes converted to f16 (exact) and summed by two
//    mma.sync.m16n8k16 f16 x f16 -> f32 per 8 tokens (swap-AB: weight rows are the MMA's
//    rows, tokens its columns), one accumulator set per K-step so the MMAs of a chunk do
//    not wait for one another; the 128-byte swizzle puts the 8 rows of each ldmatrix in 8
//    different bank groups;
//  * the eight warps' fp32 partials meet in shared memory (over the consumed ring) and are
//    summed in warp order (deterministic), then out = fma(acc * x_scale, w_scale, bias)
//    as in the other kernels.
// MXFP8 form (F = kFmtMX, at most 8 tokens, K % 128 == 0): a stage also carries, per
// operand, one 3-D copy of the 256-byte halves of its 8 scale tiles that hold the CTA's
// rows (a chunk is one tile column of 4 blocks). A 32-byte K-step is one 32-element block:
// its two MMAs sum into a zeroed temporary, which joins the accumulator as
// (sum * 2^(ea - 127)) * 2^(eb - 127) with the weight row's and the token's e8m0 scales.
// Waits are bounded as in the tcgen05 kernels (bit 16 of this file's watchdog word).
namespace rows {

constexpr int WR = 16;            // weight rows per CTA (the MMA's M)
constexpr int CHUNK = 128;        // K-bytes per TMA box (one swizzled 128-byte row)
constexpr int SC = 8;             // chunks per stage (1024 K-bytes)
constexpr int CONSUMERS = 8;      // consumer warps, one per chunk (16 measured no faster)
constexpr int KPW = (CHUNK / 32) * SC / CONSUMERS;  // K-steps per warp and stage (4)
constexpr int STAGES = 3;
constexpr int NUM_THREADS = 32 * (CONSUMERS + 1);
constexpr int MAX_TOK = 16;
constexpr uint32_t W_BOX = WR * CHUNK;                   // 2 KB
constexpr uint32_t RED_BYTES = CONSUMERS * MAX_TOK * WR * 4;     // 8 KB, over the ring
constexpr uint32_t PAR_BYTES = (MAX_TOK + 2 * WR) * 4;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint64_t kDrainLimitNs = 1000000000ull;

// MXFP8: per stage and operand the 256-byte halves of the stage's 8 scale tiles that hold
// the CTA's 16 rows (a tile holds 128 rows x 4 blocks of 32; a chunk is one tile column)
constexpr uint32_t SF_WIN = SC * 256;

// shared memory for `mpad` tokens per fragment set: [ring][params][barriers]; a stage is
// [weight boxes][token boxes][MX: weight and token scale windows]; the warps' partials
// overwrite the start of the ring once every stage has been consumed
__host__ __device__ constexpr uint32_t stage_bytes(int mpad, bool mx) {
  return SC * (W_BOX + static_cast<uint32_t>(mpad) * CHUNK) + (mx ? 2 * SF_WIN : 0u);
}
__host__ __device__ constexpr uint32_t off_par(int mpad, bool mx) {
  return STAGES * stage_bytes(mpad, mx);
}
__host__ __device__ constexpr uint32_t off_bar(int mpad, bool mx) {
  return off_par(mpad, mx) + PAR_BYTES;
}
__host__ __device__ constexpr uint32_t smem_bytes(int mpad, bool mx) {
  return off_bar(mpad, mx) + 2 * STAGES * 8 + 8 + 1024;  // + abort word, alignment slack
}
// two CTAs per SM (shared memory here; registers through the launch bounds)
static_assert(2 * (smem_bytes(MAX_TOK, true) + 1024) <= 233472, "shared memory budget");
static_assert(RED_BYTES <= STAGES * stage_bytes(8, false), "partials fit over the ring");

// an e8m0 scale as a float: 2^(e - 127) (e = 0: 2^-127, a subnormal)
__device__ __forceinline__ float e8m0_to_float(uint32_t e) {
  return __uint_as_float(e ? e << 23 : 0x00400000u);
}
static_assert(KPW * CONSUMERS == (CHUNK / 32) * SC, "K-steps split evenly");

struct Params {
  const uint8_t *wq;
  const float *xs;
  const float *ws;
  const void *bias;
  int bias_dtype;
  void *out;
  int out_dtype;
  int M, N, K, ldo;
  int chunks;   // ceil(K / 128)
  int wide;     // maps are chunk views: one copy per stage and operand (K % 128 == 0)
  int pdl;
  int pre_w;    // weight boxes may be issued before the dependency wait
};

template <int MPAD, int F>
__global__ void __launch_bounds__(NUM_THREADS, 2)
    fp8_gemm_rows_kernel(const __grid_constant__ CUtensorMap tmap_w,
                         const __grid_constant__ CUtensorMap tmap_x,
                         const __grid_constant__ CUtensorMap tmap_wsf,
                         const __grid_constant__ CUtensorMap tmap_xsf, const Params p) {
  constexpr bool MX = F == small::kFmtMX;
  constexpr uint32_t X_BOX = MPAD * CHUNK;
  constexpr uint32_t STAGE = stage_bytes(MPAD, MX);
  constexpr uint32_t SF_OFF = SC * (W_BOX + X_BOX);  // MX: weight window; token window next
  constexpr int NT = MPAD / 8;  // 8-token fragments
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar_full = sbase + off_bar(MPAD, MX);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  volatile int *abort = reinterpret_cast<volatile int *>(smem + off_bar(MPAD, MX) + 16 * STAGES);
  float *red = reinterpret_cast<float *>(smem);  // [warp][token][row], over the ring
  float *e_xs = reinterpret_cast<float *>(smem + off_par(MPAD, MX));  // [MAX_TOK]
  float *e_ws = e_xs + MAX_TOK;                                   // [WR]
  float *e_b = e_ws + WR;                                         // [WR]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * WR;
  // 128-byte chunks of K and stages (the last ones may be partial)
  const int chunks = p.chunks;
  const int nst = (chunks + SC - 1) / SC;
  auto chunks_of = [chunks](int i) { return min(SC, chunks - i * SC); };

  // MX: the CTA's rows sit in half h of their scale tiles, as 32-row group q
  const int sf_h = (n0 >> 4) & 1, sf_q = (n0 & 127) >> 5;
  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
    if constexpr (MX) {
      ptx::prefetch_tmap(&tmap_wsf);
      ptx::prefetch_tmap(&tmap_xsf);
    }
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, CONSUMERS);
    }
    *abort = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  // The first stages' weight copies, each stage armed for all its bytes (the token copies
  // follow after the dependency wait); before that wait only when the weights cannot
  // depend on the kernel this one overlaps (pre_w: it is this call's quantizer). The first
  // fill is unrolled over the compile-time ring, predicated on the real chunk count:
  // issued from runtime loops the same copies took twice as long to go out. With
  // chunk-view maps (wide) a stage is one copy per operand, the box's chunks past K
  // arriving as zeros (the consumers skip them); otherwise one 2-D box per chunk.
  const bool wide = p.wide != 0;
  auto stage_tx = [&](int i) {
    return static_cast<uint32_t>(wide ? SC : chunks_of(i)) * (W_BOX + X_BOX) +
           (MX ? 2 * SF_WIN : 0u);
  };
  // (MX runs with chunk views only: the host requires K % 128 == 0)
  auto load_w = [&](int i, uint32_t dst, uint32_t fb) {
    if (wide) {
      ptx::tma_load_3d(dst, &tmap_w, 0, n0, i * SC, fb);
      if constexpr (MX) ptx::tma_load_3d(dst + SF_OFF, &tmap_wsf, sf_h * 64, i * SC, n0 >> 7, fb);
    } else {
      const int cnt = chunks_of(i);
#pragma unroll
      for (int c = 0; c < SC; ++c)
        if (c < cnt) ptx::tma_load_2d(dst + c * W_BOX, &tmap_w, (i * SC + c) * CHUNK, n0, fb);
    }
  };
  auto load_x = [&](int i, uint32_t dst, uint32_t fb) {
    if (wide) {
      ptx::tma_load_3d(dst + SC * W_BOX, &tmap_x, 0, 0, i * SC, fb);
      if constexpr (MX) ptx::tma_load_3d(dst + SF_OFF + SF_WIN, &tmap_xsf, 0, i * SC, 0, fb);
    } else {
      const int cnt = chunks_of(i);
#pragma unroll
      for (int c = 0; c < SC; ++c)
        if (c < cnt)
          ptx::tma_load_2d(dst + SC * W_BOX + c * X_BOX, &tmap_x, (i * SC + c) * CHUNK, 0, fb);
    }
  };
  auto issue_weights = [&]() {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      if (i < nst) {
        const uint32_t fb = bar_full + 8 * i;
        ptx::mbar_arrive_expect_tx(fb, stage_tx(i));
        load_w(i, sbase + static_cast<uint32_t>(i) * STAGE, fb);
      }
    }
  };
  if (threadIdx.x == 32 * CONSUMERS) {
    // this CTA's weight rows (contiguous) into L2 whatever the launch mode, so the weight
    // stream overlaps the kernel before this one; then, under pre_w, the first stages
    ptx::bulk_prefetch_l2(p.wq + static_cast<int64_t>(n0) * p.K,
                          static_cast<uint32_t>(min(WR, p.N - n0)) * static_cast<uint32_t>(p.K));
    if (p.pre_w) issue_weights();
  }
  if (p.pdl) ptx::grid_dependency_wait();
  ptx::grid_launch_dependents();

  if (warp == CONSUMERS) {
    if (lane == 0) {
      if (!p.pre_w) issue_weights();
      // the first fill's token boxes (its stages are armed and their weight boxes issued)
#pragma unroll
      for (int i = 0; i < STAGES; ++i)
        if (i < nst) load_x(i, sbase + static_cast<uint32_t>(i) * STAGE, bar_full + 8 * i);
      int issued = nst < STAGES ? nst : STAGES;
      // refills: a stage is rewritten once its consumer warps have released it
      for (int i = STAGES; i < nst; ++i) {
        const int s = i % STAGES;
        const uint32_t fb = bar_full + 8 * s;
        const uint32_t dst = sbase + static_cast<uint32_t>(s) * STAGE;
        const uint32_t ph = static_cast<uint32_t>(i / STAGES) & 1u;
        if (!ptx::mbar_wait_bounded(bar_empty + 8 * s, ph ^ 1u, abort, kWaitLimitNs)) {
          if (!*abort) {
            atomicOr(&g_small_status, 16u);
            *abort = 1;
          }
          break;
        }
        ptx::mbar_arrive_expect_tx(fb, stage_tx(i));
        load_w(i, dst, fb);
        load_x(i, dst, fb);
        ++issued;
      }
      // no copy may still be landing when the CTA exits: wait for the last stages' data
      // (the loop stops early only at i >= STAGES, so every armed stage was issued)
      for (int i = issued - 1; i >= 0 && i >= issued - STAGES; --i)
        ptx::mbar_wait_timeout(bar_full + 8 * (i % STAGES),
                               static_cast<uint32_t>(i / STAGES) & 1u, kDrainLimitNs);
    }
  } else {
    // the epilogue's operands, loaded while the first stages land
    // (MX: the scales are inside the accumulator, out = fma(acc * 1, 1, bias))
    if (warp == 0 && lane < WR) {
      const int n = n0 + lane;
      const bool in = n < p.N;
      e_ws[lane] = in ? (MX ? 1.0f : __ldg(p.ws + n)) : 0.0f;
      e_b[lane] = in && p.bias_dtype != kNone ? small::load_bias(p.bias, p.bias_dtype, n) : 0.0f;
    } else if (warp == 1 && lane < MAX_TOK) {
      e_xs[lane] = lane < p.M ? (MX ? 1.0f : __ldg(p.xs + lane)) : 0.0f;
    }
    // Warp w takes chunk w % SC of every stage, K-steps [k0, k0 + KS) of it, with one
    // accumulator set per K-step so its MMAs do not wait for one another (a chained
    // mma.sync costs its full latency per step).
    constexpr int KS = KPW;
    const int cw = warp % SC;
    const int k0 = (warp / SC) * KS;
    float acc[KS][NT][4];
#pragma unroll
    for (int k = 0; k < KS; ++k)
#pragma unroll
      for (int j = 0; j < NT; ++j) acc[k][j][0] = acc[k][j][1] = acc[k][j][2] = acc[k][j][3] = 0.0f;
    // ldmatrix row addresses (lane 8j + i: row i of matrix j), 16-byte chunk index before
    // the swizzle: A matrices (rows 0-7 | 8-15) x (bytes 0-15 | 16-31) of a K-step; B
    // matrices (bytes 0-15 | 16-31) x (tokens 0-7 | 8-15).
    const int li = lane & 7, lj = lane >> 3;
    const uint32_t a_row = static_cast<uint32_t>(li + (lj & 1) * 8) * CHUNK;
    const int a_half = lj >> 1;
    const uint32_t b_row = static_cast<uint32_t>(li + (NT == 2 ? (lj >> 1) * 8 : 0)) * CHUNK;
    const int b_half = lj & 1;
    for (int i = 0; i < nst; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = static_cast<uint32_t>(i / STAGES) & 1u;
      // one lane per warp polls the barrier; the warp barrier then orders the other
      // lanes' reads after that lane's acquire
      int ok = 1;
      if (lane == 0) ok = ptx::mbar_wait_bounded(bar_full + 8 * s, ph, abort, kWaitLimitNs);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      __syncwarp();
      if (!ok) {
        if (lane == 0 && !*abort) {
          atomicOr(&g_small_status, 16u);
          *abort = 1;
        }
        break;
      }
      if (cw < chunks_of(i)) {
        const uint32_t wbox = sbase + static_cast<uint32_t>(s) * STAGE + cw * W_BOX;
        const uint32_t xbox = sbase + static_cast<uint32_t>(s) * STAGE + SC * W_BOX + cw * X_BOX;
        uint32_t a[KS][4], b[KS][4];
        // MX: the 4 block scales of this chunk for weight rows g, g + 8 and the lane's
        // tokens, one 32-bit word each (a row's scales of one tile are 4 consecutive bytes)
        uint32_t sw0 = 0, sw1 = 0, sx[NT][2] = {};
        if constexpr (MX) {
          const int g = lane >> 2, t = lane & 3;
          const uint8_t *sfw = smem + s * STAGE + SF_OFF + cw * 256 + sf_q * 4;
          const uint8_t *sfx = smem + s * STAGE + SF_OFF + SF_WIN + cw * 256;
          sw0 = *reinterpret_cast<const uint32_t *>(sfw + g * 16);
          sw1 = *reinterpret_cast<const uint32_t *>(sfw + (g + 8) * 16);
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            sx[j][0] = *reinterpret_cast<const uint32_t *>(sfx + (8 * j + 2 * t) * 16);
            sx[j][1] = *reinterpret_cast<const uint32_t *>(sfx + (8 * j + 2 * t + 1) * 16);
          }
        }
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int step = k0 + ks;
          ptx::ldsm_x4(wbox + a_row + (static_cast<uint32_t>((2 * step + a_half) ^ li) << 4), a[ks]);
          const uint32_t baddr = xbox + b_row + (static_cast<uint32_t>((2 * step + b_half) ^ li) << 4);
          if constexpr (NT == 2)
            ptx::ldsm_x4(baddr, b[ks]);
          else
            ptx::ldsm_x2(baddr, b[ks][0], b[ks][1]);
        }
        // Each 32-byte K-step as two f16 m16n8k16 MMAs (the codes convert to f16 exactly;
        // the e4m3 form of the warp-level MMA ran several times slower here). Lane 4g + t
        // holds bytes [4t, 4t + 4) of each 16-byte half; the MMA's K-slots (2t, 2t + 1) take
        // bytes (4t, 4t + 1) and slots (2t + 8, 2t + 9) bytes (4t + 2, 4t + 3), for weights
        // and tokens alike, so each MMA sums over exactly one half's 16 bytes.
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t af[8];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            af[4 * h + 0] = ptx::e4m3x2_to_f16x2(a[ks][2 * h], 0);
            af[4 * h + 1] = ptx::e4m3x2_to_f16x2(a[ks][2 * h + 1], 0);
            af[4 * h + 2] = ptx::e4m3x2_to_f16x2(a[ks][2 * h], 1);
            af[4 * h + 3] = ptx::e4m3x2_to_f16x2(a[ks][2 * h + 1], 1);
          }
          if constexpr (MX) {
            // the step is one 32-element block: its sum, scaled by the weight row's and
            // the token's 2^(e - 127), joins the accumulator ((sum * sa) * sb: a zero sum
            // stays zero whatever the scales); byte `step` of each scale word
            const int sh = 8 * (k0 + ks);
            const float sa0 = e8m0_to_float((sw0 >> sh) & 0xFFu);
            const float sa1 = e8m0_to_float((sw1 >> sh) & 0xFFu);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
              float tmp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t bv = b[ks][2 * j + h];
                ptx::mma_f16_16x8x16(tmp, af[4 * h], af[4 * h + 1], af[4 * h + 2],
                                     af[4 * h + 3], ptx::e4m3x2_to_f16x2(bv, 0),
                                     ptx::e4m3x2_to_f16x2(bv, 1));
              }
              const float sb0 = e8m0_to_float((sx[j][0] >> sh) & 0xFFu);
              const float sb1 = e8m0_to_float((sx[j][1] >> sh) & 0xFFu);
              acc[ks][j][0] = fmaf(tmp[0] * sa0, sb0, acc[ks][j][0]);
              acc[ks][j][1] = fmaf(tmp[1] * sa0, sb1, acc[ks][j][1]);
              acc[ks][j][2] = fmaf(tmp[2] * sa1, sb0, acc[ks][j][2]);
              acc[ks][j][3] = fmaf(tmp[3] * sa1, sb1, acc[ks][j][3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t bv = b[ks][2 * j + h];
                ptx::mma_f16_16x8x16(acc[ks][j], af[4 * h], af[4 * h + 1], af[4 * h + 2],
                                     af[4 * h + 3], ptx::e4m3x2_to_f16x2(bv, 0),
                                     ptx::e4m3x2_to_f16x2(bv, 1));
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
    }
    // this warp's partial [tokens][rows]: the K-step accumulators summed in order
#pragma unroll
    for (int k = 1; k < KS; ++k)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[0][j][e] += acc[k][j][e];
    // every consumer warp is past its last stage (and every stage it waited on has
    // landed), so the partials may overwrite the ring; the producer warp only waits on
    // barriers from here on
    asm volatile("bar.sync 1, %0;" ::"n"(32 * CONSUMERS) : "memory");
    const int g = lane >> 2, t = lane & 3;
    float *r = red + warp * (MAX_TOK * WR);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int tok = 8 * j + 2 * t;
      r[tok * WR + g] = acc[0][j][0];
      r[(tok + 1) * WR + g] = acc[0][j][1];
      r[tok * WR + g + 8] = acc[0][j][2];
      r[(tok + 1) * WR + g + 8] = acc[0][j][3];
    }
  }
  __syncwarp();
  __syncthreads();
  if (*abort) return;
  for (int idx = threadIdx.x; idx < p.M * WR; idx += NUM_THREADS) {
    const int tok = idx / WR, row = idx - tok * WR;
    const int n = n0 + row;
    if (n >= p.N) continue;
    float sum = red[tok * WR + row];
#pragma unroll
    for (int w = 1; w < CONSUMERS; ++w) sum += red[w * (MAX_TOK * WR) + tok * WR + row];
    const float val = fmaf(sum * e_xs[tok], e_ws[row], e_b[row]);
    const int64_t o = static_cast<int64_t>(tok) * p.ldo + n;
    if (p.out_dtype == kF16)
      reinterpret_cast<__half *>(p.out)[o] = __float2half_rn(val);
    else
      reinterpret_cast<__nv_bfloat16 *>(p.out)[o] = __float2bfloat16_rn(val);
  }
}

// MXFP8 (F = kFmtMX) is launched only for K % 128 == 0 (chunk views).
template <int MPAD, int F>
int launch(const GemmArgs &a, const DeviceInfo &dev, cudaStream_t stream, bool pdl) {
  constexpr bool MX = F == small::kFmtMX;
  const char *name = MX ? "mxfp8_gemm: " : "fp8_gemm: ";
  std::string err;
  CUtensorMap tw, tx, twsf, txsf;
  // chunk views (one copy per stage and operand) when K allows; 2-D boxes otherwise
  bool wide = a.K % CHUNK == 0 && make_tmap_chunks_u8(&tw, a.wq, a.K, a.N, WR, SC, &err) &&
              make_tmap_chunks_u8(&tx, a.xq, a.K, a.M, MPAD, SC, &err);
  if (MX && !wide) {
    set_error(std::string(name) + "warp-level kernel needs K % 128 == 0" +
              (err.empty() ? "" : ": " + err));
    return 4;
  }
  if (!wide && (!make_tmap_2d_u8(&tw, a.wq, a.K, a.N, CHUNK, WR, &err) ||
                !make_tmap_2d_u8(&tx, a.xq, a.K, a.M, CHUNK, MPAD, &err))) {
    set_error(name + err);
    return 4;
  }
  if constexpr (MX) {
    const uint64_t ncb = static_cast<uint64_t>((a.K / 32 + 3) / 4);
    if (!make_tmap_sf_box(&twsf, a.wsf, a.N, ncb, 64, SC, &err) ||
        !make_tmap_sf_box(&txsf, a.xsf, a.M, ncb, 64, SC, &err)) {
      set_error(name + err);
      return 4;
    }
  } else {  // unused by the kernel: any valid map
    twsf = tw;
    txsf = tw;
  }
  static std::once_flag once[64];
  static cudaError_t setup_err[64];
  const int d = dev.device & 63;
  std::call_once(once[d], [&] {
    setup_err[d] = cudaFuncSetAttribute(fp8_gemm_rows_kernel<MPAD, F>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem_bytes(MPAD, MX)));
  });
  if (setup_err[d] != cudaSuccess) {
    set_error(std::string(name) + "rows kernel setup: " + cudaGetErrorString(setup_err[d]));
    return 4;
  }
  Params p;
  p.wq = a.wq;
  p.xs = a.xs;
  p.ws = a.ws;
  p.bias = a.bias;
  p.bias_dtype = a.bias ? a.bias_dtype : kNone;
  p.out = a.out;
  p.out_dtype = a.out_dtype;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.ldo = static_cast<int>(a.ldo > 0 ? a.ldo : a.N);
  p.chunks = static_cast<int>((a.K + CHUNK - 1) / CHUNK);
  p.wide = wide ? 1 : 0;
  p.pdl = pdl ? 1 : 0;
  p.pre_w = pdl && a.weights_before_wait ? 1 : 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((a.N + WR - 1) / WR));
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem_bytes(MPAD, MX);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t ce =
      cudaLaunchKernelEx(&cfg, fp8_gemm_rows_kernel<MPAD, F>, tw, tx, twsf, txsf, p);
  if (ce != cudaSuccess) {
    set_error(std::string(name) + "rows kernel launch failed: " + cudaGetErrorString(ce));
    return 4;
  }
  return 0;
}

}  // namespace rows

int launch_gemm_small(const GemmArgs &a, cudaStream_t stream, bool pdl) {
  DeviceInfo dev;
  if (!current_device_info(&dev)) return 5;
  if (a.nv) return small::launch<small::kFmtNV>(a, dev, stream, pdl);
  if (a.mx) {
    // MXFP8 on the warp-level kernel up to 8 tokens (one 8-token fragment set); at 9-16
    // tokens it measured faster alone but slower behind the quantizer than the
    // split-K kernel
    if (a.M <= 8 && a.K % rows::CHUNK == 0)
      return rows::launch<8, small::kFmtMX>(a, dev, stream, pdl);
    return small::launch<small::kFmtMX>(a, dev, stream, pdl);
  }
  if (a.M <= 8) return rows::launch<8, small::kFmtE4M3>(a, dev, stream, pdl);
  if (a.M <= rows::MAX_TOK) return rows::launch<16, small::kFmtE4M3>(a, dev, stream, pdl);
  return small::launch<small::kFmtE4M3>(a, dev, stream, pdl);
}

cudaError_t read_small_status(unsigned int *bits, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(bits, g_small_status, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_small_status, &zero, sizeof(unsigned int));
  }
  return e;
}

}  // namespace fp8lin
