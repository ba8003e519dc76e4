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
// Two shapes of the same kernel (template parameter CG = CTAs per MMA):
//   CG = 1: one CTA per SM owns 128 x 256 output tiles (tcgen05.mma.cta_group::1,
//           M=128 N=256 K=32); used when M <= 128.
//   CG = 2: a cluster of two CTAs (one per SM) owns 256 x 256 tiles
//           (tcgen05.mma.cta_group::2, M=256 N=256 K=32, issued by the leader CTA):
//           each CTA loads its 128 rows of A and its 128 rows of B, so every SM
//           streams 32 KB per 128-byte K-block instead of 48 KB. No TMA multicast.
// Per CTA: 6 warps, persistent over tiles.
//   warp 0     TMA producer: A/B K-blocks of 128 bytes into a shared-memory ring (128-byte
//              swizzle); CG = 2 signals the leader's "full" barrier (cta_group::2 load).
//   warp 1     MMA issuer (leader CTA): one thread issues the MMAs into one of two TMEM
//              accumulators (2 x 256 fp32 columns) and commits stage/accumulator barriers
//              (multicast to both CTAs of a pair).
//   warps 2-5  epilogue: tcgen05.ld 64 columns at a time from the warp's TMEM lane
//              quarter, apply scales + bias, pack to bf16, stage in 128-byte-swizzled
//              smem and TMA-store 32 x 64 boxes (128-byte rows: half the store requests of
//              64-byte rows, measured 6% faster). Double-buffered TMEM lets the epilogue of
//              tile i overlap the main loop of tile i+1.
// Tile order: consecutive tiles (run concurrently by the persistent CTAs) walk the output
// N-fastest when M >= N, M-fastest otherwise, so the larger operand streams from HBM once
// while the concurrent tiles share it through L2.
// Every mbarrier wait is bounded (kWaitLimitNs); a wait that runs out records a bit in
// g_gemm_status, tells the CTA's other roles to stop, drains in-flight copies and MMAs,
// and the CTA frees its TMEM and returns.
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

constexpr int BM = 128;  // rows of A per CTA
constexpr int BN = 256;  // output columns per tile (the widest; per-token e4m3 also 192)
constexpr int BK = 128;  // bytes == e4m3 elements per K-block (one 128B swizzle row)
constexpr int UMMA_K = 32;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int EPI_COLS = 64;                     // columns per output store box (128 B rows)
constexpr int TMEM_COLS = 2 * BN;
constexpr uint32_t A_STAGE = BM * BK;            // 16 KB
constexpr uint32_t EPI_BUF = 32 * EPI_COLS * 2;  // 4 KB: 32 rows x 64 cols x 2 B
constexpr uint32_t PAR_BYTES = 2 * BN * 4;       // per epilogue warp: w_scale + bias of a tile
constexpr uint32_t RING_BYTES = 160 * 1024;      // operand ring (both shapes)

// Operand formats (template parameter F):
//   kFmtE4M3  per-token x per-channel e4m3 (scales applied in the epilogue);
//   kFmtMX    MXFP8: e4m3 codes, one e8m0 scale per 32 K-elements of every row;
//   kFmtNV    NVFP4: e2m1 codes packed two per byte, one ue4m3 scale per 16 K-elements.
// Both block-scaled forms keep the operand pipeline byte for byte (a K-block is 128 bytes of
// a row: 128 e4m3 or 256 e2m1 elements, four MMAs of 32 bytes) and add the scale tiles of
// the K-block to each stage, in the tiled layout of the quantizers: 512-byte tiles of 128
// rows x 4 scales. MX: one tile per K-block for this CTA's 128 rows of A and two for the
// tile's 256 rows of B; NV: four and eight (every CTA of a pair holds the scales of all 256
// B rows, which the MMA reads for its N = 256). Before a K-block's MMAs they are copied into
// TMEM (tcgen05.cp .32x128b.warpx4, 4 columns per tile) next to the accumulators. To make
// room, the two accumulators overlap by one epilogue chunk: accumulator 0 = columns 0-255,
// accumulator 1 = columns 192-447, scale factors from column 448 (MX 12 columns, NV 48);
// the epilogue reads the shared chunk first and releases it before the rest (bar_tovl).
enum : int { kFmtE4M3 = 0, kFmtMX = 1, kFmtNV = 2 };

template <int CG, int F = kFmtE4M3, int NB = BN>
struct Cfg {
  static constexpr bool MX = F != kFmtE4M3;                    // block-scaled (MX or NV)
  static constexpr bool NV = F == kFmtNV;
  static constexpr int TILE_N = NB;                            // output columns per tile
  static constexpr int SF_TILES = NV ? 4 : 1;                  // scale tiles per K-block, row block
  static constexpr int B_ROWS = NB / CG;                       // B rows this CTA loads
  static constexpr uint32_t B_STAGE = B_ROWS * BK;             // 32 KB (CG 1) / 16 KB (CG 2)
  static constexpr uint32_t SFA_STAGE = MX ? 512u * SF_TILES : 0u;   // A scales of the K-block
  static constexpr uint32_t SFB_STAGE = MX ? 1024u * SF_TILES : 0u;  // B scales, all 256 rows
  static constexpr uint32_t STAGE = A_STAGE + B_STAGE + SFA_STAGE + SFB_STAGE;
  static constexpr uint32_t RING = MX ? 168u * 1024u : RING_BYTES;
  static constexpr int STAGES = RING / STAGE;  // 3 / 5 (MX: 3 / 5, NV: 3 / 4)
  static constexpr uint32_t TX_BYTES = CG * STAGE;             // bytes landing per stage
  static constexpr int TILE_M = BM * CG;
  static constexpr uint32_t OFF_A = 0;
  static constexpr uint32_t OFF_B = OFF_A + STAGES * A_STAGE;
  static constexpr uint32_t OFF_SFA = OFF_B + STAGES * B_STAGE;
  static constexpr uint32_t OFF_SFB = OFF_SFA + STAGES * SFA_STAGE;
  static constexpr uint32_t OFF_EPI = (OFF_SFB + STAGES * SFB_STAGE + 1023u) & ~1023u;
  static constexpr uint32_t OFF_PAR = OFF_EPI + EPI_WARPS * 2 * EPI_BUF;
  static constexpr uint32_t OFF_BAR = OFF_PAR + EPI_WARPS * PAR_BYTES;
  // full, empty, tfull x2, tempty x2, drain, overlap-chunk release (MX)
  static constexpr uint32_t NUM_BARS = 2 * STAGES + 6;
  static constexpr uint32_t OFF_TMEM_SLOT = OFF_BAR + NUM_BARS * 8;
  static constexpr uint32_t OFF_ABORT = OFF_TMEM_SLOT + 4;
  static constexpr uint32_t SMEM_BYTES = OFF_ABORT + 4 + 1024;  // + base alignment slack
  static constexpr uint32_t IDESC = ptx::idesc_e4m3_f32(TILE_M, NB);
  static constexpr uint32_t IDESC_MX =
      NV ? ptx::idesc_nv_e2m1(TILE_M, BN) : ptx::idesc_mx_e4m3(TILE_M, BN, 0);
  static constexpr uint32_t ACC1_COL = MX ? BN - EPI_COLS : NB;  // accumulator 1's column
  static constexpr uint32_t SFA_COL = 2 * BN - EPI_COLS;          // block scale factors:
  static constexpr uint32_t SFB_COL = SFA_COL + 4 * SF_TILES;     // A 4/tile, B 8/tile
  static_assert(STAGES * STAGE <= RING, "ring");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(OFF_B % 1024 == 0 && OFF_EPI % 1024 == 0, "swizzle atoms need 1024 B alignment");
  static_assert(!MX || SFB_COL + 8 * SF_TILES <= TMEM_COLS, "TMEM budget");
  static_assert(NB % EPI_COLS == 0 && NB <= BN && (NB == BN || !MX), "tile width");
};

constexpr uint64_t kWaitLimitNs = 4000000000ull;   // 4 s: far above any legitimate wait
constexpr uint64_t kDrainLimitNs = 1000000000ull;  // 1 s for in-flight copies on exit

struct Params {
  const float *xs;
  const float *ws;
  const void *bias;
  int bias_dtype;
  int out_dtype;
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int ncb;           // MX / NV: scale tiles per 128-row block (ceil(K / 128) / ceil(K / 64))
  int n_fastest;     // tile order
  int direct_store;  // rows not 16-byte multiples / unaligned: no TMA store
  int wide_store;    // N % 128 == 0, no peers: one store per two 64-column chunks
  void *out;         // output base (direct stores)
  int ldo;           // output row pitch (elements)
  int n_peers;       // peer copies of every output box (P2P stores)
  void *peers[kMaxPeers];
  int pdl;
};

__device__ __forceinline__ void tile_coords(const Params &p, int t, int &mt, int &nt) {
  if (p.n_fastest) {
    mt = t / p.n_tiles;
    nt = t - mt * p.n_tiles;
  } else {
    nt = t / p.m_tiles;
    mt = t - nt * p.m_tiles;
  }
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

template <int CG, int F, int NB>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_out,
                    const __grid_constant__ CUtensorMap tmap_sfa,
                    const __grid_constant__ CUtensorMap tmap_sfb,
                    const __grid_constant__ CUtensorMap tmap_out2, const Params p) {
  using C = Cfg<CG, F, NB>;
  constexpr bool MX = C::MX;
  constexpr bool NV = C::NV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const uint32_t bar_full = sbase + C::OFF_BAR;            // STAGES barriers
  const uint32_t bar_empty = bar_full + C::STAGES * 8;     // STAGES barriers
  const uint32_t bar_tfull = bar_empty + C::STAGES * 8;    // 2 barriers
  const uint32_t bar_tempty = bar_tfull + 2 * 8;           // 2 barriers
  const uint32_t bar_drain = bar_tempty + 2 * 8;           // MMA drain on the way out
  const uint32_t bar_tovl = bar_drain + 8;                 // MX: overlap chunk read
  volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + C::OFF_TMEM_SLOT);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::OFF_ABORT);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? ptx::cluster_ctarank() : 0u;  // 0 = leader (issues MMAs)
  const bool leader = rank == 0;
  const int group = blockIdx.x / CG;   // CTA pair (or single CTA) index
  const int n_groups = gridDim.x / CG;

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_out);
    if constexpr (MX) {
      ptx::prefetch_tmap(&tmap_sfa);
      ptx::prefetch_tmap(&tmap_sfb);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(bar_tfull + 8 * a, 1);
      ptx::mbar_init(bar_tempty + 8 * a, EPI_WARPS * CG);
    }
    ptx::mbar_init(bar_drain, 1);
    ptx::mbar_init(bar_tovl, EPI_WARPS * CG);
    *abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc<CG>(sbase + C::OFF_TMEM_SLOT, TMEM_COLS);
    ptx::tmem_relinquish<CG>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) ptx::cluster_sync();  // peer barriers initialised before any signal
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Everything above overlaps the previous kernel when launched as a PDL dependent;
  // nothing produced by it is read before this point.
  if (p.pdl) ptx::grid_dependency_wait();
  // Everything before this kernel has completed: its dependents may launch (they wait for
  // it in turn before touching memory).
  ptx::grid_launch_dependents();

  const int num_tiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = group; t < num_tiles && ok; t += n_groups) {
        int mt, nt;
        tile_coords(p, t, mt, nt);
        const int a_row = mt * C::TILE_M + static_cast<int>(rank) * BM;
        const int b_row = nt * NB + static_cast<int>(rank) * C::B_ROWS;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ptx::mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1u, abort, kWaitLimitNs)) {
            if (!*abort) record_timeout(1u, abort);
            ok = false;
            break;
          }
          const uint32_t fb = bar_full + 8 * stage;
          const uint32_t dst_a = sbase + C::OFF_A + stage * A_STAGE;
          const uint32_t dst_b = sbase + C::OFF_B + stage * C::B_STAGE;
          // block-scale tiles of this K-block: tiles kb * SF_TILES .. of a 128-row block
          // (coordinates tile, row block of the [row blocks][ncb][512 B] grids); tiles and
          // row blocks past the end read as zero (scales of codes that are zero fill).
          const int sf_tile = kb * C::SF_TILES;
          const int sfa_rb = a_row >> 7;
          const int sfb_rb = (nt * BN) >> 7;
          const uint32_t dst_sfa = sbase + C::OFF_SFA + stage * C::SFA_STAGE;
          const uint32_t dst_sfb = sbase + C::OFF_SFB + stage * C::SFB_STAGE;
          if constexpr (CG == 1) {
            ptx::mbar_arrive_expect_tx(fb, C::TX_BYTES);
            ptx::tma_load_2d(dst_a, &tmap_a, kb * BK, a_row, fb);
            ptx::tma_load_2d(dst_b, &tmap_b, kb * BK, b_row, fb);
            if constexpr (MX) {
              ptx::tma_load_3d(dst_sfa, &tmap_sfa, 0, sf_tile, sfa_rb, fb);
              ptx::tma_load_3d(dst_sfb, &tmap_sfb, 0, sf_tile, sfb_rb, fb);
              ptx::tma_load_3d(dst_sfb + C::SFB_STAGE / 2, &tmap_sfb, 0, sf_tile, sfb_rb + 1, fb);
            }
          } else {
            // Both CTAs' bytes complete the leader's barrier; only the leader arms it.
            if (leader) ptx::mbar_arrive_expect_tx(fb, C::TX_BYTES);
            const uint32_t fb_leader = ptx::map_shared_rank(fb, 0);
            ptx::tma_load_2d_pair(dst_a, &tmap_a, kb * BK, a_row, fb_leader);
            ptx::tma_load_2d_pair(dst_b, &tmap_b, kb * BK, b_row, fb_leader);
            if constexpr (MX) {
              ptx::tma_load_3d_pair(dst_sfa, &tmap_sfa, 0, sf_tile, sfa_rb, fb_leader);
              ptx::tma_load_3d_pair(dst_sfb, &tmap_sfb, 0, sf_tile, sfb_rb, fb_leader);
              ptx::tma_load_3d_pair(dst_sfb + C::SFB_STAGE / 2, &tmap_sfb, 0, sf_tile,
                                    sfb_rb + 1, fb_leader);
            }
          }
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: wait (bounded) until the MMAs have released the last min(issued, STAGES)
      // stages, i.e. every load issued here has landed and been consumed.
      const uint32_t n_drain = issued < C::STAGES ? issued : C::STAGES;
      for (uint32_t i = 0; i < n_drain; ++i) {
        if (stage == 0) {
          stage = C::STAGES - 1;
          phase ^= 1u;
        } else {
          --stage;
        }
        ptx::mbar_wait_timeout(bar_empty + 8 * stage, phase, kDrainLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = group; t < num_tiles && ok; t += n_groups, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!ptx::mbar_wait_bounded(bar_tempty + 8 * acc, acc_phase ^ 1u, abort, kWaitLimitNs)) {
          if (!*abort) record_timeout(2u, abort);
          break;
        }
        // MX: the previous tile's epilogue must also have read the chunk the accumulators
        // share before this tile's first MMA overwrites it.
        if (MX && it > 0 &&
            !ptx::mbar_wait_bounded(bar_tovl, static_cast<uint32_t>(it - 1) & 1u, abort,
                                    kWaitLimitNs)) {
          if (!*abort) record_timeout(2u, abort);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (acc ? C::ACC1_COL : 0u);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ptx::mbar_wait_bounded(bar_full + 8 * stage, phase, abort, kWaitLimitNs)) {
            if (!*abort) record_timeout(2u, abort);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint64_t adesc = ptx::sw128_kmajor_desc(sbase + C::OFF_A + stage * A_STAGE);
          const uint64_t bdesc = ptx::sw128_kmajor_desc(sbase + C::OFF_B + stage * C::B_STAGE);
          if constexpr (MX) {
            // this K-block's scales into TMEM, ahead of its MMAs in the same pipe: tile j
            // of A to columns SFA_COL + 4j, tile j of B rows 0-127 / 128-255 to
            // SFB_COL + 8j / + 8j + 4
            const uint32_t sfa_s = sbase + C::OFF_SFA + stage * C::SFA_STAGE;
            const uint32_t sfb_s = sbase + C::OFF_SFB + stage * C::SFB_STAGE;
#pragma unroll
            for (int j = 0; j < C::SF_TILES; ++j) {
              ptx::tmem_cp_32x128b_x4<CG>(tmem_base + C::SFA_COL + 4 * j,
                                          ptx::sf_block_desc(sfa_s + 512 * j));
              ptx::tmem_cp_32x128b_x4<CG>(tmem_base + C::SFB_COL + 8 * j,
                                          ptx::sf_block_desc(sfb_s + 512 * j));
              ptx::tmem_cp_32x128b_x4<CG>(tmem_base + C::SFB_COL + 8 * j + 4,
                                          ptx::sf_block_desc(sfb_s + C::SFB_STAGE / 2 + 512 * j));
            }
          }
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // advance the start address by kk*32 bytes inside the swizzle atom
            const uint64_t koff = static_cast<uint64_t>((kk * UMMA_K) >> 4);
            const uint32_t accumulate = (kb | kk) != 0 ? 1u : 0u;
            if constexpr (NV) {
              // 64 elements = four 16-element blocks = the whole scale word of tile kk
              ptx::mma_nvf4<CG>(d_tmem, adesc + koff, bdesc + koff, C::IDESC_MX,
                                tmem_base + C::SFA_COL + 4 * kk,
                                tmem_base + C::SFB_COL + 8 * kk, accumulate);
            } else if constexpr (MX) {
              // scale byte kk of each 32-bit scale word: the kk-th 32-element block
              const uint32_t sfid = static_cast<uint32_t>(kk) << 30;
              ptx::mma_mxf8f6f4<CG>(d_tmem, adesc + koff, bdesc + koff,
                                    C::IDESC_MX | ptx::idesc_mx_e4m3(0, 0, kk),
                                    (tmem_base + C::SFA_COL) | sfid,
                                    (tmem_base + C::SFB_COL) | sfid, accumulate);
            } else if constexpr (CG == 1) {
              ptx::mma_f8f6f4(d_tmem, adesc + koff, bdesc + koff, C::IDESC, accumulate);
            } else {
              ptx::mma_f8f6f4_pair(d_tmem, adesc + koff, bdesc + koff, C::IDESC, accumulate);
            }
          }
          // the stage is reusable (in both CTAs) once these MMAs have read it
          if constexpr (CG == 1)
            ptx::mma_commit(bar_empty + 8 * stage);
          else
            ptx::mma_commit_pair_mc(bar_empty + 8 * stage, 0x3);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // accumulator complete (both CTAs' halves)
        if constexpr (CG == 1)
          ptx::mma_commit(bar_tfull + 8 * acc);
        else
          ptx::mma_commit_pair_mc(bar_tfull + 8 * acc, 0x3);
      }
      // No MMA may still be running when the CTAs free TMEM: commit everything issued
      // so far to the drain barrier and wait (bounded) for it.
      if constexpr (CG == 1)
        ptx::mma_commit(bar_drain);
      else
        ptx::mma_commit_pair(bar_drain);
      ptx::mbar_wait_timeout(bar_drain, 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int ew = warp - 2;
    const uint32_t buf0 = sbase + C::OFF_EPI + static_cast<uint32_t>(ew) * 2 * EPI_BUF;
    uint8_t *buf0_ptr = smem + C::OFF_EPI + ew * 2 * EPI_BUF;
    float *par_ws = reinterpret_cast<float *>(smem + C::OFF_PAR + ew * PAR_BYTES);
    float *par_b = par_ws + BN;
    uint32_t st_cnt = 0;
    int it = 0;
    for (int t = group; t < num_tiles; t += n_groups, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      int mt, nt;
      tile_coords(p, t, mt, nt);
      // Stage this tile's per-column w_scale and bias (as fp32) in the warp's own
      // smem slice while the main loop runs; columns past N read as 0.
      __syncwarp();
      for (int i = lane; i < NB; i += 32) {
        const int n = nt * NB + i;
        const bool in = n < p.N;
        par_ws[i] = in ? (MX ? 1.0f : __ldg(p.ws + n)) : 0.0f;  // MX: scales are in acc
        par_b[i] = in ? load_bias(p.bias, p.bias_dtype, n) : 0.0f;
      }
      __syncwarp();
      if (!ptx::mbar_wait_bounded(bar_tfull + 8 * acc, acc_phase, abort, kWaitLimitNs)) {
        if (lane == 0 && !*abort) record_timeout(4u, abort);
        break;
      }
      ptx::tc_fence_after();
      const int row0 = mt * C::TILE_M + static_cast<int>(rank) * BM + quarter * 32;
      const int row = row0 + lane;
      const float xs = MX ? 1.0f : (row < p.M ? __ldg(p.xs + row) : 0.0f);
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             (acc ? C::ACC1_COL : 0u);
      const bool rows_live = row0 < p.M;  // a quarter wholly below M stores nothing
      // MX: the chunk the two accumulators share (accumulator 0's last, accumulator 1's
      // first) is read first and released on bar_tovl as soon as it is in registers, so
      // the next tile's first MMA waits for one TMEM load, not for a chunk's stores.
      bool ovl_done = !MX;
      auto release_overlap = [&]() {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1)
            ptx::mbar_arrive(bar_tovl);
          else
            ptx::mbar_arrive_cluster(ptx::map_shared_rank(bar_tovl, 0));
        }
        ovl_done = true;
      };
#pragma unroll 1
      for (int ci = 0; ci < NB / EPI_COLS; ++ci) {
        if (MX && ci == 1 && !ovl_done) release_overlap();
        // MX, accumulator 0: chunks in descending order, the shared (last) one first; the
        // pairs stored together, {3, 2} and {1, 0}, stay adjacent
        const int c = (MX && acc == 0) ? NB / EPI_COLS - 1 - ci : ci;
        const int n0 = nt * NB + c * EPI_COLS;
        if (!rows_live) break;   // warp-uniform
        if (n0 >= p.N) {
          if (MX) continue;      // chunk order is not ascending
          break;
        }
        uint32_t r[64];
        ptx::tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * EPI_COLS),
                                *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        ptx::tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * EPI_COLS + 32),
                                *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        ptx::tmem_wait_ld();
        if (MX && !ovl_done) release_overlap();  // chunk 0 is the shared one
        uint32_t packed[32];
        const float4 *w4 = reinterpret_cast<const float4 *>(par_ws + c * EPI_COLS);
        const float4 *b4 = reinterpret_cast<const float4 *>(par_b + c * EPI_COLS);
#pragma unroll
        for (int j4 = 0; j4 < EPI_COLS / 4; ++j4) {
          const float4 w = w4[j4];
          const float4 bb = b4[j4];
          // fmaf(acc * x_scale, w_scale, bias), two columns per instruction
          const float2 v01 = ptx::mul_fma2(
              make_float2(__uint_as_float(r[4 * j4 + 0]), __uint_as_float(r[4 * j4 + 1])), xs,
              make_float2(w.x, w.y), make_float2(bb.x, bb.y));
          const float2 v23 = ptx::mul_fma2(
              make_float2(__uint_as_float(r[4 * j4 + 2]), __uint_as_float(r[4 * j4 + 3])), xs,
              make_float2(w.z, w.w), make_float2(bb.z, bb.w));
          const float v0 = v01.x, v1 = v01.y, v2 = v23.x, v3 = v23.y;
          if (p.out_dtype == kF16) {
            packed[2 * j4] = ptx::pack_f16x2(v0, v1);
            packed[2 * j4 + 1] = ptx::pack_f16x2(v2, v3);
          } else {
            packed[2 * j4] = ptx::pack_bf16x2(v0, v1);
            packed[2 * j4 + 1] = ptx::pack_bf16x2(v2, v3);
          }
        }
        const uint32_t b = st_cnt & 1u;
        if (p.wide_store) {
          // Chunks 2k and 2k + 1 fill the two 4 KB halves of the warp's 8 KB box (each in
          // the 32 x 64 swizzled layout below) and leave in one 3-D store once both are
          // staged: tmap_out2 views the output as [N / 64 chunks][M rows][64 columns],
          // box {64, 32, 2}. N % 128 == 0, so a pair is wholly inside or outside N.
          const bool first = (ci & 1) == 0;  // first of its pair in processing order
          if (first) {
            if (lane == 0) ptx::bulk_wait_group_read<0>();  // the previous box has been read
            __syncwarp();
          }
          uint8_t *dst = buf0_ptr + (c & 1) * EPI_BUF + lane * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4 *>(dst + ((q ^ (lane & 7)) << 4)) = make_uint4(
                packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          if (!first) {
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              ptx::tma_store_3d(&tmap_out2, buf0, 0, row0, (n0 / EPI_COLS) & ~1);
              ptx::bulk_commit_group();
            }
          }
        } else if (!p.direct_store) {
          // Reuse a staging buffer only after the store issued two boxes ago has read it.
          if (lane == 0) ptx::bulk_wait_group_read<1>();
          __syncwarp();
          // row `lane` of the box: 8 16-byte chunks, 128-byte swizzle (chunk ^= row % 8)
          uint8_t *dst = buf0_ptr + b * EPI_BUF + lane * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4 *>(dst + ((q ^ (lane & 7)) << 4)) = make_uint4(
                packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(&tmap_out, buf0 + b * EPI_BUF, n0, row0);
            ptx::bulk_commit_group();
          }
          if (p.n_peers > 0) {
            // Same box to every peer GPU's buffer over NVLink: re-read it coalesced
            // (lane -> row 4i + lane/8, 16-byte chunk lane%8), one full 128-byte line
            // per 8 lanes per store instruction. Plain P2P stores; no TMA to peers.
            const int pr = lane >> 3, pc = lane & 7;
            const uint8_t *box = buf0_ptr + b * EPI_BUF;
            uint4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = 4 * i + pr;
              v[i] = *reinterpret_cast<const uint4 *>(box + rr * 128 + ((pc ^ (rr & 7)) << 4));
            }
            const bool col_ok = n0 + pc * 8 < p.N;
            for (int q = 0; q < p.n_peers; ++q) {
              uint16_t *dst = reinterpret_cast<uint16_t *>(p.peers[q]);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int rr = row0 + 4 * i + pr;
                if (col_ok && rr < p.M)
                  *reinterpret_cast<uint4 *>(dst + static_cast<int64_t>(rr) * p.ldo + n0 + pc * 8) =
                      v[i];
              }
            }
            __syncwarp();
          }
        } else {
          // Row pitch not a multiple of 16 bytes: transpose the 32 x 64 box through smem
          // so that each store instruction writes 32 consecutive columns of one row.
          uint8_t *box = buf0_ptr + b * EPI_BUF;
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4 *>(box + lane * 128 + q * 16) = make_uint4(
                packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          __syncwarp();
          const uint16_t *box16 = reinterpret_cast<const uint16_t *>(box);
          uint16_t *out16 = reinterpret_cast<uint16_t *>(p.out);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int col = n0 + h * 32 + lane;
            if (col < p.N) {
              for (int r2 = 0; r2 < 32 && row0 + r2 < p.M; ++r2)
                out16[static_cast<int64_t>(row0 + r2) * p.ldo + col] = box16[r2 * 64 + h * 32 + lane];
            }
          }
        }
        ++st_cnt;
      }
      if (MX && !ovl_done) release_overlap();
      // All TMEM reads of this accumulator are complete (wait::ld above): release it to
      // the MMA issuer (the leader CTA's barrier for a pair).
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 1)
          ptx::mbar_arrive(bar_tempty + 8 * acc);
        else
          ptx::mbar_arrive_cluster(ptx::map_shared_rank(bar_tempty + 8 * acc, 0));
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    // Peer copies are plain stores to other GPUs' memory: make them visible system-wide
    // before this kernel's completion is signalled to anything that reads them.
    if (p.n_peers > 0) __threadfence_system();
    __syncwarp();
  }

  __syncwarp();  // role loops ran on single lanes: reconverge before the CTA barrier
  ptx::tc_fence_before();
  __syncthreads();
  // A pair stays resident until both CTAs are done: the leader's MMAs read the peer's
  // shared memory and write its TMEM, and the peer arrives on the leader's barriers.
  if constexpr (CG == 2) ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<CG>(tmem_base, TMEM_COLS);
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

// [outer][mid][inner] array with byte strides mid_bytes / outer_bytes, box
// box_inner x box_mid x 1, no swizzle: the block-scale grids as
// [128-row blocks][scale tiles][128 words of 4 scales].
bool make_tmap_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                  uint64_t mid, uint64_t outer, uint64_t mid_bytes, uint64_t outer_bytes,
                  uint32_t box_inner, uint32_t box_mid, std::string *err) {
  auto fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is unavailable (driver entry point query failed)";
    return false;
  }
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {mid_bytes, outer_bytes};
  cuuint32_t box[3] = {box_inner, box_mid, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

// The output [M, ldo] (16-bit elements, N % 64 == 0) as [N / 64 chunks][M rows][64 columns]:
// a box {64, 32, 2} is two adjacent 64-column chunks of 32 rows, 128-byte swizzled.
bool make_tmap_out_wide(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                        uint64_t M, uint64_t N, uint64_t ldo, std::string *err) {
  auto fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is unavailable (driver entry point query failed)";
    return false;
  }
  cuuint64_t dims[3] = {64, M, N / 64};
  cuuint64_t strides[2] = {ldo * 2, 128};
  cuuint32_t box[3] = {64, 32, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
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

// Per-device launch facts of one kernel shape: smem attribute set, co-resident groups.
struct LaunchInfo {
  bool ready = false;
  cudaError_t err = cudaSuccess;
  int max_groups = 0;
};

template <int CG, int F, int NB>
LaunchInfo &launch_info(int device, int sm_count) {
  static LaunchInfo info[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  LaunchInfo &li = info[device & 63];
  if (!li.ready) {
    li.ready = true;
    li.err = cudaFuncSetAttribute(fp8_gemm_kernel<CG, F, NB>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(Cfg<CG, F, NB>::SMEM_BYTES));
    li.max_groups = sm_count / CG;
    if (li.err == cudaSuccess && CG == 2) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sm_count);
      cfg.blockDim = dim3(NUM_THREADS);
      cfg.dynamicSmemBytes = Cfg<CG, F, NB>::SMEM_BYTES;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = CG;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      li.err = cudaOccupancyMaxActiveClusters(&clusters, fp8_gemm_kernel<CG, F, NB>, &cfg);
      if (li.err == cudaSuccess) li.max_groups = std::min(li.max_groups, clusters);
      if (li.err == cudaSuccess && li.max_groups < 1) li.err = cudaErrorInvalidConfiguration;
    }
  }
  return li;
}

template <int CG, int F, int NB = BN>
int launch_shape(const GemmArgs &a, const DeviceInfo &dev, cudaStream_t stream, bool pdl) {
  using C = Cfg<CG, F, NB>;
  constexpr bool MX = C::MX;
  const char *name = C::NV ? "nvfp4_gemm: " : MX ? "mxfp8_gemm: " : "fp8_gemm: ";
  std::string err;
  CUtensorMap ta, tb, tout, tsfa, tsfb;
  // bytes of a row of codes (NV: two e2m1 codes per byte) and scale tiles per 128-row
  // block (4 scales of 32 (MX) or 16 (NV) elements per tile)
  const int64_t kbytes = C::NV ? a.K / 2 : a.K;
  const int64_t ncb = C::NV ? (a.K / 16 + 3) / 4 : (a.K / 32 + 3) / 4;
  if constexpr (MX) {
    // the tiled scale grids as [row blocks][ncb tiles][128 words]; a box is the
    // SF_TILES tiles of one K-block of one row block
    const uint64_t rb_a = static_cast<uint64_t>((a.M + 127) / 128);
    const uint64_t rb_b = static_cast<uint64_t>((a.N + 127) / 128);
    const uint64_t nt = static_cast<uint64_t>(ncb);
    if (!make_tmap_3d(&tsfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.xsf, 128, nt, rb_a, 512, nt * 512,
                      128, C::SF_TILES, &err) ||
        !make_tmap_3d(&tsfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.wsf, 128, nt, rb_b, 512, nt * 512,
                      128, C::SF_TILES, &err)) {
      set_error(name + err);
      return 4;
    }
  }
  const int64_t ldo = a.ldo > 0 ? a.ldo : a.N;
  const bool direct = (a.N % 8) != 0 || (ldo % 8) != 0 ||
                      (reinterpret_cast<uintptr_t>(a.out) % 16) != 0;
  if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.xq, kbytes, a.M, kbytes, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B, &err) ||
      !make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wq, kbytes, a.N, kbytes, BK, C::B_ROWS,
                    CU_TENSOR_MAP_SWIZZLE_128B, &err) ||
      // rows of N bf16 are a 16-byte multiple only for N % 8 == 0: otherwise the
      // epilogue stores directly and the (unused) output map is a placeholder over xq
      !make_tmap_2d(&tout,
                    a.out_dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                    direct ? static_cast<const void *>(a.xq) : a.out, direct ? 8 : a.N, direct ? 1 : a.M, direct ? 16 : ldo * 2,
                    direct ? 8 : EPI_COLS, direct ? 1 : 32, direct ? CU_TENSOR_MAP_SWIZZLE_NONE
                                                             : CU_TENSOR_MAP_SWIZZLE_128B,
                    &err)) {
    set_error(name + err);
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
  p.m_tiles = static_cast<int>((a.M + C::TILE_M - 1) / C::TILE_M);
  p.n_tiles = static_cast<int>((a.N + NB - 1) / NB);
  p.k_blocks = static_cast<int>((kbytes + BK - 1) / BK);
  p.ncb = static_cast<int>(ncb);
  p.n_fastest = a.M >= a.N ? 1 : 0;
  p.direct_store = direct ? 1 : 0;
  CUtensorMap tout2 = tout;
  p.wide_store = 0;
  // (paired 64-column chunks stay inside a tile only at width 256)
  if (NB == BN && !direct && a.n_peers == 0 && a.N % 128 == 0) {
    std::string werr;  // a view the driver does not take: 64-column boxes instead
    if (make_tmap_out_wide(&tout2,
                           a.out_dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           a.out, a.M, a.N, ldo, &werr))
      p.wide_store = 1;
    else
      tout2 = tout;
  }
  p.out = a.out;
  p.ldo = static_cast<int>(ldo);
  p.n_peers = a.n_peers;
  for (int i = 0; i < kMaxPeers; ++i) p.peers[i] = i < a.n_peers ? a.peers[i] : nullptr;
  if (a.n_peers > 0 && direct) {
    set_error("fp8_gemm: peer outputs need 16-byte rows (N and the row pitch multiples of 8, "
              "16-byte aligned buffers)");
    return 2;
  }
  p.pdl = pdl ? 1 : 0;
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  if (tiles > 0x7fffffffLL) {
    set_error("fp8_gemm: too many output tiles");
    return 2;
  }
  LaunchInfo &li = launch_info<CG, F, NB>(dev.device, dev.sm_count);
  if (li.err != cudaSuccess) {
    set_error(std::string("fp8_gemm: kernel setup: ") + cudaGetErrorString(li.err));
    return 4;
  }
  const int groups = static_cast<int>(std::min<int64_t>(tiles, li.max_groups));

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups * CG);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (CG == 2) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = CG;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if constexpr (!MX) {  // unused by the kernel: any valid map
    tsfa = ta;
    tsfb = ta;
  }
  cudaError_t ce =
      cudaLaunchKernelEx(&cfg, fp8_gemm_kernel<CG, F, NB>, ta, tb, tout, tsfa, tsfb, tout2, p);
  if (ce != cudaSuccess) {
    set_error(std::string("fp8_gemm: launch failed: ") + cudaGetErrorString(ce));
    return 4;
  }
  return 0;
}

}  // namespace gemm

bool make_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                     uint32_t box_inner, uint32_t box_outer, std::string *err) {
  return gemm::make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, inner, outer, inner,
                            box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_128B, err);
}

bool make_tmap_chunks_u8(CUtensorMap *map, const void *base, uint64_t K, uint64_t rows,
                         uint32_t box_rows, uint32_t box_chunks, std::string *err) {
  auto fn = gemm::encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is unavailable (driver entry point query failed)";
    return false;
  }
  cuuint64_t dims[3] = {128, rows, K / 128};
  cuuint64_t strides[2] = {K, 128};
  cuuint32_t box[3] = {128, box_rows, box_chunks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled (chunk view) failed with CUresult " +
           std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

// A tiled scale grid of `rows` rows as [row blocks][ncb tiles][128 words]; a box is
// `tiles_per_box` consecutive tiles of one row block.
bool make_tmap_sf(CUtensorMap *map, const void *base, uint64_t rows, uint64_t ncb,
                  uint32_t tiles_per_box, std::string *err) {
  return gemm::make_tmap_3d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, base, 128, ncb,
                            (rows + 127) / 128, 512, ncb * 512, 128, tiles_per_box, err);
}

// The same grid with a box of `box_words` 32-bit words of `tiles_per_box` consecutive tiles
// of one row block (box_words 64: one half of each tile, 32 rows' scale lines).
bool make_tmap_sf_box(CUtensorMap *map, const void *base, uint64_t rows, uint64_t ncb,
                      uint32_t box_words, uint32_t tiles_per_box, std::string *err) {
  return gemm::make_tmap_3d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, base, 128, ncb,
                            (rows + 127) / 128, 512, ncb * 512, box_words, tiles_per_box, err);
}

int launch_gemm(const GemmArgs &a, cudaStream_t stream, bool pdl) {
  if (a.M == 0 || a.N == 0) return 0;
  DeviceInfo dev;
  if (!current_device_info(&dev)) return 5;
  if (dev.cc_major != 10) {
    set_error("fp8_gemm needs an sm_100 (B200-class) device; current device is sm_" +
              std::to_string(dev.cc_major) + std::to_string(dev.cc_minor));
    return 5;
  }
  if (a.M > 0x7fffffffLL || a.N > 0x7fffffffLL || a.K > 0x7fffffffLL || a.ldo > 0x7fffffffLL ||
      a.n_peers < 0 || a.n_peers > kMaxPeers) {
    set_error("fp8_gemm: dimensions must fit in int32 and at most 7 peers");
    return 2;
  }
  // MXFP8 / NVFP4: the few-token kernel for M <= 128, and up to 256 where it gets a
  // K-split; CTA pairs otherwise.
  if (a.mx) {
    if (a.n_peers != 0) {
      set_error("block-scaled gemm: peer outputs are not supported");
      return 2;
    }
    if (a.M <= kFewTokenMaxM && !a.pairs_only) {
      const int rc = launch_gemm_small(a, stream, pdl);
      if (rc != kSmallDeclined) return rc;
    }
    if (a.nv) return gemm::launch_shape<2, gemm::kFmtNV>(a, dev, stream, pdl);
    return gemm::launch_shape<2, gemm::kFmtMX>(a, dev, stream, pdl);
  }
  // Few tokens: stream the weights with swap-AB split-K tiles (M <= 128; up to 256 where
  // the kernel gets a K-split). Otherwise CTA pairs with 256-row tiles (or single CTAs
  // with 128-row tiles for peer outputs at M <= 128).
  if (a.M <= kFewTokenMaxM && a.n_peers == 0 && !a.pairs_only) {
    const int rc = launch_gemm_small(a, stream, pdl);
    if (rc != kSmallDeclined) return rc;
  }
  if (a.M <= gemm::BM && !a.pairs_only)
    return gemm::launch_shape<1, gemm::kFmtE4M3>(a, dev, stream, pdl);
  const int tn = a.n_peers > 0 ? 256 : a.tile_n > 0 ? a.tile_n : pair_tile_n(a.M, a.N, dev.sm_count);
  if (tn == 192) return gemm::launch_shape<2, gemm::kFmtE4M3, 192>(a, dev, stream, pdl);
  return gemm::launch_shape<2, gemm::kFmtE4M3>(a, dev, stream, pdl);
}

int pair_tile_n(int64_t M, int64_t N, int sm_count) {
  // 192-column tiles when all of them fit in one wave of CTA pairs: more pairs busy, each
  // with a shorter tile (sweep_M1024 13.95 against 14.52 us). Past one wave the kernel is
  // bound by the total operand stream from L2, which narrower tiles enlarge (a 2304 x
  // 15360 -> 3072 linear: 88.3 against 87.5 us, though 256-column tiles leave its second
  // wave half empty).
  const int64_t pairs = std::max(1, sm_count / 2);
  const int64_t mt = (M + 2 * gemm::BM - 1) / (2 * gemm::BM);
  return mt * ((N + 191) / 192) <= pairs ? 192 : 256;
}

namespace {
__device__ unsigned int g_selftest_result;

// One thread waits on a barrier whose single expected arrival never comes, through the
// same bounded wait the GEMM uses; the run-out is recorded and the kernel returns.
__global__ void watchdog_selftest_kernel(uint64_t limit_ns) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ int abort_flag;
  const uint32_t b = ptx::smem_u32(&bar);
  ptx::mbar_init(b, 1);
  abort_flag = 0;
  ptx::fence_mbar_init();
  const bool done = ptx::mbar_wait_bounded(b, 0, &abort_flag, limit_ns);
  g_selftest_result = done ? 0u : 32u;
}
}  // namespace

cudaError_t launch_watchdog_selftest(unsigned int limit_us, unsigned int *status,
                                     cudaStream_t stream) {
  const unsigned int zero = 0xFFFFFFFFu;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_selftest_result, &zero, sizeof(zero), 0,
                                          cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  watchdog_selftest_kernel<<<1, 1, 0, stream>>>(static_cast<uint64_t>(limit_us) * 1000ull);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  e = cudaMemcpyFromSymbolAsync(status, g_selftest_result, sizeof(unsigned int), 0,
                                cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(stream);
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
