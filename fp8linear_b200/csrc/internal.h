// internal.h -- declarations shared by the kernels' translation units and the C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

namespace fp8lin {

enum DType : int { kBF16 = 0, kF16 = 1, kF32 = 2, kNone = -1 };

constexpr float kE4M3Max = 448.0f;
constexpr float kScaleFloor = 1e-12f;

// Thread-local last-error message used by the C ABI.
void set_error(const std::string &msg);
void clear_error();

// Per-device facts the launchers need (cached after the first query).
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
};
// Fills `info` for the calling thread's current device; false + error message on failure.
bool current_device_info(DeviceInfo *info);

// ---- quantize.cu
// A device range to bring into L2 (16-byte aligned start, size a multiple of 16).
struct L2Prefetch {
  const void *ptr = nullptr;
  int64_t bytes = 0;
};
// Per-token quantization (activation path). Returns cudaSuccess or the launch error.
// `prefetch`: the range the kernel launched next reads (a fused linear's weights), which
// the quantizer's CTAs bring into L2 before their dependency wait, i.e. while the kernel
// before still runs (the pipelined form only; the grid widens so each CTA takes ~64 KB).
cudaError_t launch_quantize_rows(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                                 float *scale, cudaStream_t stream, bool trigger_dependents,
                                 const L2Prefetch &prefetch = {});
// MXFP8 block quantization (per 32 elements along K, e8m0 scales in the tiled
// block-scale layout; the whole padded scale grid of mx_scale_bytes(M, K) is written).
// K % 32 == 0, x 16-byte aligned, xq 8-byte aligned, scales 4-byte aligned.
cudaError_t launch_quantize_mx(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                               uint8_t *scales, cudaStream_t stream, bool trigger_dependents);
inline int64_t mx_scale_bytes(int64_t rows, int64_t K) {
  return (rows + 127) / 128 * ((K / 32 + 3) / 4) * 512;
}
// NVFP4 block quantization (per 16 elements: e4m3 scale, e2m1 codes packed two per byte
// into xq [M, K/2]); scale grid of nv_scale_bytes(M, K) written whole. K % 32 == 0, x
// 16-byte aligned, xq and scales 4-byte aligned.
cudaError_t launch_quantize_nv(const void *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                               uint8_t *scales, cudaStream_t stream, bool trigger_dependents);
inline int64_t nv_scale_bytes(int64_t rows, int64_t K) {
  return (rows + 127) / 128 * ((K / 16 + 3) / 4) * 512;
}
// LayerNorm (no affine) + modulation y = LN(x) * (1 + scale[b]) + shift[b], then the
// per-token e4m3 quantizer on y; rows m of batch b = m / (M / batches); shift and scale
// [batches, K] of x's dtype, 16-byte aligned rows. K % 8 == 0, K <= kLnMaxK.
constexpr int64_t kLnMaxK = 8192;
cudaError_t launch_ln_modulate_quantize(const void *x, int dtype, int64_t M, int64_t K,
                                        int64_t batches, const void *shift, const void *scale,
                                        float eps, uint8_t *xq, float *x_scale,
                                        cudaStream_t stream, bool trigger_dependents);
// Reads (and optionally clears) the quantizer watchdog bits (8) of the current device.
cudaError_t read_quant_status(unsigned int *bits, bool clear);
// Per-channel weight quantization (ATen semantics of the reference's quantize_weight).
cudaError_t launch_quantize_weight(const void *w, int dtype, int64_t N, int64_t K, uint8_t *wq,
                                   float *scale, cudaStream_t stream);

// ---- gemm_sm100.cu
struct GemmArgs {
  const uint8_t *xq;
  const float *xs;
  const uint8_t *wq;
  const float *ws;
  const void *bias;
  int bias_dtype;
  void *out;
  int out_dtype;
  int64_t M, N, K;
  // Output row pitch in elements (0: N). With ldo > N the output is a column block of
  // a wider matrix, `out` pointing at the block's first column.
  int64_t ldo = 0;
  // Copies of the output block written to other GPUs' buffers (peer-mapped pointers,
  // same layout as `out`), straight from the epilogue.
  int n_peers = 0;
  void *const *peers = nullptr;
  // Block-scaled forms: xs/ws unused; xsf/wsf are the tiled scale grids of xq and wq,
  // 16-byte aligned. mx alone: MXFP8 (e8m0 grids of mx_scale_bytes(M or N, K)); mx and nv:
  // NVFP4 (xq [M, K/2] / wq [N, K/2] packed e2m1, ue4m3 grids of nv_scale_bytes).
  bool mx = false;
  bool nv = false;
  const uint8_t *xsf = nullptr;
  const uint8_t *wsf = nullptr;
  // Skip the few-token kernel and run CTA pairs at any M (same per-element summation
  // order as every larger M): the row chunks of one host-buffer call.
  bool pairs_only = false;
  // The weights (and their scales) may be read before the programmatic dependency wait.
  // Set only when the kernel launched just before on the stream is this library's
  // quantizer of the same call: it lets its dependents launch only after its own wait
  // has returned, so every kernel before it (a weight writer included) has completed.
  bool weights_before_wait = false;
  // Per-token e4m3 CTA-pair tiles: output columns per tile (256 or 192; 0: pair_tile_n of
  // this call's M and N). A call split into row chunks passes the whole call's choice.
  int tile_n = 0;
};
constexpr int kMaxPeers = 7;
// Token counts up to which the GEMM may run a few-token kernel (it streams the weights once).
constexpr int64_t kFewTokenMaxM = 256;
// Launches the tcgen05 GEMM + fused epilogue. `pdl` launches it as a programmatic
// dependent of the previous kernel on the stream: its set-up overlaps that kernel's tail
// and it waits for it (griddepcontrol.wait) before reading activations or scales and
// before writing anything. Returns an fp8lin_status code and sets the error message on
// failure.
int launch_gemm(const GemmArgs &a, cudaStream_t stream, bool pdl);
// Tile width (256 or 192 columns) of the per-token e4m3 CTA-pair kernel for an [M, N] output.
int pair_tile_n(int64_t M, int64_t N, int sm_count);
// Reads (and optionally clears) the GEMM watchdog bits of the current device.
cudaError_t read_gemm_status(unsigned int *bits, bool clear);

// Launches one thread that waits, bounded by `limit_us`, on an mbarrier nothing arrives
// on (the watchdog path every kernel's waits share) and copies the outcome to the host:
// *status = 32 when the wait ran out and the kernel returned. Synchronous.
cudaError_t launch_watchdog_selftest(unsigned int limit_us, unsigned int *status,
                                     cudaStream_t stream);

// ---- gemm_small_sm100.cu (M <= 256: swap-AB, split-K over a cluster)
// Returns an fp8lin_status code, or kSmallDeclined without launching when M > 128 and
// the (weight tile, token block) clusters would get no K-split (split 1: every CTA
// streams all of K alone, slower than the CTA-pair kernel); the caller then launches that.
constexpr int kSmallDeclined = -1;
int launch_gemm_small(const GemmArgs &a, cudaStream_t stream, bool pdl);
cudaError_t read_small_status(unsigned int *bits, bool clear);
// 2-D uint8 tensor map with 128-byte swizzle (shared by both GEMM shapes).
bool make_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                     uint32_t box_inner, uint32_t box_outer, std::string *err);
// A row-major uint8 [rows, K] matrix (K % 128 == 0) viewed as (128 bytes, row, 128-byte
// chunk): a box of `box_rows` rows x `box_chunks` chunks lands as [chunk][row][128 B], each
// chunk's rows 128-byte swizzled, i.e. the same shared-memory image as that many 2-D boxes
// of 128 bytes x `box_rows` rows, in one copy. Every coordinate inside its extent addresses
// inside the matrix.
bool make_tmap_chunks_u8(CUtensorMap *map, const void *base, uint64_t K, uint64_t rows,
                         uint32_t box_rows, uint32_t box_chunks, std::string *err);

}  // namespace fp8lin
