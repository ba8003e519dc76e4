/*
 * fp8linear_b200.h -- C ABI of the B200 (sm_100a) fused FP8 linear.
 *
 * Plain pointers and sizes only; no framework types cross this boundary. Every
 * device pointer is a CUDA device address on the calling thread's current device,
 * and every call is asynchronous on `stream` (a cudaStream_t passed as void*;
 * NULL means the legacy default stream). Apart from the peer-buffer set-up calls
 * (fp8lin_peer_buffer_*), no call synchronises the host or allocates device memory.
 *
 * Each entry point replaces one operator of drbh/fp8linear (paths relative to the
 * reference project root); the argument meaning and error conditions follow the
 * reference's host code, with the differences stated per function.
 *
 * Return value: FP8LIN_OK (0) or an fp8lin_status error; fp8lin_last_error()
 * gives this thread's message for the last failed call.
 */
#ifndef FP8LINEAR_B200_H
#define FP8LINEAR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FP8LIN_ABI_VERSION 1

#if defined(__GNUC__)
#define FP8LIN_API __attribute__((visibility("default")))
#else
#define FP8LIN_API
#endif

typedef enum fp8lin_status {
  FP8LIN_OK = 0,
  FP8LIN_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad dtype code */
  FP8LIN_ERR_UNSUPPORTED = 2,      /* shape/alignment outside what the kernels take */
  FP8LIN_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  FP8LIN_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed */
  FP8LIN_ERR_DEVICE = 5            /* no sm_100 device current */
} fp8lin_status;

/* Element types (codes shared by every dtype argument). */
typedef enum fp8lin_dtype {
  FP8LIN_DTYPE_BF16 = 0,
  FP8LIN_DTYPE_F16 = 1,
  FP8LIN_DTYPE_F32 = 2,
  FP8LIN_DTYPE_NONE = -1 /* "no tensor" (only valid for the optional bias) */
} fp8lin_dtype;

/* Library ABI version (FP8LIN_ABI_VERSION) and a human-readable build string. */
FP8LIN_API int fp8lin_abi_version(void);
FP8LIN_API const char *fp8lin_build_info(void);

/* Message for the last failed call on this thread ("" if none). */
FP8LIN_API const char *fp8lin_last_error(void);

/*
 * Per-token dynamic e4m3 quantization.
 * Replaces quantize_fp8 (csrc/quantize.cu:199-234; kernel csrc/quantize.cu:45-73).
 *   x       [M, K] row-major, x_dtype BF16 or F16
 *   xq      [M, K] row-major e4m3fn codes (1 byte each)
 *   x_scale [M] fp32, x_scale[m] = max(amax_m / 448, 1e-12)
 * xq[m,k] = e4m3_satfinite(clamp(x[m,k] * (1 / x_scale[m]), -448, 448)), bit-identical
 * to the reference kernel. M == 0 is a no-op. Any K >= 1 is accepted.
 */
FP8LIN_API int fp8lin_quantize_fp8(const void *x, int x_dtype, int64_t M, int64_t K,
                                   void *xq, float *x_scale, void *stream);

/*
 * Bytes of the MXFP8 block-scale grid for `rows` rows of K elements (K % 32 == 0):
 * ceil(rows / 128) * ceil((K / 32) / 4) * 512, the padded tile grid of
 * csrc/quantize.cu:244-250 (quantize_mxfp8's scales tensor size).
 */
FP8LIN_API size_t fp8lin_mx_scale_bytes(int64_t rows, int64_t K);

/*
 * MXFP8 block quantization (OCP microscaling: e4m3 codes, one power-of-two e8m0 scale per
 * 32 elements along K).
 * Replaces quantize_mxfp8 (csrc/quantize.cu:239-285; kernel csrc/quantize.cu:92-131);
 * applies to activations and, offline, to weights (quantize_weight_mxfp8).
 *   x      [M, K] row-major, x_dtype BF16 or F16, K % 32 == 0, 16-byte aligned
 *   xq     [M, K] e4m3fn codes, 8-byte aligned
 *   scales fp8lin_mx_scale_bytes(M, K) bytes, 4-byte aligned: the e8m0 scale of block
 *          (r, c) at (r/128)*ncb*512 + (c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4,
 *          ncb = ceil((K/32)/4) (csrc/quantize.cu:75-83); padding entries are written
 *          with 127 (scale 1.0), so the buffer needs no prefill.
 * Codes and scales are bit-identical to the reference kernel. M == 0 is a no-op.
 */
FP8LIN_API int fp8lin_quantize_mxfp8(const void *x, int x_dtype, int64_t M, int64_t K,
                                     void *xq, void *scales, void *stream);

/*
 * Per-output-channel e4m3 weight quantization (offline, once per weight).
 * Replaces the per-channel branch of quantize_weight (csrc/quantize.cu:341-366),
 * which the reference evaluates with ATen ops on the GPU:
 *   w_scale[n] = max(amax_n * (1/448), 1e-12)   (ATen's scalar divide is a
 *                                                reciprocal multiply on CUDA)
 *   wq[n,k]    = e4m3(clamp(w[n,k] / w_scale[n], -448, 448))  (true divide)
 *   w       [N, K] row-major, w_dtype BF16, F16 or F32
 *   wq      [N, K] e4m3fn codes; w_scale [N] fp32. NaN propagates as in ATen.
 * The reference's opt-in MXFP8/NVFP4 diversions (FP8LINEAR_USE_MX /
 * FP8LINEAR_USE_NVFP4, csrc/quantize.cu:344-357) are applied by the torch op
 * quantize_weight, which calls fp8lin_quantize_mxfp8 / fp8lin_quantize_nvfp4 instead;
 * this entry point is the per-channel quantizer only.
 */
FP8LIN_API int fp8lin_quantize_weight(const void *w, int w_dtype, int64_t N, int64_t K,
                                      void *wq, float *w_scale, void *stream);

/*
 * FP8 GEMM with the dequant + bias epilogue fused in.
 * Replaces fp8_gemm (csrc/fp8_gemm.cu:139-194): the cuBLASLt e4m3 matmul into an
 * fp32 [M,N] buffer (csrc/fp8_gemm.cu:180-184) followed by dequant_bias_kernel
 * (csrc/fp8_gemm.cu:65-80), here one tcgen05 kernel with no fp32 intermediate:
 *   out[m,n] = (sum_k xq[m,k]*wq[n,k]) * x_scale[m] * w_scale[n] + bias[n]
 *   xq [M,K] e4m3 row-major; wq [N,K] e4m3 row-major (K-major, i.e. nn.Linear layout)
 *   x_scale [M] fp32; w_scale [N] fp32
 *   bias [N] of bias_dtype (BF16/F16/F32) or NULL with FP8LIN_DTYPE_NONE
 *   out [M,N] row-major, out_dtype BF16 or F16 (the reference always writes fp16)
 * Requirements (checked): K % 16 == 0 and K > 0 (as csrc/fp8_gemm.cu:154), xq/wq
 * 16-byte aligned. Any N: output rows that are a multiple of 16 bytes (N % 8 == 0, out
 * 16-byte aligned) are written with TMA stores, others with plain stores.
 * M == 0 or N == 0 is a no-op.
 */
FP8LIN_API int fp8lin_fp8_gemm(const void *xq, const float *x_scale, const void *wq,
                               const float *w_scale, const void *bias, int bias_dtype,
                               void *out, int out_dtype, int64_t M, int64_t N, int64_t K,
                               void *stream);

/*
 * MXFP8 GEMM with block scales applied inside the tensor-core MMA and the bias fused.
 * Replaces mxfp8_gemm (csrc/fp8_gemm.cu:233-340: cuBLASLt VEC32_UE8M0 block-scaled matmul,
 * bias epilogue, fp16 out), here one tcgen05 kind::mxf8f6f4.block_scale kernel:
 *   out[m,n] = sum_k xq[m,k] 2^(xs[m,k/32]-127) * wq[n,k] 2^(ws[n,k/32]-127) + bias[n]
 *   xq [M,K], wq [N,K] e4m3 row-major, 16-byte aligned; K % 32 == 0
 *   x_scales / w_scales: the tiled e8m0 grids of fp8lin_quantize_mxfp8 for M / N rows
 *   (fp8lin_mx_scale_bytes bytes), 16-byte aligned
 *   bias [N] BF16/F16/F32 or NULL; out [M,N] BF16 or F16 (the reference writes fp16)
 * M == 0 or N == 0 is a no-op.
 */
FP8LIN_API int fp8lin_mxfp8_gemm(const void *xq, const void *x_scales, const void *wq,
                                 const void *w_scales, const void *bias, int bias_dtype,
                                 void *out, int out_dtype, int64_t M, int64_t N, int64_t K,
                                 void *stream);

/* Workspace fp8lin_mxfp8_linear needs: the codes (M*K) and the scale grid, each rounded
 * up to 256 bytes. */
FP8LIN_API size_t fp8lin_mxfp8_linear_workspace_size(int64_t M, int64_t K);

/*
 * Fused MXFP8 linear: fp8lin_quantize_mxfp8 of x into the workspace, then the block-scaled
 * GEMM launched as its programmatic dependent. Replaces mxfp8_linear
 * (csrc/fp8_gemm.cu:335-345) and the MXFP8 branch of fp8_linear (csrc/fp8_gemm.cu:206-213).
 * wq / w_scales from fp8lin_quantize_mxfp8 of the weight (quantize_weight_mxfp8).
 */
FP8LIN_API int fp8lin_mxfp8_linear(const void *x, int x_dtype, const void *wq,
                                   const void *w_scales, const void *bias, int bias_dtype,
                                   void *out, int out_dtype, int64_t M, int64_t N, int64_t K,
                                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * Bytes of the NVFP4 block-scale grid for `rows` rows of K elements (K % 32 == 0):
 * ceil(rows / 128) * ceil((K / 16) / 4) * 512 (csrc/quantize.cu:301-309, quantize_nvfp4's
 * scales tensor size).
 */
FP8LIN_API size_t fp8lin_nv_scale_bytes(int64_t rows, int64_t K);

/*
 * NVFP4 block quantization: e2m1 codes packed two per byte, one ue4m3 scale per 16
 * elements along K. Replaces quantize_nvfp4 (csrc/quantize.cu:290-334; kernel
 * csrc/quantize.cu:157-194); applies to activations and, offline, to weights
 * (quantize_weight_nvfp4).
 *   x      [M, K] row-major, x_dtype BF16 or F16, K % 32 == 0, 16-byte aligned
 *   xq     [M, K/2] bytes, 4-byte aligned: element 2j in the low nibble of byte j
 *   scales fp8lin_nv_scale_bytes(M, K) bytes, 4-byte aligned, in the tiled layout of
 *          fp8lin_quantize_mxfp8 with ncb = ceil((K/16)/4); padding entries are written
 *          with 0x38 (e4m3 1.0), so the buffer needs no prefill.
 * Per block: s = e4m3_satfinite(min(amax * fl(1/6), 448)); codes = e2m1 of
 * clamp(x * (1 / s), -6, 6) by the round-to-nearest thresholds (ties up), 1/s = 0 when
 * s = 0. Codes and scales are bit-identical to the reference kernel. M == 0 is a no-op.
 */
FP8LIN_API int fp8lin_quantize_nvfp4(const void *x, int x_dtype, int64_t M, int64_t K,
                                     void *xq, void *scales, void *stream);

/*
 * NVFP4 GEMM with block scales applied inside the tensor-core MMA and the bias fused.
 * Replaces nvfp4_gemm (csrc/fp8_gemm.cu:352-445: cuBLASLt VEC16_UE4M3 block-scaled e2m1
 * matmul, bias epilogue, fp16 out), here one tcgen05 kind::mxf4nvf4.block_scale kernel:
 *   out[m,n] = sum_k e2m1(xq[m,k]) xs[m,k/16] * e2m1(wq[n,k]) ws[n,k/16] + bias[n]
 *   xq [M, K/2], wq [N, K/2] packed e2m1 (fp8lin_quantize_nvfp4), 16-byte aligned;
 *   K (elements) % 32 == 0
 *   x_scales / w_scales: the tiled ue4m3 grids for M / N rows (fp8lin_nv_scale_bytes
 *   bytes), 16-byte aligned
 *   bias [N] BF16/F16/F32 or NULL; out [M,N] BF16 or F16 (the reference writes fp16)
 * M == 0 or N == 0 is a no-op.
 */
FP8LIN_API int fp8lin_nvfp4_gemm(const void *xq, const void *x_scales, const void *wq,
                                 const void *w_scales, const void *bias, int bias_dtype,
                                 void *out, int out_dtype, int64_t M, int64_t N, int64_t K,
                                 void *stream);

/* Workspace fp8lin_nvfp4_linear needs: the packed codes (M*K/2) and the scale grid, each
 * rounded up to 256 bytes. */
FP8LIN_API size_t fp8lin_nvfp4_linear_workspace_size(int64_t M, int64_t K);

/*
 * Fused NVFP4 linear: fp8lin_quantize_nvfp4 of x into the workspace, then the block-scaled
 * GEMM launched as its programmatic dependent. Replaces nvfp4_linear
 * (csrc/fp8_gemm.cu:447-457) and the NVFP4 branch of fp8_linear (csrc/fp8_gemm.cu:206-209).
 * wq / w_scales from fp8lin_quantize_nvfp4 of the weight (quantize_weight_nvfp4).
 */
FP8LIN_API int fp8lin_nvfp4_linear(const void *x, int x_dtype, const void *wq,
                                   const void *w_scales, const void *bias, int bias_dtype,
                                   void *out, int out_dtype, int64_t M, int64_t N, int64_t K,
                                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * The per-token quantizer fused into the op that precedes the linear in a FLUX / DiT
 * block (AdaLayerNormZero modulation): for each row m of x (batch b = m / (M / batches))
 *   y = LayerNorm(x[m]) * (1 + scale[b]) + shift[b]     (LayerNorm without affine, eps)
 * rounded to x's type after each of the four steps as the unfused bf16/fp16 torch ops
 * round it, then quantized exactly as fp8lin_quantize_fp8 quantizes y. y never goes to
 * memory. No reference counterpart: it replaces, at the reference's call site
 * (torch-ext/fp8linear/layers.py:165-167, the input of Fp8Linear.forward), the chain
 * LayerNorm -> modulation -> quantize_fp8 (csrc/quantize.cu:199-234).
 *   x      [M, K] x_dtype BF16 or F16, 16-byte aligned; K % 8 == 0, 8 <= K <= 8192
 *   shift, scale [batches, K] of x_dtype, 16-byte aligned; batches divides M
 *   xq [M, K] e4m3 codes; x_scale [M] fp32
 * mean and variance are fp32 sums in a fixed order and rstd = 1 / sqrt(var + eps) with
 * IEEE operations, so results are reproducible bit for bit (the CPU oracle restates the
 * order). M == 0 is a no-op.
 */
FP8LIN_API int fp8lin_layernorm_modulate_quantize_fp8(const void *x, int x_dtype, int64_t M,
                                                      int64_t K, int64_t batches,
                                                      const void *shift, const void *scale,
                                                      float eps, void *xq, float *x_scale,
                                                      void *stream);

/*
 * fp8lin_layernorm_modulate_quantize_fp8 into the workspace (fp8lin_linear_workspace_size),
 * then the FP8 GEMM with the fused dequant + bias epilogue launched as its programmatic
 * dependent: out [M, N] = fp8_linear(y, wq, w_scale, bias) without y in memory. Arguments
 * as fp8lin_layernorm_modulate_quantize_fp8 and fp8lin_fp8_linear.
 */
FP8LIN_API int fp8lin_fp8_linear_modulated(const void *x, int x_dtype, int64_t M, int64_t K,
                                           int64_t batches, const void *shift,
                                           const void *scale, float eps, const void *wq,
                                           const float *w_scale, const void *bias,
                                           int bias_dtype, void *out, int out_dtype,
                                           int64_t N, void *workspace, size_t workspace_bytes,
                                           void *stream);

/*
 * fp8lin_fp8_linear with x and out in host memory (page-locked for the copies to be
 * asynchronous): the path of a host that keeps activations in its own memory. Rows go in
 * chunks of up to 512; the upload of chunk i+1, the quantizer + GEMM of chunk i and the
 * download of chunk i-1 run on three streams of the library's own, so PCIe carries both
 * directions at once and the kernels hide behind the copies. The work is ordered after
 * what is already queued on `stream`, and `stream` waits for its end: synchronize
 * `stream` before reading out. Calls on one device from several host threads are
 * queued one after another. wq, w_scale and bias are device pointers as in
 * fp8lin_fp8_linear. Replaces the host-side copies around the reference's fp8_linear
 * (csrc/fp8_gemm.cu:196-221), which takes device tensors only.
 */
FP8LIN_API size_t fp8lin_fp8_linear_host_workspace_size(int64_t M, int64_t N, int64_t K);
FP8LIN_API int fp8lin_fp8_linear_host(const void *x_host, int x_dtype, const void *wq,
                                      const float *w_scale, const void *bias, int bias_dtype,
                                      void *out_host, int out_dtype, int64_t M, int64_t N,
                                      int64_t K, void *workspace, size_t workspace_bytes,
                                      void *stream);

/*
 * Device workspace fp8lin_fp8_linear needs for M tokens of width K: the e4m3 codes
 * and the per-token scales of x (aligned sub-buffers).
 */
FP8LIN_API size_t fp8lin_linear_workspace_size(int64_t M, int64_t K);

/*
 * Fused dynamic-quant FP8 linear: fp8lin_quantize_fp8 then fp8lin_fp8_gemm, the
 * GEMM launched as a programmatic dependent of the quantizer so its prologue
 * overlaps the quantizer's tail.
 * Replaces fp8_linear's per-channel branch (csrc/fp8_gemm.cu:196-221). The caller
 * flattens x's leading dimensions into M (the reference's x.reshape(-1, K)).
 *   x [M,K] (BF16/F16); wq/w_scale/bias as in fp8lin_fp8_gemm; out [M,N] out_dtype
 *   workspace: >= fp8lin_linear_workspace_size(M, K) bytes of device memory,
 *   256-byte aligned, owned by the caller and reusable after the call's stream
 *   work completes.
 */
FP8LIN_API int fp8lin_fp8_linear(const void *x, int x_dtype, const void *wq,
                                 const float *w_scale, const void *bias, int bias_dtype,
                                 void *out, int out_dtype, int64_t M, int64_t N, int64_t K,
                                 void *workspace, size_t workspace_bytes, void *stream);

/*
 * Column-parallel FP8 linear with the output all-gather fused into the GEMM epilogue
 * (the N-shard of the multi-GPU split; no reference counterpart, the reference has no
 * multi-GPU code). This rank holds N output channels (wq/w_scale/bias rows) of a wider
 * [M, ldo] output; each output box the epilogue produces is written to outs[0] (this
 * GPU, TMA store) and to outs[1..n_outs-1] (other GPUs' buffers mapped into this process,
 * e.g. with fp8lin_peer_buffer_open, written with 16-byte P2P stores), so the gather
 * overlaps the math and no separate collective or interleave copy runs.
 *   outs[i]: pointer to this rank's first output column in buffer i; rows of ldo
 *            elements; all buffers 16-byte aligned; N and ldo multiples of 8
 *   n_outs:  1..8 (1 = this GPU only)
 * Other arguments as fp8lin_fp8_linear. The caller orders the peers' reads after every
 * rank's call completes (e.g. a one-element all-reduce on the stream after the call),
 * and orders each call's writes after the peers' last reads of the buffer it writes
 * (e.g. two buffers used in turn, so the all-reduce of the call in between covers it).
 */
FP8LIN_API int fp8lin_fp8_linear_allgather(const void *x, int x_dtype, const void *wq,
                                           const float *w_scale, const void *bias,
                                           int bias_dtype, void *const *outs, int n_outs,
                                           int out_dtype, int64_t M, int64_t N, int64_t K,
                                           int64_t ldo, void *workspace,
                                           size_t workspace_bytes, void *stream);

/*
 * Peer buffers for fp8lin_fp8_linear_allgather when every GPU is driven by its own
 * process (one process per GPU). No counterpart in the reference (it has no multi-GPU
 * code). Plain CUDA peer memory over NVLink: the buffers are ordinary device
 * allocations mapped into the other processes with CUDA IPC handles; no NVLink
 * multicast object is created or bound.
 *   fp8lin_peer_buffer_alloc: allocates `bytes` on the current device (256-byte
 *     aligned) into *ptr and writes its FP8LIN_PEER_HANDLE_BYTES-byte handle to
 *     handle_out, for the other processes of the node.
 *   fp8lin_peer_buffer_open: maps another process's buffer from its handle into this
 *     process (current device) and returns the address this process's kernels use for
 *     it. A process cannot open its own handle.
 *   fp8lin_peer_buffer_close: unmaps a buffer opened here.
 *   fp8lin_peer_buffer_free: frees a buffer allocated here; call it only after every
 *     process that opened it has closed it.
 * These are set-up calls: they allocate, map or free device memory and may synchronise
 * the device. Not for use during stream capture.
 */
#define FP8LIN_PEER_HANDLE_BYTES 64
FP8LIN_API int fp8lin_peer_buffer_alloc(size_t bytes, void **ptr, unsigned char *handle_out);
FP8LIN_API int fp8lin_peer_buffer_open(const unsigned char *handle, void **ptr);
FP8LIN_API int fp8lin_peer_buffer_close(void *ptr);
FP8LIN_API int fp8lin_peer_buffer_free(void *ptr);

/*
 * Size of the device scratch array fp8lin_fp8_linear_noalloc works in (64 MiB).
 * Every GPU that loads the library holds this array until the process exits.
 */
#define FP8LIN_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)

/*
 * fp8lin_fp8_linear for callers that cannot allocate device memory: no workspace
 * argument; the activations' e4m3 codes and scales go to a fixed array of
 * FP8LIN_NOALLOC_SCRATCH_BYTES inside the library instead. Meant for hosts that give
 * an op only its input and output buffers (plugin/custom-op interfaces whose device
 * memory is owned by the host's pool) or cannot afford cudaMalloc's implicit
 * synchronisation. No counterpart in the reference.
 *   Arguments, results and errors as fp8lin_fp8_linear, plus FP8LIN_ERR_WORKSPACE when
 *   fp8lin_linear_workspace_size(M, K) > FP8LIN_NOALLOC_SCRATCH_BYTES.
 *   All calls on a device share the one array: calls whose GPU work overlaps race on
 *   it and must be serialised by the caller. It keeps the last call's contents;
 *   nothing in it needs to start at zero.
 *   The first call on each device looks up the array's device address
 *   (cudaGetSymbolAddress, with that device current); make it before any stream
 *   capture. No call allocates or frees device memory.
 */
FP8LIN_API int fp8lin_fp8_linear_noalloc(const void *x, int x_dtype, const void *wq,
                                         const float *w_scale, const void *bias,
                                         int bias_dtype, void *out, int out_dtype, int64_t M,
                                         int64_t N, int64_t K, void *stream);

/*
 * Watchdog status of the kernels on the current device: every wait in them is
 * bounded; a wait that runs out sets a bit here and the kernel returns early instead
 * of hanging (GEMM: 1 = TMA producer, 2 = MMA issuer, 4 = epilogue; 8 = quantizer;
 * 16 = few-token GEMM).
 * *status receives the bits; clear != 0 resets them. Synchronous on the device.
 * No counterpart in the reference (cuBLASLt has no such report).
 */
FP8LIN_API int fp8lin_device_status(unsigned int *status, int clear);

/*
 * Exercises the watchdog on the GPU without a fault: one thread waits, through the same
 * bounded wait every kernel here uses, on an mbarrier that nothing arrives on, for
 * limit_us microseconds (1..1000000); the wait runs out, the kernel records it and
 * returns, and *status receives 32. Synchronous on `stream`. No reference counterpart.
 */
FP8LIN_API int fp8lin_selftest_watchdog(unsigned int limit_us, unsigned int *status,
                                        void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FP8LINEAR_B200_H */
