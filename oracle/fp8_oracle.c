/*
 * fp8_oracle.c -- CPU restatement of drbh/fp8linear's per-channel FP8 linear path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle that the CUDA kernels of
 * fp8linear_b200 are compared against; it is never linked into, called by or
 * shipped with the product. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it (through oracle/oracle.py).
 *
 * Each function restates one piece of the reference (paths relative to the
 * reference project root):
 *   oracle_e4m3_encode      __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)
 *                           (csrc/quantize.cu:71) and c10::Float8_e4m3fn's
 *                           non-saturating cast (csrc/quantize.cu:364)
 *   oracle_quantize_rows    quant_rowwise_kernel + block_reduce_max
 *                           (csrc/quantize.cu:28-73), launched by quantize_fp8
 *                           (csrc/quantize.cu:199-234)
 *   oracle_quantize_weight  per-channel branch of quantize_weight
 *                           (csrc/quantize.cu:359-365), as ATen evaluates it on CUDA
 *   oracle_gemm_dequant     cuBLASLt unscaled e4m3 matmul (csrc/fp8_gemm.cu:109-131,
 *                           180-184) followed by dequant_bias_kernel
 *                           (csrc/fp8_gemm.cu:65-80)
 *   oracle_mx_sf_offset     the tiled block-scale layout sf_offset (csrc/quantize.cu:75-83)
 *   oracle_quantize_mxfp8   quant_mxfp8_kernel (csrc/quantize.cu:92-131), launched by
 *                           quantize_mxfp8 (csrc/quantize.cu:239-285)
 *   oracle_quantize_nvfp4   quant_nvfp4_kernel + f2e2m1 (csrc/quantize.cu:136-194),
 *                           launched by quantize_nvfp4 (csrc/quantize.cu:290-334)
 *   oracle_nvfp4_gemm       the block-scaled e2m1 product nvfp4_gemm asks cuBLASLt for
 *                           (VEC16_UE4M3, bias epilogue, fp16 out; csrc/fp8_gemm.cu:347-446)
 *   oracle_mxfp8_gemm       cuBLASLt VEC32_UE8M0 block-scaled e4m3 matmul with the bias
 *                           epilogue, fp16 out (csrc/fp8_gemm.cu:233-333)
 *   oracle_ln_modulate_quantize
 *                           no reference function: the chain LayerNorm -> AdaLN modulation
 *                           -> quantize_fp8 that feeds Fp8Linear.forward in a FLUX block
 *                           (torch-ext/fp8linear/layers.py:165-167), in the fixed reduction
 *                           order of the fused kernel, then oracle_quantize_rows' rule
 *
 * Arithmetic is IEEE binary32 with round-to-nearest-even and no flush-to-zero,
 * which is what nvcc emits for the reference without --use_fast_math.
 * Build: cc -O2 -fPIC -shared -ffp-contract=off -fno-fast-math fp8_oracle.c -o liboracle.so
 * (-ffp-contract=off keeps x*inv and (acc*xs)*ws as separate roundings.)
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define E4M3_MAX 448.0f

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* bf16 / fp16 storage -> fp32 (exact). */
float oracle_bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }

float oracle_f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1f;
  uint32_t m = h & 0x3ffu;
  if (e == 0) {
    /* zero or subnormal: m * 2^-24 is exact in fp32 */
    float v = (float)m * u2f(0x33800000u); /* 2^-24 */
    return s ? -v : v;
  }
  if (e == 31) return u2f(s | 0x7f800000u | (m << 13));
  return u2f(s | ((e + 112u) << 23) | (m << 13));
}

/* fp32 -> fp16 storage, round-to-nearest-even (IEEE __float2half_rn). */
uint16_t oracle_f32_to_f16(float f) {
  uint32_t u = f2u(f);
  uint16_t s = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7fffffffu;
  if (a >= 0x7f800000u) return (uint16_t)(s | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0));
  float af = u2f(a);
  if (af >= 65520.0f) return (uint16_t)(s | 0x7c00u); /* rounds to inf */
  if (af < 6.103515625e-05f) {                         /* below 2^-14: subnormal */
    float q = rintf(af * 16777216.0f);                   /* units of 2^-24, RNE */
    return (uint16_t)(s | (uint16_t)q);                  /* q==1024 -> smallest normal */
  }
  uint32_t e = (a >> 23) - 112u;
  uint32_t m = a & 0x7fffffu;
  uint32_t keep = m >> 13, rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (keep & 1u))) keep++;
  if (keep == 0x400u) { keep = 0; e++; }
  return (uint16_t)(s | (e << 10) | keep);
}

/* fp32 -> bf16 storage, round-to-nearest-even (__float2bfloat16_rn); NaN stays NaN. */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

/*
 * fp32 -> e4m3fn byte, round-to-nearest-even.
 * saturate != 0: finite magnitudes above 448 clamp to 448 and NaN gives 0x7F
 *                (the __NV_SATFINITE hardware convert).
 * saturate == 0: magnitudes that round above 448 (>= 464) and NaN give NaN with
 *                the input's sign (c10::Float8_e4m3fn's software cast).
 */
uint8_t oracle_e4m3_encode(float v, int saturate) {
  uint32_t u = f2u(v);
  uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return saturate ? 0x7f : (uint8_t)(sign | 0x7f);
  float af = u2f(a);
  if (af >= 464.0f) { /* includes +inf */
    if (saturate) return (uint8_t)(sign | 0x7e);
    return (uint8_t)(sign | 0x7f);
  }
  if (af > E4M3_MAX) /* (448, 464): rounds to 448 under RNE (480 is not a finite code) */
    return (uint8_t)(sign | 0x7e);
  if (af < 0.015625f) { /* below 2^-6: subnormal grid of 2^-9 */
    float q = rintf(af * 512.0f); /* exact scale, RNE to integer 0..8 */
    return (uint8_t)(sign | (uint8_t)q); /* q == 8 encodes 2^-6 (exp 1, mant 0) */
  }
  int e = (int)(a >> 23) - 127; /* -6 .. 8 */
  uint32_t m = a & 0x7fffffu;
  uint32_t keep = m >> 20, rem = m & 0xfffffu;
  if (rem > 0x80000u || (rem == 0x80000u && (keep & 1u))) keep++;
  if (keep == 8u) { keep = 0; e++; }
  return (uint8_t)(sign | (uint8_t)((e + 7) << 3) | (uint8_t)keep);
}

float oracle_e4m3_decode(uint8_t b) {
  uint32_t s = b & 0x80u;
  uint32_t e = (b >> 3) & 0xfu;
  uint32_t m = b & 7u;
  float v;
  if (e == 15 && m == 7) return u2f(0x7fc00000u | (s << 24));
  if (e == 0) v = (float)m * 0.001953125f; /* m * 2^-9 */
  else v = u2f(((e + 120u) << 23) | (m << 20));
  return s ? -v : v;
}

/*
 * Per-token quantization, csrc/quantize.cu:45-73.
 *   amax = fmaxf-reduce |x| (NaN inputs are ignored by fmaxf; quantize.cu:52-55)
 *   sc   = fmaxf(amax / 448, 1e-12)  (IEEE divide; quantize.cu:60)
 *   inv  = 1 / sc                    (quantize.cu:62)
 *   q    = e4m3_satfinite(fminf(fmaxf(x * inv, -448), 448))  (quantize.cu:69-71)
 * dtype 0 = bf16 input, 1 = fp16 input.
 */
void oracle_quantize_rows(const uint16_t *x, int dtype, int64_t M, int64_t K,
                          uint8_t *xq, float *scale) {
  for (int64_t r = 0; r < M; ++r) {
    const uint16_t *row = x + r * K;
    float amax = 0.0f;
    for (int64_t j = 0; j < K; ++j) {
      float v = dtype ? oracle_f16_to_f32(row[j]) : oracle_bf16_to_f32(row[j]);
      amax = fmaxf(amax, fabsf(v));
    }
    volatile float sc = fmaxf(amax / E4M3_MAX, 1e-12f);
    volatile float inv = 1.0f / sc;
    scale[r] = sc;
    for (int64_t j = 0; j < K; ++j) {
      float v = dtype ? oracle_f16_to_f32(row[j]) : oracle_bf16_to_f32(row[j]);
      volatile float p = v * inv;
      float c = fminf(fmaxf(p, -E4M3_MAX), E4M3_MAX);
      xq[r * K + j] = oracle_e4m3_encode(c, 1);
    }
  }
}

/*
 * Per-channel weight quantization, csrc/quantize.cu:360-364, as ATen runs it on CUDA:
 *   amax  = |w|.amax(1).float()        (NaN propagates through amax)
 *   scale = (amax / 448).clamp_min(1e-12)
 *           ATen's CUDA true-divide by a host scalar multiplies by the fp32
 *           reciprocal: amax * (1.0f / 448.0f). recip_scalar != 0 selects that;
 *           0 selects a true division (ATen's CPU kernel).
 *   wq    = (w.float() / scale[:,None]).clamp(-448, 448).to(float8_e4m3fn)
 *           (true division; clamp and the cast propagate NaN; the cast does not
 *           saturate).
 * dtype 0 = bf16 input, 1 = fp16 input, 2 = fp32 input.
 */
void oracle_quantize_weight(const void *w, int dtype, int64_t N, int64_t K,
                            int recip_scalar, uint8_t *wq, float *scale) {
  const uint16_t *w16 = (const uint16_t *)w;
  const float *w32 = (const float *)w;
  const float inv448 = 1.0f / E4M3_MAX;
  for (int64_t r = 0; r < N; ++r) {
    float amax = 0.0f;
    int has_nan = 0;
    for (int64_t j = 0; j < K; ++j) {
      float v = dtype == 2 ? w32[r * K + j]
                : dtype == 1 ? oracle_f16_to_f32(w16[r * K + j])
                             : oracle_bf16_to_f32(w16[r * K + j]);
      float a = fabsf(v);
      if (a != a) has_nan = 1;
      else if (a > amax) amax = a;
    }
    volatile float s;
    if (has_nan) s = u2f(0x7fffffffu);
    else if (recip_scalar) s = amax * inv448;
    else s = amax / E4M3_MAX;
    float sc = (s != s) ? s : (s < 1e-12f ? 1e-12f : s);
    scale[r] = sc;
    for (int64_t j = 0; j < K; ++j) {
      float v = dtype == 2 ? w32[r * K + j]
                : dtype == 1 ? oracle_f16_to_f32(w16[r * K + j])
                             : oracle_bf16_to_f32(w16[r * K + j]);
      volatile float q = v / sc;
      float c = q;
      if (c == c) c = c < -E4M3_MAX ? -E4M3_MAX : (c > E4M3_MAX ? E4M3_MAX : c);
      wq[r * K + j] = oracle_e4m3_encode(c, 0);
    }
  }
}

/*
 * acc[m,n] = sum_k e4m3(xq[m,k]) * e4m3(wq[n,k])   (csrc/fp8_gemm.cu:109-131, 180-184;
 *            products of two e4m3 values are exact in fp32, the sum is taken in
 *            double here and rounded once, i.e. the exact-sum limit of any fp32
 *            accumulation order)
 * out[m,n] = (acc * xs[m]) * ws[n] + float(bias16[n])   (csrc/fp8_gemm.cu:75-77)
 * bias16 is the bias already rounded to fp16 (csrc/fp8_gemm.cu:171), or NULL.
 * round_out != 0 rounds out to fp16 like csrc/fp8_gemm.cu:78 (returned widened to fp32).
 */
void oracle_gemm_dequant(const uint8_t *xq, const float *xs, const uint8_t *wq,
                         const float *ws, const uint16_t *bias16, int64_t M,
                         int64_t N, int64_t K, int round_out, float *acc_out,
                         float *out) {
  float lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = oracle_e4m3_decode((uint8_t)i);
  for (int64_t m = 0; m < M; ++m) {
    const uint8_t *a = xq + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const uint8_t *b = wq + n * K;
      double s = 0.0;
      for (int64_t k = 0; k < K; ++k) s += (double)lut[a[k]] * (double)lut[b[k]];
      float acc = (float)s;
      if (acc_out) acc_out[m * N + n] = acc;
      volatile float t = acc * xs[m];
      volatile float v = t * ws[n];
      if (bias16) v = v + oracle_f16_to_f32(bias16[n]);
      out[m * N + n] = round_out ? oracle_f16_to_f32(oracle_f32_to_f16(v)) : v;
    }
  }
}

/*
 * Block-scale layout, csrc/quantize.cu:75-83: 512-byte tiles of 128 rows x 4 scale
 * columns, tiles K-major (column-tile stride 512 B, row-tile stride 512 * ncb B); inside
 * a tile, scale (r, c) sits at (r % 32) * 16 + ((r % 128) / 32) * 4 + c % 4.
 */
int64_t oracle_mx_sf_offset(int64_t r, int64_t c, int64_t ncb) {
  return (r / 128) * (ncb * 512) + (c / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4);
}

/* Bytes of the padded scale grid for `rows` rows of K elements (K % 32 == 0). */
int64_t oracle_mx_sf_bytes(int64_t rows, int64_t K) {
  return ((rows + 127) / 128) * ((K / 32 + 3) / 4) * 512;
}

/*
 * MXFP8 quantization, csrc/quantize.cu:92-131 (one 32-element block of a row):
 *   amax = fmaxf-reduce |x| over the block (NaN ignored unless the block is all NaN)
 *   amax > 0 (false for 0 and NaN):
 *       e8 = clamp(floor(log2(amax)) - 8 + 127, 0, 254), where floor(log2(amax)) is
 *            the binary exponent of amax (frexpf's exponent - 1). The reference
 *            evaluates floorf(log2f(amax)); for every bf16 and fp16 amax the two agree
 *            (pinned against the reference over all of them). An infinite amax takes
 *            the upper clamp: e8 = 254.
 *   otherwise e8 = 127
 *   x_inv = 2^(127 - e8)  (exact power of two)
 *   q     = e4m3_satfinite(fminf(fmaxf(x * x_inv, -448), 448))
 * The scale grid (oracle_mx_sf_bytes) is prefilled with 127 (e8m0 1.0) and each block's
 * e8 written at oracle_mx_sf_offset(row, block, ncb) (csrc/quantize.cu:253-257).
 */
void oracle_quantize_mxfp8(const uint16_t *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                           uint8_t *scales) {
  const int64_t nblk = K / 32, ncb = (nblk + 3) / 4;
  memset(scales, 127, (size_t)oracle_mx_sf_bytes(M, K));
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < nblk; ++g) {
      const uint16_t *blk = x + r * K + g * 32;
      float v[32];
      float amax = 0.0f;
      int first = 1;
      for (int j = 0; j < 32; ++j) {
        v[j] = dtype ? oracle_f16_to_f32(blk[j]) : oracle_bf16_to_f32(blk[j]);
        float a = fabsf(v[j]);
        amax = first ? a : fmaxf(amax, a);
        first = 0;
      }
      int e8;
      float x_inv;
      if (amax > 0.0f) {
        if (isinf(amax)) {
          e8 = 254;
        } else {
          int e2;
          (void)frexpf(amax, &e2);
          int ee = (e2 - 1) - 8 + 127;
          e8 = ee < 0 ? 0 : (ee > 254 ? 254 : ee);
        }
        x_inv = ldexpf(1.0f, 127 - e8);
      } else {
        e8 = 127;
        x_inv = 1.0f;
      }
      scales[oracle_mx_sf_offset(r, g, ncb)] = (uint8_t)e8;
      for (int j = 0; j < 32; ++j) {
        volatile float p = v[j] * x_inv;
        float c = fminf(fmaxf(p, -E4M3_MAX), E4M3_MAX);
        xq[r * K + g * 32 + j] = oracle_e4m3_encode(c, 1);
      }
    }
  }
}

/*
 * MXFP8 GEMM, csrc/fp8_gemm.cu:233-333: D = A * B with per-32 e8m0 block scales on both
 * operands, bias epilogue, fp16 out:
 *   acc[m,n] = sum_k e4m3(xq[m,k]) 2^(xs[m,k/32]-127) * e4m3(wq[n,k]) 2^(ws[n,k/32]-127)
 *              (each term exact in double; the sum in double, rounded once to fp32)
 *   out[m,n] = acc + float(bias16[n])  (bias16: the bias rounded to fp16, :257-260)
 * round_out != 0 rounds out to fp16 (returned widened to fp32). Scale arrays are in
 * the tiled layout of their operand (rows M for xs, N for ws).
 */
void oracle_mxfp8_gemm(const uint8_t *xq, const uint8_t *xs, const uint8_t *wq,
                       const uint8_t *ws, const uint16_t *bias16, int64_t M, int64_t N,
                       int64_t K, int round_out, float *out) {
  float lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = oracle_e4m3_decode((uint8_t)i);
  const int64_t nblk = K / 32, ncb = (nblk + 3) / 4;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double s = 0.0;
      for (int64_t g = 0; g < nblk; ++g) {
        const double sa = ldexp(1.0, (int)xs[oracle_mx_sf_offset(m, g, ncb)] - 127);
        const double sb = ldexp(1.0, (int)ws[oracle_mx_sf_offset(n, g, ncb)] - 127);
        double part = 0.0;
        for (int64_t j = 0; j < 32; ++j)
          part += (double)lut[xq[m * K + g * 32 + j]] * (double)lut[wq[n * K + g * 32 + j]];
        s += part * sa * sb;
      }
      volatile float v = (float)s;
      if (bias16) v = v + oracle_f16_to_f32(bias16[n]);
      out[m * N + n] = round_out ? oracle_f16_to_f32(oracle_f32_to_f16(v)) : v;
    }
  }
}

/*
 * NVFP4 e2m1 encoding of csrc/quantize.cu:136-150: sign bit 8 when v < 0 (so -0.0 and
 * NaN get no sign), magnitude code by thresholds (ties go up):
 * |v| < 0.25 -> 0, < 0.75 -> 1 (0.5), < 1.25 -> 2 (1), < 1.75 -> 3 (1.5), < 2.5 -> 4 (2),
 * < 3.5 -> 5 (3), < 5 -> 6 (4), else 7 (6).
 */
uint8_t oracle_e2m1_encode(float v) {
  uint8_t s = v < 0.0f ? 8 : 0;
  float a = fabsf(v);
  uint8_t c;
  if (a < 0.25f) c = 0;
  else if (a < 0.75f) c = 1;
  else if (a < 1.25f) c = 2;
  else if (a < 1.75f) c = 3;
  else if (a < 2.5f) c = 4;
  else if (a < 3.5f) c = 5;
  else if (a < 5.0f) c = 6;
  else c = 7;
  return (uint8_t)(s | c);
}

float oracle_e2m1_decode(uint8_t c) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float v = mag[c & 7];
  return (c & 8) ? -v : v;
}

/* Bytes of the NVFP4 scale grid: 16-element blocks, so ceil((K / 16) / 4) tile columns. */
int64_t oracle_nv_sf_bytes(int64_t rows, int64_t K) {
  return ((rows + 127) / 128) * ((K / 16 + 3) / 4) * 512;
}

/*
 * NVFP4 quantization, csrc/quantize.cu:157-194 (one 16-element block of a row):
 *   amax  = fmaxf-reduce |x| (NaN ignored unless the block is all NaN)
 *   s     = fminf(amax * fl(1/6), 448)      (fminf ignores a NaN amax: 448)
 *   s8    = e4m3_satfinite(s), sdec = decode(s8)
 *   x_inv = sdec > 0 ? 1 / sdec : 0         (IEEE divide)
 *   code  = e2m1(fminf(fmaxf(x * x_inv, -6), 6))
 * Codes pack two per byte, element 2j in the low nibble; scales land at
 * oracle_mx_sf_offset(row, block, ncb) of a grid prefilled with 0x38 (e4m3 1.0).
 */
void oracle_quantize_nvfp4(const uint16_t *x, int dtype, int64_t M, int64_t K, uint8_t *xq,
                           uint8_t *scales) {
  const int64_t nblk = K / 16, ncb = (nblk + 3) / 4;
  const float inv6 = 1.0f / 6.0f;
  memset(scales, 0x38, (size_t)oracle_nv_sf_bytes(M, K));
  for (int64_t r = 0; r < M; ++r) {
    for (int64_t g = 0; g < nblk; ++g) {
      const uint16_t *blk = x + r * K + g * 16;
      float v[16];
      float amax = 0.0f;
      for (int j = 0; j < 16; ++j) {
        v[j] = dtype ? oracle_f16_to_f32(blk[j]) : oracle_bf16_to_f32(blk[j]);
        float a = fabsf(v[j]);
        amax = j == 0 ? a : fmaxf(amax, a);
      }
      volatile float sp = amax * inv6;
      float sc = fminf(sp, E4M3_MAX);
      uint8_t s8 = oracle_e4m3_encode(sc, 1);
      float sdec = oracle_e4m3_decode(s8);
      volatile float x_inv = sdec > 0.0f ? 1.0f / sdec : 0.0f;
      scales[oracle_mx_sf_offset(r, g, ncb)] = s8;
      for (int j = 0; j < 16; j += 2) {
        volatile float p0 = v[j] * x_inv, p1 = v[j + 1] * x_inv;
        uint8_t lo = oracle_e2m1_encode(fminf(fmaxf(p0, -6.0f), 6.0f));
        uint8_t hi = oracle_e2m1_encode(fminf(fmaxf(p1, -6.0f), 6.0f));
        xq[(r * K + g * 16 + j) / 2] = (uint8_t)(lo | (hi << 4));
      }
    }
  }
}

/*
 * NVFP4 GEMM: out[m,n] = sum_k e2m1(xq[m,k]) s_x[m,k/16] * e2m1(wq[n,k]) s_w[n,k/16]
 * + float(bias16[n]); the scales are e4m3 bytes of the tiled grids; each term exact
 * in double, the sum in double rounded once to fp32; round_out rounds to fp16.
 * xq / wq: packed [rows, K/2].
 */
void oracle_nvfp4_gemm(const uint8_t *xq, const uint8_t *xs, const uint8_t *wq,
                       const uint8_t *ws, const uint16_t *bias16, int64_t M, int64_t N,
                       int64_t K, int round_out, float *out) {
  const int64_t nblk = K / 16, ncb = (nblk + 3) / 4;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double s = 0.0;
      for (int64_t g = 0; g < nblk; ++g) {
        const double sa = oracle_e4m3_decode(xs[oracle_mx_sf_offset(m, g, ncb)]);
        const double sb = oracle_e4m3_decode(ws[oracle_mx_sf_offset(n, g, ncb)]);
        double part = 0.0;
        for (int64_t j = 0; j < 16; ++j) {
          const int64_t k = g * 16 + j;
          const uint8_t a = (uint8_t)((xq[(m * K + k) / 2] >> ((k & 1) * 4)) & 15);
          const uint8_t b = (uint8_t)((wq[(n * K + k) / 2] >> ((k & 1) * 4)) & 15);
          part += (double)oracle_e2m1_decode(a) * (double)oracle_e2m1_decode(b);
        }
        s += part * sa * sb;
      }
      volatile float v = (float)s;
      if (bias16) v = v + oracle_f16_to_f32(bias16[n]);
      out[m * N + n] = round_out ? oracle_f16_to_f32(oracle_f32_to_f16(v)) : v;
    }
  }
}

/*
 * LayerNorm (no affine, eps) + modulation + per-token quantization, in the order of the
 * fused kernel (fp8linear_b200's ln_mod_quant_kernel):
 *   sum  = fp32 partial sums per lane l = 0..31 over the elements of its 8-element chunks
 *          l, l + 32, l + 64, ... in sequence, then a butterfly over xor offsets
 *          16, 8, 4, 2, 1 (lane l adds lane l^o's partial)
 *   mean = sum / K; var = (same order over (x - mean)^2, a multiply then an add) / K
 *   rstd = 1 / sqrtf(var + eps)
 *   y    = R(R(R((x - mean) * rstd) * R(1 + scale[b])) + shift[b]), R = round to x's type
 * then the rule of oracle_quantize_rows on y. Row r belongs to batch r / (M / batches);
 * shift and scale are [batches, K] of x's type. dtype 0 = bf16, 1 = fp16.
 */
static float round_to(float v, int dtype) {
  return dtype ? oracle_f16_to_f32(oracle_f32_to_f16(v)) : oracle_bf16_to_f32(oracle_f32_to_bf16(v));
}

static float lane_tree(float *part) {
  float tmp[32];
  for (int o = 16; o > 0; o >>= 1) {
    for (int l = 0; l < 32; ++l) tmp[l] = part[l] + part[l ^ o];
    memcpy(part, tmp, sizeof(tmp));
  }
  return part[0];
}

void oracle_ln_modulate_quantize(const uint16_t *x, int dtype, int64_t M, int64_t K,
                                 int64_t batches, const uint16_t *shift, const uint16_t *scale,
                                 float eps, uint16_t *y, uint8_t *xq, float *xs) {
  const int64_t nch = K / 8, rpb = M / batches;
  for (int64_t r = 0; r < M; ++r) {
    const uint16_t *row = x + r * K;
    float part[32];
    for (int l = 0; l < 32; ++l) {
      part[l] = 0.0f;
      for (int64_t c = l; c < nch; c += 32)
        for (int e = 0; e < 8; ++e) {
          float v = dtype ? oracle_f16_to_f32(row[8 * c + e]) : oracle_bf16_to_f32(row[8 * c + e]);
          part[l] = part[l] + v;
        }
    }
    volatile float mean = lane_tree(part) / (float)K;
    for (int l = 0; l < 32; ++l) {
      part[l] = 0.0f;
      for (int64_t c = l; c < nch; c += 32)
        for (int e = 0; e < 8; ++e) {
          float v = dtype ? oracle_f16_to_f32(row[8 * c + e]) : oracle_bf16_to_f32(row[8 * c + e]);
          volatile float d = v - mean;
          volatile float dd = d * d;
          part[l] = part[l] + dd;
        }
    }
    volatile float var = lane_tree(part) / (float)K;
    volatile float den = sqrtf(var + eps);
    volatile float rstd = 1.0f / den;
    const int64_t b = r / rpb;
    uint16_t *yr = y + r * K;
    for (int64_t j = 0; j < K; ++j) {
      float v = dtype ? oracle_f16_to_f32(row[j]) : oracle_bf16_to_f32(row[j]);
      float sc = dtype ? oracle_f16_to_f32(scale[b * K + j]) : oracle_bf16_to_f32(scale[b * K + j]);
      float sh = dtype ? oracle_f16_to_f32(shift[b * K + j]) : oracle_bf16_to_f32(shift[b * K + j]);
      volatile float dv = v - mean;
      float ln = round_to(dv * rstd, dtype);
      float m1 = round_to(1.0f + sc, dtype);
      float t = round_to(ln * m1, dtype);
      float yv = round_to(t + sh, dtype);
      yr[j] = dtype ? oracle_f32_to_f16(yv) : oracle_f32_to_bf16(yv);
    }
  }
  oracle_quantize_rows(y, dtype, M, K, xq, xs);
}
