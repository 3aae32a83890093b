/*
 * CPU oracle for the quantized-linear hot path.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
 * reference legs load this; the product path (rdna2_ops + the CUDA library)
 * never does.
 *
 * Every routine restates the reference algorithm in plain C with IEEE fp32
 * arithmetic.  Build with -ffp-contract=off (oracle/build.py does): a*b+c must
 * round twice unless fmaf() is written explicitly.
 *
 * Reference anchors (paths inside unixyo/rdna2-gfx1030-ai-handbook):
 *   integer GEMM      rdna2-ops/bench_int8_gemm.py:193 (INT64 oracle a@b)
 *   fused epilogue    rdna2-ops/rdna2_ops/int8_gemm.py:53-63
 *                     float(acc)*(sa*sb) (+bias fp32), FMA off unless
 *                     rounding="fused" (int8_gemm.py:191)
 *   Kitchen epilogue  rdna2-ops/production/MOSS_RDNA2_INT8/backend.py:128-143
 *                     (float(acc)*(sx*sw)).to(out) then + bias.to(out)
 *   row quantizer     rdna2-ops/rdna2_ops/fp8_weight_gemm_v06.py:76-92 (absmax/127
 *                     per row; ties here are RNE as the north-star contract says)
 *   INT4 packer       rdna2-ops/rdna2_ops/int4_weight_gemm_v07.py:49-92
 *   FP8 decode        rdna2-ops/rdna2_ops/fp8_weight_gemm_v06.py:22-37
 *   ConvRot rotation  comfy_kitchen 0.2.40 _build_hadamard/_rotate_activation is
 *                     not vendored (call site backend.py:112-118); the frozen
 *                     contract is: fp32 butterflies h=1,2,..,B/2 on pairs
 *                     (i,i+h) -> (a+b, a-b), then one multiply by
 *                     fp32(1/sqrt(B)).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };
enum { EPI_SEPARATE = 0, EPI_FMA = 1, EPI_KITCHEN = 2 };

/* ------------------------------------------------------------------ codecs */

static inline uint32_t bits_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float float_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Round-to-nearest-even of an unsigned mantissa shifted right by s (1..31). */
static inline uint32_t rne_shift(uint32_t m, int s) {
  uint32_t q = m >> s, rem = m & ((1u << s) - 1u), half = 1u << (s - 1);
  if (rem > half || (rem == half && (q & 1u))) q++;
  return q;
}

uint16_t b2o_f32_to_f16(float f) {
  uint32_t x = bits_of(f), sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
  if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
  int e = (int)(ax >> 23) - 127;
  uint32_t m = (ax & 0x7fffffu) | (ax >= 0x00800000u ? 0x800000u : 0u);
  if (ax < 0x00800000u) e = -126;            /* fp32 subnormal */
  if (e > 15) return (uint16_t)(sign | 0x7c00u);
  if (e >= -14) {                            /* half normal range */
    uint32_t h = ((uint32_t)(e + 15) << 10) | ((m >> 13) & 0x3ffu);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  /* may carry to inf */
    return (uint16_t)(sign | h);
  }
  int s = -(e + 1);                          /* value / 2^-24 = m * 2^(e+1) */
  if (s >= 25) return (uint16_t)sign;
  return (uint16_t)(sign | rne_shift(m, s));
}

float b2o_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 0x3ffu;
  if (e == 31) return float_of(sign | 0x7f800000u | (m << 13));
  if (e == 0) {
    float v = (float)m * 5.9604644775390625e-08f;   /* 2^-24, exact */
    return sign ? -v : v;
  }
  return float_of(sign | ((e + 112u) << 23) | (m << 13));
}

uint16_t b2o_f32_to_bf16(float f) {
  uint32_t x = bits_of(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

float b2o_bf16_to_f32(uint16_t h) { return float_of((uint32_t)h << 16); }

/* e4m3 "fn" flavour: bias 7, no infinities, 0x7f/0xff are NaN, max 448.
 * Encoding is round-to-nearest-even with saturation to +-448 (satfinite). */
uint8_t b2o_f32_to_e4m3(float f) {
  uint32_t x = bits_of(f), sign = (x >> 24) & 0x80u, ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return (uint8_t)(sign | 0x7fu);
  if (ax >= 0x43e00000u) return (uint8_t)(sign | 0x7eu);   /* >= 448 */
  int e = (int)(ax >> 23) - 127;
  uint32_t m = (ax & 0x7fffffu) | (ax >= 0x00800000u ? 0x800000u : 0u);
  if (ax < 0x00800000u) e = -126;
  if (e >= -6) {
    uint32_t v = ((uint32_t)(e + 7) << 3) | ((m >> 20) & 7u);
    uint32_t rem = m & 0xfffffu;
    if (rem > 0x80000u || (rem == 0x80000u && (v & 1u))) v++;
    if (v > 0x7eu) v = 0x7eu;                                 /* satfinite */
    return (uint8_t)(sign | v);
  }
  int s = 14 - e;                            /* value / 2^-9 = m * 2^(e-14) */
  if (s >= 25) return (uint8_t)sign;
  return (uint8_t)(sign | rne_shift(m, s));
}

float b2o_e4m3_to_f32(uint8_t b) {
  uint32_t e = (b >> 3) & 15u, m = b & 7u;
  float v;
  if (e == 15 && m == 7) return float_of(0x7fc00000u | ((uint32_t)(b & 0x80u) << 24));
  if (e == 0) v = (float)m * 0.001953125f;                    /* 2^-9 */
  else v = float_of(((e + 120u) << 23) | (m << 20));
  return (b & 0x80u) ? -v : v;
}

static inline float load_elem(const void* base, int dtype, int64_t i) {
  if (dtype == DT_F32) return ((const float*)base)[i];
  if (dtype == DT_F16) return b2o_f16_to_f32(((const uint16_t*)base)[i]);
  return b2o_bf16_to_f32(((const uint16_t*)base)[i]);
}

static inline void store_elem(void* base, int dtype, int64_t i, float v) {
  if (dtype == DT_F32) ((float*)base)[i] = v;
  else if (dtype == DT_F16) ((uint16_t*)base)[i] = b2o_f32_to_f16(v);
  else ((uint16_t*)base)[i] = b2o_f32_to_bf16(v);
}

/* Round a float through the storage dtype (identity for fp32). */
static inline float through(int dtype, float v) {
  if (dtype == DT_F16) return b2o_f16_to_f32(b2o_f32_to_f16(v));
  if (dtype == DT_BF16) return b2o_bf16_to_f32(b2o_f32_to_bf16(v));
  return v;
}

/* --------------------------------------------------------- prologue math */

/* In-place orthonormal block-Hadamard of one fp32 row (block = power of 2). */
static void fwht_row(float* x, int64_t K, int block, float inv) {
  for (int64_t b0 = 0; b0 < K; b0 += block) {
    float* v = x + b0;
    for (int h = 1; h < block; h <<= 1)
      for (int i = 0; i < block; i++)
        if (!(i & h)) {
          float a = v[i], c = v[i + h];
          v[i] = a + c;
          v[i + h] = a - c;
        }
    for (int i = 0; i < block; i++) v[i] = v[i] * inv;
  }
}

float b2o_rotation_scale(int block) { return (float)(1.0 / sqrt((double)block)); }

/* x: [M,K] with row stride ldx (elements) of dtype; block 0 = no rotation.
 * out: [M,K] fp32 contiguous. */
void b2o_rotate_rows(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                     int block, float* out) {
  float inv = block > 1 ? b2o_rotation_scale(block) : 1.0f;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; r++) {
    float* o = out + r * K;
    for (int64_t k = 0; k < K; k++) o[k] = load_elem(x, dtype, r * ldx + k);
    if (block > 1) fwht_row(o, K, block, inv);
  }
}

/* Per-row symmetric INT8: s = absmax/127 (IEEE division), s := 1 when it is
 * not positive, q = clamp(rint(x/s), -127, 127) with ties to even. */
void b2o_quant_rows_int8(const float* x, int64_t M, int64_t K, int8_t* q,
                         int64_t ldq, float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; r++) {
    const float* v = x + r * K;
    float amax = 0.0f;
    for (int64_t k = 0; k < K; k++) { float a = fabsf(v[k]); if (a > amax) amax = a; }
    float s = amax / 127.0f;
    if (!(s > 0.0f)) s = 1.0f;
    for (int64_t k = 0; k < K; k++) {
      float z = rintf(v[k] / s);
      if (z > 127.0f) z = 127.0f;
      if (z < -127.0f) z = -127.0f;
      q[r * ldq + k] = (int8_t)z;
    }
    for (int64_t k = K; k < ldq; k++) q[r * ldq + k] = 0;
    scale[r] = s;
  }
}

/* The reference's in-repo row quantizer _quant_rows
 * (rdna2-ops/rdna2_ops/fp8_weight_gemm_v06.py:76-92): step = max(absmax/127,
 * 1e-20); z = x/step; q = z >= 0 ? floor(z + 0.5) : ceil(z - 0.5) with the
 * fp32 rounding of z +- 0.5; clamp to [-127, 127]. */
void b2o_quant_rows_ref(const float* x, int64_t M, int64_t K, int8_t* q, int64_t ldq,
                        float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; r++) {
    const float* v = x + r * K;
    float amax = 0.0f;
    for (int64_t k = 0; k < K; k++) { float a = fabsf(v[k]); if (a > amax) amax = a; }
    float s = amax / 127.0f;
    if (s < 1.0e-20f) s = 1.0e-20f;
    for (int64_t k = 0; k < K; k++) {
      float z = v[k] / s;
      float t = z >= 0.0f ? floorf(z + 0.5f) : ceilf(z - 0.5f);
      if (t > 127.0f) t = 127.0f;
      if (t < -127.0f) t = -127.0f;
      q[r * ldq + k] = (int8_t)t;
    }
    scale[r] = s;
  }
}

float b2o_e5m2_to_f32(uint8_t b) { return b2o_f16_to_f32((uint16_t)((uint16_t)b << 8)); }

void b2o_decode_e5m2(const uint8_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = b2o_e5m2_to_f32(x[i]);
}

/* Per-row e4m3: s = absmax/448, s := 1 when not positive, q = e4m3_rn_sat(x/s). */
void b2o_quant_rows_e4m3(const float* x, int64_t M, int64_t K, uint8_t* q,
                         int64_t ldq, float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; r++) {
    const float* v = x + r * K;
    float amax = 0.0f;
    for (int64_t k = 0; k < K; k++) { float a = fabsf(v[k]); if (a > amax) amax = a; }
    float s = amax / 448.0f;
    if (!(s > 0.0f)) s = 1.0f;
    for (int64_t k = 0; k < K; k++) q[r * ldq + k] = b2o_f32_to_e4m3(v[k] / s);
    for (int64_t k = K; k < ldq; k++) q[r * ldq + k] = 0;
    scale[r] = s;
  }
}

/* ------------------------------------------------------------- GEMM core */

/* c[m,n] = sum_k a[m,k]*b[n,k] exactly (|sum| < 2^31 for K <= 131071).
 * a: [M,K] row stride lda; b: [N,K] row stride ldb (weight layout). */
void b2o_gemm_s8(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb,
                 int64_t M, int64_t N, int64_t K, int32_t* c, int64_t ldc,
                 int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  const int64_t BM = 16, BN = 64;
  int64_t tm = (M + BM - 1) / BM, tn = (N + BN - 1) / BN;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t t = 0; t < tm * tn; t++) {
    int64_t m0 = (t / tn) * BM, n0 = (t % tn) * BN;
    int64_t m1 = m0 + BM < M ? m0 + BM : M, n1 = n0 + BN < N ? n0 + BN : N;
    for (int64_t m = m0; m < m1; m++) {
      const int8_t* ar = a + m * lda;
      for (int64_t n = n0; n < n1; n++) {
        const int8_t* br = b + n * ldb;
        int32_t acc = 0;
        for (int64_t k = 0; k < K; k++) acc += (int32_t)ar[k] * (int32_t)br[k];
        c[m * ldc + n] = acc;
      }
    }
  }
}

/* Fused or Kitchen epilogue over an INT32 accumulator.
 * sb_count is N (per channel) or 1 (scalar); bias may be NULL.
 * EPI_SEPARATE: v = float(acc)*(sa*sb); v = v + float(bias); out = cvt(v)
 * EPI_FMA:      v = fma(float(acc), sa*sb, float(bias))        (bias present)
 * EPI_KITCHEN:  y = cvt(float(acc)*(sa*sb)); y = cvt(y + cvt(bias))  */
void b2o_epilogue_s32(const int32_t* acc, int64_t ldacc, const float* sa,
                      const float* sb, int64_t sb_count, const void* bias,
                      int bias_dtype, int64_t M, int64_t N, int mode,
                      void* out, int out_dtype, int64_t ldo) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; m++) {
    for (int64_t n = 0; n < N; n++) {
      float s = sa[m] * sb[sb_count == 1 ? 0 : n];
      float a = (float)acc[m * ldacc + n];
      float v;
      if (mode == EPI_KITCHEN) {
        v = through(out_dtype, a * s);
        if (bias) v = through(out_dtype, v + through(out_dtype, load_elem(bias, bias_dtype, n)));
      } else if (mode == EPI_FMA && bias) {
        v = fmaf(a, s, load_elem(bias, bias_dtype, n));
      } else {
        v = a * s;
        if (bias) v = v + load_elem(bias, bias_dtype, n);
      }
      store_elem(out, out_dtype, m * ldo + n, v);
    }
  }
}

/* Same epilogue over an fp32 accumulator (FP8 path): v = acc*(sa*sb) (+bias). */
void b2o_epilogue_f32(const double* acc, int64_t ldacc, const float* sa,
                      const float* sb, const void* bias, int bias_dtype, int64_t M,
                      int64_t N, void* out, int out_dtype, int64_t ldo) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; m++)
    for (int64_t n = 0; n < N; n++) {
      float v = (float)acc[m * ldacc + n] * (sa[m] * sb[n]);
      if (bias) v = v + load_elem(bias, bias_dtype, n);
      store_elem(out, out_dtype, m * ldo + n, v);
    }
}

/* Full W8A8 linear: rotate (optional) + row-quantize x, exact GEMM against the
 * already-quantized weight, epilogue.  Scratch buffers are caller-owned:
 * xr [M*K] fp32, q [M*K] int8, sa [M] fp32, acc [M*N] int32. */
void b2o_w8a8_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                     int block, const int8_t* w, int64_t ldw, const float* sw,
                     int64_t sw_count, const void* bias, int bias_dtype, int64_t N,
                     int mode, void* out, int out_dtype, float* xr, int8_t* q,
                     float* sa, int32_t* acc, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  b2o_rotate_rows(x, x_dtype, M, K, ldx, block, xr);
  b2o_quant_rows_int8(xr, M, K, q, K, sa);
  b2o_gemm_s8(q, K, w, ldw, M, N, K, acc, N, threads);
  b2o_epilogue_s32(acc, N, sa, sw, sw_count, bias, bias_dtype, M, N, mode, out,
                   out_dtype, N);
}

/* ------------------------------------------------------------ FP8 / INT4 */

/* acc[m,n] = sum_k dec(a[m,k]) * dec(b[n,k]) in double (e4m3 codes). */
void b2o_gemm_e4m3_f64(const uint8_t* a, int64_t lda, const uint8_t* b, int64_t ldb,
                       int64_t M, int64_t N, int64_t K, double* c, int threads) {
  static float lut[256];
  for (int i = 0; i < 256; i++) lut[i] = b2o_e4m3_to_f32((uint8_t)i);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t m = 0; m < M; m++)
    for (int64_t n = 0; n < N; n++) {
      double s = 0.0;
      for (int64_t k = 0; k < K; k++)
        s += (double)lut[a[m * lda + k]] * (double)lut[b[n * ldb + k]];
      c[m * N + n] = s;
    }
}

/* Affine/symmetric group INT4 packer, restating pack_int4_cpu
 * (int4_weight_gemm_v07.py:49-82) for layout "nk", order "low"/"high".
 * w: [N,K] fp32 contiguous.  Outputs: data [N,K/8] int32 words of signed
 * nibbles (q-8 for affine), scales [N,K/G] fp32, zeros [N,K/G] int32 (zu-8),
 * sums [N,K/G] int32. */
void b2o_pack_int4(const float* w, int64_t N, int64_t K, int G, int symmetric,
                   int order_high, int32_t* data, float* scales, int32_t* zeros,
                   int32_t* sums) {
  int64_t ng = K / G;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; n++) {
    for (int64_t g = 0; g < ng; g++) {
      const float* x = w + n * K + g * G;
      float scale;
      int32_t zero = 0, zu = 0, empty = 0;
      if (symmetric) {
        float amax = 0.0f;
        for (int i = 0; i < G; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
        scale = amax / 7.0f;
        if (scale == 0.0f) scale = 1.0f;
      } else {
        float lo = 0.0f, hi = 0.0f;
        for (int i = 0; i < G; i++) { if (x[i] < lo) lo = x[i]; if (x[i] > hi) hi = x[i]; }
        scale = (hi - lo) / 15.0f;
        empty = scale == 0.0f;
        if (empty) scale = 1.0f;
        float z = rintf(-lo / scale);
        if (z < 0.0f) z = 0.0f;
        if (z > 15.0f) z = 15.0f;
        zu = (int32_t)z;
        zero = empty ? 0 : zu - 8;
      }
      int32_t total = 0;
      for (int i = 0; i < G; i++) {
        int32_t q;
        if (symmetric) {
          float z = rintf(x[i] / scale);
          if (z < -7.0f) z = -7.0f;
          if (z > 7.0f) z = 7.0f;
          q = (int32_t)z;
        } else {
          float z = rintf(x[i] / scale) + (float)zu;
          if (z < 0.0f) z = 0.0f;
          if (z > 15.0f) z = 15.0f;
          q = empty ? 0 : (int32_t)z - 8;
        }
        total += q;
        int64_t k = g * G + i;
        int shift = (int)(k % 8) * 4;
        if (order_high) shift = 28 - shift;
        uint32_t* word = (uint32_t*)&data[n * (K / 8) + k / 8];
        if (k % 8 == 0) *word = 0;
        *word |= ((uint32_t)q & 15u) << shift;
      }
      scales[n * ng + g] = scale;
      zeros[n * ng + g] = zero;
      sums[n * ng + g] = total;
    }
  }
}

/* Dequantized INT4 weight as the W4A16 kernel sees it:
 * w = round_to(dtype, float(q - z) * s) with s already in storage precision.
 * words: [N,K/8] signed-nibble words (order low), scales/zeros fp32 [N,K/G]. */
void b2o_dequant_int4(const int32_t* words, const float* scales, const float* zeros,
                      int64_t N, int64_t K, int G, int out_dtype, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; n++)
    for (int64_t k = 0; k < K; k++) {
      uint32_t word = (uint32_t)words[n * (K / 8) + k / 8];
      int32_t q = (int32_t)((word >> ((k % 8) * 4)) & 15u);
      if (q >= 8) q -= 16;
      float s = scales[n * (K / G) + k / G], z = zeros[n * (K / G) + k / G];
      out[n * K + k] = through(out_dtype, ((float)q - z) * s);
    }
}

/* acc[m,n] = sum_k a[m,k]*w[n,k] in double over fp32 operands. */
void b2o_gemm_f32_f64(const float* a, int64_t M, const float* w, int64_t N, int64_t K,
                      double* c, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t m = 0; m < M; m++)
    for (int64_t n = 0; n < N; n++) {
      double s = 0.0;
      const float* ar = a + m * K;
      const float* wr = w + n * K;
      for (int64_t k = 0; k < K; k++) s += (double)ar[k] * (double)wr[k];
      c[m * N + n] = s;
    }
}

/* Bulk codec helpers so Python can convert arrays without per-element calls. */
void b2o_encode(const float* x, int64_t n, int dtype, void* out) {
  for (int64_t i = 0; i < n; i++) store_elem(out, dtype, i, x[i]);
}
void b2o_decode(const void* x, int64_t n, int dtype, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = load_elem(x, dtype, i);
}
void b2o_encode_e4m3(const float* x, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; i++) out[i] = b2o_f32_to_e4m3(x[i]);
}
void b2o_decode_e4m3(const uint8_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = b2o_e4m3_to_f32(x[i]);
}
/*
 * W4A8 grouped linear, restating rdna2-ops/int4_model_switches_v07.py:19-34
 * (grouped_integer_reference) and the float order of the reference kernels
 * (rdna2-ops/rdna2_ops/int4_weight_gemm_v07.py:194-216, enable_fp_fusion
 * off): for every group g the integer dot e = sum_k a[m,k] * c[n,k] over
 * the group's k (exact), total = total + fp32(e) * s[n,g] in group order
 * (product and sum each rounded), y = total * sa[m], then + bias[n].
 * integer != 0 returns the exact sum over all k instead (INTEGER mode).
 * a [M,K] int8 (row stride lda); c [N,K] int8 centered weights q - z;
 * s [N, K/G] fp32.
 */
void b2o_w4a8_linear(const int8_t* a, int64_t lda, int64_t M, int64_t K, const int8_t* c, int64_t N,
                     const float* s, int G, const float* sa, const float* bias, int integer,
                     float* out_f32, int32_t* out_i32) {
  const int64_t ng = K / G;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; m++) {
    for (int64_t n = 0; n < N; n++) {
      float total = 0.0f;
      int64_t exact_all = 0;
      for (int64_t g = 0; g < ng; g++) {
        int64_t e = 0;
        for (int64_t k = g * G; k < (g + 1) * G; k++) e += (int64_t)a[m * lda + k] * (int64_t)c[n * K + k];
        exact_all += e;
        const float prod = (float)e * s[n * ng + g];
        total = total + prod;
      }
      if (integer) {
        out_i32[m * N + n] = (int32_t)exact_all;
      } else {
        float y = total * sa[m];
        if (bias) y = y + bias[n];
        out_f32[m * N + n] = y;
      }
    }
  }
}

int b2o_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
