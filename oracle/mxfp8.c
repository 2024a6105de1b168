/*
 * CPU oracle of the MXFP8 quantiser — TEST INFRASTRUCTURE ONLY (built into
 * oracle/_build/libce4oracle.so and loaded by tests/ through oracle/mxfp8.py).
 *
 * Restates the quantiser the reference's custom MXFP8 path uses (ThunderKittens
 * mxfp8_quantize, third_party/ThunderKittens/kernels/gemm/mxfp8_b200/mxfp8_b200_gemm.cu
 * :380-426, wrapped by src/chess_engine_4/kernels/dense.py:46-60), from the OCP MX
 * format definitions (E8M0: 8-bit biased power-of-two exponent, bias 127, 0xFF = NaN;
 * E4M3 "fn": 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, max 448, 0x7F = NaN):
 *
 *   per row, per 32-column block:  amax = max |x| (x BF16)
 *   s  = max(amax * 0.002232142857f, 1e-12f)            (FP32)
 *   S  = E8M0(s) rounded toward +inf, saturating to the largest finite code (254)
 *   q  = E4M3(x * (1 / 2^(S - 127))) rounded to nearest-even, saturating to +-448
 *
 * Scale bytes are stored per 128x128 tile as [32][16]: the byte of tile row r and
 * 32-column block kb (0..3) sits at (r % 32) * 16 + (r / 32) * 4 + kb
 * (mxfp8_b200_gemm.cu:415-422), tiles ordered [row tile][column tile].
 * An all-zero block therefore gets S = 88 (2^-39, from the 1e-12 floor).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static uint32_t f32_bits(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  return b;
}

static float bits_f32(uint32_t b) {
  float v;
  memcpy(&v, &b, 4);
  return v;
}

static float bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* Smallest E8M0 code whose value 2^(S-127) is >= v (v > 0, finite), saturating at 254. */
uint8_t ce4o_e8m0_round_up(float v) {
  const uint32_t b = f32_bits(v);
  const int exp = (int)((b >> 23) & 0xFF);
  const uint32_t mant = b & 0x7FFFFF;
  if (exp == 0xFF) return 254; /* inf: saturate (NaN does not occur: amax >= 0) */
  int s;
  if (exp == 0) {
    /* FP32 subnormal: value = mant * 2^-149 < 2^-126; round up to a power of two. */
    if (mant == 0) return 0;
    int top = 31;
    while (!(mant & (1u << top))) --top;                 /* value in [2^(top-149), 2^(top-148)) */
    const int e = (mant & ((1u << top) - 1)) ? top - 148 : top - 149;
    s = e + 127;
  } else {
    s = exp + (mant != 0 ? 1 : 0); /* biased exponent of the next power of two */
  }
  if (s < 0) s = 0;
  if (s > 254) s = 254;
  return (uint8_t)s;
}

/* Value of an E8M0 code (S = 0..254). */
float ce4o_e8m0_value(uint8_t s) { return ldexpf(1.0f, (int)s - 127); }

/* FP32 -> E4M3 ("fn"), round to nearest even, saturating finite values to +-448. */
uint8_t ce4o_e4m3_rne_satfinite(float v) {
  const uint32_t b = f32_bits(v);
  const uint8_t sign = (uint8_t)((b >> 24) & 0x80);
  const int exp = (int)((b >> 23) & 0xFF);
  const uint32_t mant = b & 0x7FFFFF;
  if (exp == 0xFF && mant != 0) return (uint8_t)(sign | 0x7F); /* NaN */
  if (exp == 0xFF) return (uint8_t)(sign | 0x7E);              /* inf -> max finite */
  if (exp == 0) return sign;                                   /* FP32 subnormal -> 0 */
  const int e = exp - 127;
  uint32_t code;
  if (e >= -6) {
    /* Normal E4M3: keep 3 of the 23 mantissa bits. */
    uint32_t m = mant >> 20;
    const uint32_t rem = mant & 0xFFFFF;
    int ee = e;
    if (rem > 0x80000 || (rem == 0x80000 && (m & 1))) ++m;
    if (m == 8) {
      m = 0;
      ++ee;
    }
    if (ee > 8 || (ee == 8 && m > 6)) return (uint8_t)(sign | 0x7E); /* > 448: saturate */
    code = ((uint32_t)(ee + 7) << 3) | m;
  } else {
    /* Subnormal E4M3: q = round(v * 2^9), an integer 0..8 (8 = smallest normal). */
    const uint32_t sig = 0x800000 | mant; /* 1.mant * 2^23 */
    const int shift = 23 - (e + 9);       /* > 23 because e < -6 */
    if (shift >= 32) return sign;
    uint32_t q = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) ++q;
    code = q; /* q == 8 encodes exponent field 1, mantissa 0 */
  }
  return (uint8_t)(sign | code);
}

/* Quantise a BF16 [rows, cols] matrix (rows, cols multiples of 128). */
void ce4o_quantize_mxfp8(const uint16_t* x, int rows, int cols, uint8_t* values, uint8_t* scales) {
  const int col_tiles = cols / 128;
  for (int r = 0; r < rows; ++r) {
    for (int blk = 0; blk < cols / 32; ++blk) {
      const uint16_t* src = x + (size_t)r * cols + blk * 32;
      float amax = 0.0f;
      for (int j = 0; j < 32; ++j) {
        const float a = fabsf(bf16_to_f32(src[j]));
        if (a > amax) amax = a;
      }
      float s = amax * 0.002232142857f;
      if (!(s > 1e-12f)) s = 1e-12f;
      const uint8_t code = ce4o_e8m0_round_up(s);
      const float inv = 1.0f / ce4o_e8m0_value(code);
      for (int j = 0; j < 32; ++j) {
        values[(size_t)r * cols + blk * 32 + j] = ce4o_e4m3_rne_satfinite(bf16_to_f32(src[j]) * inv);
      }
      const int tile = (r / 128) * col_tiles + (blk * 32) / 128;
      const int tr = r % 128;
      const int kb = blk % 4;
      scales[(size_t)tile * 512 + (tr % 32) * 16 + (tr / 32) * 4 + kb] = code;
    }
  }
}

/* Value of an E4M3 code. */
float ce4o_e4m3_value(uint8_t c) {
  const float sign = (c & 0x80) ? -1.0f : 1.0f;
  const int e = (c >> 3) & 0xF;
  const int m = c & 7;
  if (e == 0xF && m == 7) return NAN;
  if (e == 0) return sign * ldexpf((float)m, -9);
  return sign * ldexpf(1.0f + m / 8.0f, e - 7);
}
