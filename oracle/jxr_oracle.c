/*
 * CPU oracle for the threefry2x32 random-bits path of jaxR.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, __graft_entry__.smoke()
 * and the CPU baseline leg of bench.py.  Nothing in the product links or calls
 * it.  Compiled with -ffp-contract=off so that every float operation below is
 * rounded exactly as written; fused multiply-adds appear only where fmaf/fma
 * is called explicitly.
 *
 * Reference lines cited are paths within the jaxR project.
 */
#include "jxr_oracle.h"
#include "erfinv_tables.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifdef _OPENMP
#define ORC_PAR_FOR _Pragma("omp parallel for schedule(static) num_threads(orc_get_threads())")
#else
#define ORC_PAR_FOR
#endif

static int g_threads = 0;

void orc_set_threads(int n) { g_threads = n; }

int orc_get_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---- the cipher ------------------------------------------------------------------------ */

static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

/* R/prng.R:51-86: key schedule ks = (k0, k1, k0^k1^0x1BD11BDA); x = (c0+ks0, c1+ks1);
 * five steps of four rounds (x0 += x1; x1 = rotl(x1, r); x1 ^= x0) with the rotation
 * sets (13,15,26,6) and (17,29,16,24) alternating, each step followed by the injection
 * x0 += ks[(i+1)%3], x1 += ks[(i+2)%3] + (i+1). */
static inline void tf(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t* o0,
                      uint32_t* o1) {
  static const int rot[2][4] = {{13, 15, 26, 6}, {17, 29, 16, 24}};
  const uint32_t ks[3] = {k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
  uint32_t x0 = c0 + ks[0], x1 = c1 + ks[1];
  for (int i = 0; i < 5; ++i) {
    const int* r = rot[i & 1];
    for (int j = 0; j < 4; ++j) {
      x0 += x1;
      x1 = rotl32(x1, r[j]);
      x1 ^= x0;
    }
    x0 += ks[(i + 1) % 3];
    x1 += ks[(i + 2) % 3] + (uint32_t)(i + 1);
  }
  *o0 = x0;
  *o1 = x1;
}

void orc_threefry2x32(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t out[2]) {
  tf(k0, k1, c0, c1, &out[0], &out[1]);
}

void orc_threefry2x32_arr(const uint32_t* k0, const uint32_t* k1, const uint32_t* c0,
                          const uint32_t* c1, uint32_t* x0, uint32_t* x1, int64_t n) {
  for (int64_t i = 0; i < n; ++i) tf(k0[i], k1[i], c0[i], c1[i], &x0[i], &x1[i]);
}

/* R/prng.R:102-120: pad odd n with one zero; block j hashes (flat[j], flat[half+j]);
 * the output is [x0 of all blocks, x1 of all blocks] cut to n. */
void orc_threefry_2x32(const uint32_t key[2], const uint32_t* count, int64_t n, uint32_t* out) {
  const int64_t half = (n + 1) / 2;
  for (int64_t j = 0; j < half; ++j) {
    uint32_t a, b;
    tf(key[0], key[1], count[j], half + j < n ? count[half + j] : 0u, &a, &b);
    out[j] = a;
    if (half + j < n) out[half + j] = b;
  }
}

/* Word g of threefry_2x32(key, iota(n)) without materialising the iota. */
static inline uint32_t iota_hash_word(const uint32_t key[2], uint64_t n, uint64_t g) {
  const uint64_t half = (n + 1) / 2;
  uint32_t a, b;
  if (g < half) {
    tf(key[0], key[1], (uint32_t)g, half + g < n ? (uint32_t)(half + g) : 0u, &a, &b);
    return a;
  }
  tf(key[0], key[1], (uint32_t)(g - half), (uint32_t)g, &a, &b);
  return b;
}

/* ---- seed / split / fold_in ------------------------------------------------------------ */

/* R/prng.R:160-170 with the int64 -> int32 wrap of R/prng.R:505-514: k1 is the seed
 * shifted right (logically) by 32, which is 0 for an int32 seed, k2 its low word. */
void orc_seed(int64_t seed, int x64, uint32_t out[2]) {
  if (x64) {
    out[0] = (uint32_t)((uint64_t)seed >> 32);
    out[1] = (uint32_t)(uint64_t)seed;
  } else {
    out[0] = 0u;
    out[1] = (uint32_t)(uint64_t)seed;
  }
}

/* Key s of split_original(key, num) (R/prng.R:173-177): threefry_2x32(key, iota(2 num))
 * reshaped to (num, 2). */
static inline void split_original_key(const uint32_t key[2], uint64_t num, uint64_t s,
                                      uint32_t out[2]) {
  out[0] = iota_hash_word(key, 2 * num, 2 * s);
  out[1] = iota_hash_word(key, 2 * num, 2 * s + 1);
}

/* R/prng.R:180-191. */
void orc_split(const uint32_t key[2], int64_t num, int partitionable, uint32_t* out) {
  for (int64_t j = 0; j < num; ++j) {
    if (partitionable) {
      tf(key[0], key[1], (uint32_t)((uint64_t)j >> 32), (uint32_t)j, &out[2 * j],
         &out[2 * j + 1]);
    } else {
      split_original_key(key, (uint64_t)num, (uint64_t)j, &out[2 * j]);
    }
  }
}

/* R/prng.R:194: threefry_2x32(key, seed(data)) with seed(uint32 d) = (0, d), one block. */
void orc_fold_in(const uint32_t key[2], uint32_t data, uint32_t out[2]) {
  tf(key[0], key[1], 0u, data, &out[0], &out[1]);
}

/* ---- random bits ----------------------------------------------------------------------- */

/* Word g of the original-layout stream of max_count uint32 words (R/prng.R:230-245):
 * below 2^32-1 words one hash of iota(max_count); otherwise the key is split into
 * nblocks+1 keys, each hashing iota(2^32-1) except the last, which hashes iota(rem). */
static inline uint32_t original_word(const uint32_t key[2], uint64_t max_count, uint64_t g) {
  const uint64_t U = 0xFFFFFFFFull;
  const uint64_t nblocks = max_count / U, rem = max_count % U;
  if (nblocks == 0) return iota_hash_word(key, max_count, g);
  const uint64_t s = g / U, local = g % U;
  uint32_t sk[2];
  split_original_key(key, nblocks + 1, s, sk);
  return iota_hash_word(sk, s < nblocks ? U : rem, local);
}

uint64_t orc_bits_at(const uint32_t key[2], int bit_width, uint64_t size, int partitionable,
                     uint64_t i) {
  if (partitionable) {
    /* R/prng.R:213-227 with the C-order iota split into (hi, lo) words (R/prng.R:130-148). */
    uint32_t x0, x1;
    tf(key[0], key[1], (uint32_t)(i >> 32), (uint32_t)i, &x0, &x1);
    if (bit_width == 64) return ((uint64_t)x0 << 32) | x1;
    const uint32_t x = x0 ^ x1;
    if (bit_width == 32) return x;
    if (bit_width == 16) return (uint16_t)x;
    return (uint8_t)x;
  }
  /* R/prng.R:246-261 */
  if (bit_width == 64) {
    const uint64_t mc = 2 * size;
    return ((uint64_t)original_word(key, mc, i) << 32) | original_word(key, mc, size + i);
  }
  if (bit_width == 32) return original_word(key, size, i);
  const uint64_t per = 32 / (uint64_t)bit_width;
  const uint64_t mc = ((uint64_t)bit_width * size + 31) / 32;
  const uint32_t w = original_word(key, mc, i / per);
  const uint32_t v = w >> (bit_width * (int)(i % per));
  return bit_width == 16 ? (uint16_t)v : (uint8_t)v;
}

/* Bulk partitionable 32-bit words, written so that the compiler vectorises it. */
__attribute__((target_clones("avx512f", "avx2", "default"))) static void bulk_part32(
    uint32_t k0, uint32_t k1, uint64_t begin, uint64_t count, uint32_t* out) {
  const uint32_t ks2 = k0 ^ k1 ^ 0x1BD11BDAu;
  for (uint64_t t = 0; t < count; ++t) {
    const uint64_t i = begin + t;
    uint32_t x0 = (uint32_t)(i >> 32) + k0, x1 = (uint32_t)i + k1;
#define ORC_R(r) x0 += x1; x1 = rotl32(x1, r); x1 ^= x0;
    ORC_R(13) ORC_R(15) ORC_R(26) ORC_R(6)  x0 += k1;  x1 += ks2 + 1u;
    ORC_R(17) ORC_R(29) ORC_R(16) ORC_R(24) x0 += ks2; x1 += k0 + 2u;
    ORC_R(13) ORC_R(15) ORC_R(26) ORC_R(6)  x0 += k0;  x1 += k1 + 3u;
    ORC_R(17) ORC_R(29) ORC_R(16) ORC_R(24) x0 += k1;  x1 += ks2 + 4u;
    ORC_R(13) ORC_R(15) ORC_R(26) ORC_R(6)  x0 += ks2; x1 += k0 + 5u;
#undef ORC_R
    out[t] = x0 ^ x1;
  }
}


int orc_random_bits(const uint32_t key[2], int bit_width, uint64_t size, int partitionable,
                    uint64_t begin, uint64_t count, void* out) {
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64) return 1;
  if (begin > size || count > size - begin) return 2;
  if (partitionable && bit_width == 32) {
    const int64_t chunk = 1 << 16;
    const int64_t nchunks = (int64_t)((count + chunk - 1) / chunk);
    uint32_t* o = (uint32_t*)out;
    ORC_PAR_FOR
    for (int64_t c = 0; c < nchunks; ++c) {
      const uint64_t s = (uint64_t)c * chunk;
      const uint64_t n = count - s < (uint64_t)chunk ? count - s : (uint64_t)chunk;
      bulk_part32(key[0], key[1], begin + s, n, o + s);
    }
    return 0;
  }
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t) {
    const uint64_t v = orc_bits_at(key, bit_width, size, partitionable, begin + (uint64_t)t);
    switch (bit_width) {
      case 64: ((uint64_t*)out)[t] = v; break;
      case 32: ((uint32_t*)out)[t] = (uint32_t)v; break;
      case 16: ((uint16_t*)out)[t] = (uint16_t)v; break;
      default: ((uint8_t*)out)[t] = (uint8_t)v; break;
    }
  }
  return 0;
}

/* ---- 16-bit float helpers -------------------------------------------------------------- */

static inline float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
static inline double bits_f64(uint64_t b) { double d; memcpy(&d, &b, 8); return d; }

/* float -> 16-bit float with round to nearest even.  man = mantissa bits kept (10 for
 * float16, 7 for bfloat16), ebias/emax describe the target exponent. */
static uint16_t f32_to_half_bits(float f, int bf16) {
  const uint32_t b = f32_bits(f);
  if (bf16) {
    if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu)) return (uint16_t)((b >> 16) | 0x40);
    const uint32_t lsb = (b >> 16) & 1u;
    return (uint16_t)((b + 0x7FFFu + lsb) >> 16);
  }
  const _Float16 h = (_Float16)f;
  uint16_t r;
  memcpy(&r, &h, 2);
  return r;
}

static float half_bits_to_f32(uint16_t h, int bf16) {
  if (bf16) return bits_f32((uint32_t)h << 16);
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

/* double -> float rounded to odd, so that a following round to a 16-bit float is a
 * single correct rounding of the double. */
static float f64_to_f32_odd(double x) {
  float f = (float)x;
  if (isfinite(x) && (double)f != x) {
    if (fabs((double)f) > fabs(x)) f = nextafterf(f, 0.0f);
    f = bits_f32(f32_bits(f) | 1u);
  }
  return f;
}

/* One rounding to the 16-bit type of a float computed exactly or with one rounding
 * (f32 has more than 2p+2 bits for both 16-bit types, so double rounding is harmless
 * for a single +, -, *). */
static inline float rh(float f, int bf16) { return half_bits_to_f32(f32_to_half_bits(f, bf16), bf16); }

/* ---- log1p ----------------------------------------------------------------------------- */

static inline double bits_to_f64(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static inline uint64_t f64_to_bits(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

/* Logarithms in double precision after W. J. Cody and W. Waite, "Software Manual for the
 * Elementary Functions" (1980), performing the same operations in the same order as the
 * kernels (jaxr_b200/csrc/samplers.cuh), so both produce the same doubles: t = 2^e m with
 * m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s) = 2 (s + s^3/3 + s^5/5 + ...) with
 * s = (m - 1) / (m + 1), |s| < 0.1716, ten terms, plus a correction term corr added
 * before the exponent part.  t = 0 gives -inf, t < 0 or NaN NaN, t = inf inf.  Within
 * 2 ulp of correctly rounded results. */
static double log_core(double t, double corr) {
  const uint64_t b64 = f64_to_bits(t);
  const uint32_t hi = (uint32_t)(b64 >> 32), mh = hi & 0x000FFFFFu;
  const int big = mh >= 0x6A09Eu; /* mantissa >= sqrt(2): use m / 2 */
  const int e = (int)((hi >> 20) & 0x7FFu) - 1023 + big;
  const double m =
      bits_to_f64(((uint64_t)(mh | ((big ? 1022u : 1023u) << 20)) << 32) | (b64 & 0xFFFFFFFFull));
  const double a = m - 1.0, b = m + 1.0;
  double r = (double)(1.0f / (float)b); /* 1 / b to float precision, then two Newton steps */
  r = fma(r, fma(-b, r, 1.0), r);
  const double s0 = a * r;
  const double s = fma(r, fma(-b, s0, a), s0);
  const double z = s * s;
  double p = 0x1.8618618618618p-5; /* 1/21 */
  p = fma(p, z, 0x1.af286bca1af28p-5); /* 1/19 */
  p = fma(p, z, 0x1.e1e1e1e1e1e1ep-5); /* 1/17 */
  p = fma(p, z, 0x1.1111111111111p-4); /* 1/15 */
  p = fma(p, z, 0x1.3b13b13b13b14p-4); /* 1/13 */
  p = fma(p, z, 0x1.745d1745d1746p-4); /* 1/11 */
  p = fma(p, z, 0x1.c71c71c71c71cp-4); /* 1/9 */
  p = fma(p, z, 0x1.2492492492492p-3); /* 1/7 */
  p = fma(p, z, 0x1.999999999999ap-3); /* 1/5 */
  p = fma(p, z, 0x1.5555555555555p-2); /* 1/3 */
  const double s2 = s + s;
  const double lm = fma(s2 * z, p, s2);
  const double LN2_HI = 0x1.62e42fefa3800p-1, LN2_LO = 0x1.ef35793c76730p-45;
  double res = fma((double)e, LN2_HI, fma((double)e, LN2_LO, lm + corr));
  if (!(t > 0.0)) res = (t == 0.0) ? -INFINITY : NAN;
  if (t == INFINITY) res = INFINITY;
  return res;
}

/* log1p(y) for y <= 0 (and NaN), the argument erf_inv gives it (y = -x*x): t = 1 + y and
 * the rounding error of that sum added back as (y - (t - 1)) / t. */
static double log1p_neg(double y) {
  const double t = 1.0 + y;
  const double corr = (y - (t - 1.0)) * (double)(1.0f / (float)t);
  return log_core(t, corr);
}

/* log(x) for x > 0. */
static double log_pos(double x) { return log_core(x, 0.0); }

double orc_log1p_neg(double y) { return log1p_neg(y); }
double orc_log_pos(double x) { return log_pos(x); }

/* ---- erf_inv --------------------------------------------------------------------------- */

/* Giles (2011), single precision: two polynomials in w = -log(1 - x^2), split at w = 5. */
static const float GS_LT5[9] = {2.81022636e-08f, 3.43273939e-07f, -3.5233877e-06f,
                                -4.39150654e-06f, 0.00021858087f, -0.00125372503f,
                                -0.00417768164f, 0.246640727f, 1.50140941f};
static const float GS_GE5[9] = {-0.000200214257f, 0.000100950558f, 0.00134934322f,
                                -0.00367342844f, 0.00573950773f, -0.0076224613f,
                                0.00943887047f, 1.00167406f, 2.83297682f};

/* ---- accurate erf_inv (jax_accurate_erf_inv; R/lax_special.R:1022-1082) ---------------
 *
 * erf_inv_core(x, q = 1 - |x|) without the far-tail pieces: w = -log(q (1 + |x|)).  Below
 * the first split (float32 w < 3.5, float64 w < 4.5) the result is x * P(w - c1); above
 * it z = sqrt(w) is carried as z_h (the top half of its mantissa, so z_h^2 is exact) plus
 * z_l = (w - z_h^2) / (z + z_h), and the result is sign(x) (z_h + (z_l + P(z - shift))).
 * The polynomials are JAX's Sollya fits as the reference holds them (erfinv_tables.h),
 * evaluated by Horner from the highest coefficient down.  |x| > 1 or NaN gives NaN,
 * |x| = 1 gives x * inf. */
static const float EA32_P1[JXR_ERFINV32_P1_N] = {JXR_ERFINV32_P1};
static const float EA32_P2[JXR_ERFINV32_P2_N] = {JXR_ERFINV32_P2};
static const double EA64_P1[JXR_ERFINV64_P1_N] = {JXR_ERFINV64_P1};
static const double EA64_P2[JXR_ERFINV64_P2_N] = {JXR_ERFINV64_P2};
static const double EA64_P3[JXR_ERFINV64_P3_N] = {JXR_ERFINV64_P3};

static float erfinv_accurate_f32(float x, int fused) {
  const float ax = fabsf(x);
  if (!(ax <= 1.0f)) return NAN;
  if (ax == 1.0f) return x * INFINITY;
  const float q = 1.0f - ax;
  const float arg = q * (1.0f + ax);
  const float w = -(float)log_pos((double)arg); /* the logarithm rounded once */
  const int first = w < 3.5f;
  const float w_safe = first ? 1.0f : w;
  const float z = sqrtf(w_safe);
  uint32_t zb;
  memcpy(&zb, &z, 4);
  zb &= 0xFFFFF000u;
  float z_h;
  memcpy(&z_h, &zb, 4);
  const float z_l = (w_safe - z_h * z_h) / (z + z_h);
  const float t = first ? w - 1.75f : z - 3.0f;
  const float* c = first ? EA32_P1 : EA32_P2;
  float p = c[JXR_ERFINV32_P1_N - 1];
  for (int i = JXR_ERFINV32_P1_N - 2; i >= 0; --i) p = fused ? fmaf(p, t, c[i]) : p * t + c[i];
  if (first) return x * p;
  const float mag = z_h + (z_l + p);
  return x < 0.0f ? -mag : mag;
}

static double erfinv_accurate_f64(double x, int fused) {
  const double ax = fabs(x);
  if (!(ax <= 1.0)) return NAN;
  if (ax == 1.0) return x * INFINITY;
  const double q = 1.0 - ax;
  const double w = -log_pos(q * (1.0 + ax));
  const int piece = (w < 4.5) ? 0 : (w < 16.0) ? 1 : 2;
  const double w_safe = piece == 0 ? 1.0 : w;
  const double z = sqrt(w_safe);
  uint64_t zb;
  memcpy(&zb, &z, 8);
  zb &= 0xFFFFFFFFF8000000ull;
  double z_h;
  memcpy(&z_h, &zb, 8);
  const double z_l = (w_safe - z_h * z_h) / (z + z_h);
  const double shift = piece == 1 ? 3.0 : 5.0;
  const double t = piece == 0 ? w - 2.25 : z - shift;
  const double* c = piece == 0 ? EA64_P1 : piece == 1 ? EA64_P2 : EA64_P3;
  double p = c[JXR_ERFINV64_P1_N - 1];
  for (int i = JXR_ERFINV64_P1_N - 2; i >= 0; --i) p = fused ? fma(p, t, c[i]) : p * t + c[i];
  if (piece == 0) return x * p;
  const double mag = z_h + (z_l + p);
  return x < 0.0 ? -mag : mag;
}

float orc_erfinv_f32(float x, int fma) {
  if (fma & ORC_ERFINV_ACCURATE) return erfinv_accurate_f32(x, fma & 1);
  /* log1p of the rounded float -(x*x), evaluated in double and rounded once */
  const float w0 = -(float)log1p_neg((double)(-(x * x)));
  const int lt = w0 < 5.0f;
  const float* c = lt ? GS_LT5 : GS_GE5;
  const float w = lt ? w0 - 2.5f : sqrtf(w0) - 3.0f;
  float p = c[0];
  for (int i = 1; i < 9; ++i) p = fma ? fmaf(p, w, c[i]) : c[i] + p * w;
  if (fabsf(x) == 1.0f) return x * INFINITY;
  return p * x;
}

/* Giles (2011), double precision: three polynomials split at w = 6.25 and w = 16. */
static const double GD_LT625[23] = {
    -3.6444120640178196996e-21, -1.685059138182016589e-19, 1.2858480715256400167e-18,
    1.115787767802518096e-17,   -1.333171662854620906e-16, 2.0972767875968561637e-17,
    6.6376381343583238325e-15,  -4.0545662729752068639e-14, -8.1519341976054721522e-14,
    2.6335093153082322977e-12,  -1.2975133253453532498e-11, -5.4154120542946279317e-11,
    1.051212273321532285e-09,   -4.1126339803469836976e-09, -2.9070369957882005086e-08,
    4.2347877827932403518e-07,  -1.3654692000834678645e-06, -1.3882523362786468719e-05,
    0.0001867342080340571352,   -0.00074070253416626697512, -0.0060336708714301490533,
    0.24015818242558961693,     1.6536545626831027356};
static const double GD_LT16[19] = {
    2.2137376921775787049e-09,  9.0756561938885390979e-08,  -2.7517406297064545428e-07,
    1.8239629214389227755e-08,  1.5027403968909827627e-06,  -4.013867526981545969e-06,
    2.9234449089955446044e-06,  1.2475304481671778723e-05,  -4.7318229009055733981e-05,
    6.8284851459573175448e-05,  2.4031110387097893999e-05,  -0.0003550375203628474796,
    0.00095328937973738049703,  -0.0016882755560235047313, 0.0024914420961078508066,
    -0.0037512085075692412107, 0.005370914553590063617,   1.0052589676941592334,
    3.0838856104922207635};
static const double GD_GE16[17] = {
    -2.7109920616438573243e-11, -2.5556418169965252055e-10, 1.5076572693500548083e-09,
    -3.7894654401267369937e-09, 7.6157012080783393804e-09,  -1.4960026627149240478e-08,
    2.9147953450901080826e-08,  -6.7711997758452339498e-08, 2.2900482228026654717e-07,
    -9.9298272942317002539e-07, 4.5260625972231537039e-06,  -1.9681778105531670567e-05,
    7.5995277030017761139e-05,  -0.00021503011930044477347, -0.00013871931833623122026,
    1.0103004648645343977,      4.8499064014085844221};

double orc_erfinv_f64(double x, int fma_) {
  if (fma_ & ORC_ERFINV_ACCURATE) return erfinv_accurate_f64(x, fma_ & 1);
  const double w0 = -log1p_neg(-(x * x));
  const double* c;
  int n;
  double w;
  if (w0 < 6.25) {
    c = GD_LT625; n = 23; w = w0 - 3.125;
  } else if (w0 < 16.0) {
    c = GD_LT16; n = 19; w = sqrt(w0) - 3.25;
  } else {
    c = GD_GE16; n = 17; w = sqrt(w0) - 5.0;
  }
  double p = c[0];
  for (int i = 1; i < n; ++i) p = fma_ ? fma(p, w, c[i]) : c[i] + p * w;
  if (fabs(x) == 1.0) return x * INFINITY;
  return p * x;
}

void orc_erfinv_arr(const void* x, int64_t n, int dtype, int fma_, void* out) {
  ORC_PAR_FOR
  for (int64_t i = 0; i < n; ++i) {
    if (dtype == ORC_F32) ((float*)out)[i] = orc_erfinv_f32(((const float*)x)[i], fma_);
    else ((double*)out)[i] = orc_erfinv_f64(((const double*)x)[i], fma_);
  }
}

/* ---- samplers -------------------------------------------------------------------------- */

static inline double xla_max(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}

/* R/random.R:288-304: bits >> (nbits - nmant) | bits(1.0), bitcast, - 1, then
 * floats * (maxval - minval) + minval and max(minval, .), all in the target dtype. */
double orc_uniform_at(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                      double minval, double maxval, int mul_add_fma, uint64_t i) {
  switch (dtype) {
    case ORC_F32: {
      const uint32_t b = (uint32_t)orc_bits_at(key, 32, size, partitionable, i);
      const float f = bits_f32((b >> 9) | 0x3F800000u) - 1.0f;
      const float mn = (float)minval, mx = (float)maxval;
      const float d = mx - mn;
      const float r = mul_add_fma ? fmaf(f, d, mn) : f * d + mn;
      return (float)xla_max(mn, r);
    }
    case ORC_F64: {
      const uint64_t b = orc_bits_at(key, 64, size, partitionable, i);
      const double f = bits_f64((b >> 12) | 0x3FF0000000000000ull) - 1.0;
      const double d = maxval - minval;
      const double r = mul_add_fma ? fma(f, d, minval) : f * d + minval;
      return xla_max(minval, r);
    }
    case ORC_F16:
    case ORC_BF16: {
      const int bf = dtype == ORC_BF16;
      /* float16: 16 random bits, shift 6, one = 0x3C00; bfloat16: 8 random bits
       * widened to 16, shift 1, one = 0x3F80 (nmant < 8 uses 8-bit draws). */
      const uint32_t b = (uint32_t)orc_bits_at(key, bf ? 8 : 16, size, partitionable, i);
      const uint16_t fb = bf ? (uint16_t)((b >> 1) | 0x3F80u) : (uint16_t)((b >> 6) | 0x3C00u);
      const float f = rh(half_bits_to_f32(fb, bf) - 1.0f, bf);
      const float mn = rh(f64_to_f32_odd(minval), bf), mx = rh(f64_to_f32_odd(maxval), bf);
      const float d = rh(mx - mn, bf);
      /* fused: the exact f * d + mn (22-bit product, in double) rounded once */
      const float r = mul_add_fma ? rh(f64_to_f32_odd((double)f * (double)d + (double)mn), bf)
                                  : rh(rh(f * d, bf) + mn, bf);
      return xla_max(mn, r);
    }
  }
  return NAN;
}

/* R/random.R:502-508: u = uniform(lo = nextafter(-1, 0), hi = 1), sqrt(2) * erf_inv(u). */
double orc_normal_at(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                     int erfinv_fma, uint64_t i) {
  switch (dtype) {
    case ORC_F32: {
      const float u = (float)orc_uniform_at(key, ORC_F32, size, partitionable,
                                            -1.0 + 0x1p-24, 1.0, 0, i);
      return (float)1.41421356237309504880 * orc_erfinv_f32(u, erfinv_fma);
    }
    case ORC_F64: {
      const double u = orc_uniform_at(key, ORC_F64, size, partitionable, -1.0 + 0x1p-53, 1.0,
                                      0, i);
      return 1.41421356237309504880 * orc_erfinv_f64(u, erfinv_fma);
    }
    case ORC_F16:
    case ORC_BF16: {
      const int bf = dtype == ORC_BF16;
      const double lo = bf ? -1.0 + 0x1p-8 : -1.0 + 0x1p-11;
      const float u = (float)orc_uniform_at(key, dtype, size, partitionable, lo, 1.0, 0, i);
      /* erf_inv of a 16-bit float is evaluated in float32 and rounded back. */
      const float e = rh(orc_erfinv_f32(u, erfinv_fma), bf);
      return rh(rh((float)1.41421356237309504880, bf) * e, bf);
    }
  }
  return NAN;
}

static void store_float(void* out, int dtype, int64_t t, double v) {
  switch (dtype) {
    case ORC_F32: ((float*)out)[t] = (float)v; break;
    case ORC_F64: ((double*)out)[t] = v; break;
    default: ((uint16_t*)out)[t] = f32_to_half_bits((float)v, dtype == ORC_BF16); break;
  }
}

int orc_uniform(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                double minval, double maxval, int mul_add_fma, uint64_t begin,
                uint64_t count, void* out) {
  if (dtype < ORC_F32 || dtype > ORC_BF16) return 1;
  if (begin > size || count > size - begin) return 2;
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t)
    store_float(out, dtype, t,
                orc_uniform_at(key, dtype, size, partitionable, minval, maxval, mul_add_fma,
                               begin + (uint64_t)t));
  return 0;
}

int orc_normal(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
               int erfinv_fma, uint64_t begin, uint64_t count, void* out) {
  if (dtype < ORC_F32 || dtype > ORC_BF16) return 1;
  if (begin > size || count > size - begin) return 2;
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t)
    store_float(out, dtype, t,
                orc_normal_at(key, dtype, size, partitionable, erfinv_fma, begin + (uint64_t)t));
  return 0;
}

/* R/random.R:656-666, mode "low": uniform(key, shape, dtype(p)) < p. */
int orc_bernoulli(const uint32_t key[2], int p_dtype, double p, uint64_t size,
                  int partitionable, uint64_t begin, uint64_t count, uint8_t* out) {
  if (p_dtype < ORC_F32 || p_dtype > ORC_BF16) return 1;
  if (begin > size || count > size - begin) return 2;
  double pc = p;
  if (p_dtype == ORC_F32) pc = (float)p;
  if (p_dtype == ORC_F16 || p_dtype == ORC_BF16) pc = rh(f64_to_f32_odd(p), p_dtype == ORC_BF16);
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t)
    out[t] = orc_uniform_at(key, p_dtype, size, partitionable, 0.0, 1.0, 0,
                            begin + (uint64_t)t) < pc;
  return 0;
}

/* ---- log-transform samplers (R/random.R:1422-1516) ------------------------------------- */

/* u = uniform(lo, 1) in dtype (fused multiply-add, as the recorded samples have it), then
 * exponential -log1p(-u) (:1431-1434), gumbel mode "low" -log(-log(u)) (:1488), logistic
 * log(u) - log1p(-u) (:1512-1515), laplace sign(u) log1p(-|u|) (:1500-1504), with
 * lo = 0, tiny, tiny, -1 + 2^-(nmant+1).  Each float operation is rounded to the dtype
 * once; 16-bit dtypes evaluate each function in float32 and round the result to 16 bits,
 * as XLA does. */
double orc_sample_at(const uint32_t key[2], int kind, int dtype, uint64_t size,
                     int partitionable, uint64_t i) {
  switch (dtype) {
    case ORC_F32: {
      const double lo = kind == ORC_EXPONENTIAL ? 0.0
                        : kind == ORC_LAPLACE   ? -1.0 + 0x1p-24
                                                : 0x1p-126;
      const float u = (float)orc_uniform_at(key, ORC_F32, size, partitionable, lo, 1.0, 1, i);
      switch (kind) {
        case ORC_EXPONENTIAL: return -(float)log1p_neg(-(double)u);
        case ORC_GUMBEL: {
          const float a = (float)log_pos((double)u);
          return -(float)log_pos(-(double)a);
        }
        case ORC_LOGISTIC: {
          const float a = (float)log_pos((double)u);
          const float c = (float)log1p_neg(-(double)u);
          return (float)(a - c);
        }
        default: {
          const float l = (float)log1p_neg(-(double)fabsf(u));
          return u < 0.0f ? -l : l;
        }
      }
    }
    case ORC_F64: {
      const double lo = kind == ORC_EXPONENTIAL ? 0.0
                        : kind == ORC_LAPLACE   ? -1.0 + 0x1p-53
                                                : 0x1p-1022;
      const double u = orc_uniform_at(key, ORC_F64, size, partitionable, lo, 1.0, 1, i);
      switch (kind) {
        case ORC_EXPONENTIAL: return -log1p_neg(-u);
        case ORC_GUMBEL: return -log_pos(-log_pos(u));
        case ORC_LOGISTIC: return log_pos(u) - log1p_neg(-u);
        default: {
          const double l = log1p_neg(-fabs(u));
          return u < 0.0 ? -l : l;
        }
      }
    }
    case ORC_F16:
    case ORC_BF16: {
      const int bf = dtype == ORC_BF16;
      const double tiny = bf ? 0x1p-126 : 0x1p-14;
      const double lo = kind == ORC_EXPONENTIAL ? 0.0
                        : kind == ORC_LAPLACE   ? -1.0 + (bf ? 0x1p-8 : 0x1p-11)
                                                : tiny;
      const float u = (float)orc_uniform_at(key, dtype, size, partitionable, lo, 1.0, 1, i);
#define LG(v) rh((float)(v), bf)
      switch (kind) {
        case ORC_EXPONENTIAL: return -LG(log1p_neg(-(double)u));
        case ORC_GUMBEL: return -LG(log_pos(-(double)LG(log_pos((double)u))));
        case ORC_LOGISTIC: return rh(LG(log_pos((double)u)) - LG(log1p_neg(-(double)u)), bf);
        default: {
          const float l = LG(log1p_neg(-(double)fabsf(u)));
          return u < 0.0f ? -l : l;
        }
      }
#undef LG
    }
  }
  return NAN;
}

int orc_sample(const uint32_t key[2], int kind, int dtype, uint64_t size, int partitionable,
               uint64_t begin, uint64_t count, void* out) {
  if (dtype < ORC_F32 || dtype > ORC_BF16) return 1;
  if (kind < ORC_EXPONENTIAL || kind > ORC_LAPLACE) return 1;
  if (begin > size || count > size - begin) return 2;
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t)
    store_float(out, dtype, t,
                orc_sample_at(key, kind, dtype, size, partitionable, begin + (uint64_t)t));
  return 0;
}

/* The float32 samplers of given 32-bit draws (each float32 sample depends only on
 * bits >> 9), for exhaustive checks over all 2^23 draws: kind 0..3 the log-transform
 * samplers as orc_sample_at evaluates them (R/random.R:1428-1516), 4 the normal as
 * orc_normal_at does (R/random.R:501-508, fused Horner steps). */
static float unit_f32_of(uint32_t b) { return bits_f32((b >> 9) | 0x3F800000u) - 1.0f; }

void orc_sample_f32_from_bits(const uint32_t* bits, int64_t n, int kind, float* out) {
  ORC_PAR_FOR
  for (int64_t t = 0; t < n; ++t) {
    const float f = unit_f32_of(bits[t]);
    if (kind == 4) {
      const float lo = (float)(-1.0 + 0x1p-24);
      const float u = (float)xla_max(lo, f * 2.0f + lo);
      out[t] = (float)1.41421356237309504880 * orc_erfinv_f32(u, 1);
      continue;
    }
    const float mn = kind == ORC_EXPONENTIAL ? 0.0f
                     : kind == ORC_LAPLACE   ? (float)(-1.0 + 0x1p-24)
                                             : 0x1p-126f;
    const float d = 1.0f - mn;
    const float u = (float)xla_max(mn, fmaf(f, d, mn));
    switch (kind) {
      case ORC_EXPONENTIAL: out[t] = -(float)log1p_neg(-(double)u); break;
      case ORC_GUMBEL: {
        const float a = (float)log_pos((double)u);
        out[t] = -(float)log_pos(-(double)a);
        break;
      }
      case ORC_LOGISTIC: {
        const float a = (float)log_pos((double)u);
        const float c = (float)log1p_neg(-(double)u);
        out[t] = a - c;
        break;
      }
      default: {
        const float l = (float)log1p_neg(-(double)fabsf(u));
        out[t] = u < 0.0f ? -l : l;
      }
    }
  }
}

/* ---- gumbel modes "high" and "highest" (R/random.R:1465-1489) ------------------------- */

/* XLA shifts: amounts of 32 or more give 0. */
static inline uint32_t xshl(uint32_t x, uint32_t s) { return s >= 32u ? 0u : x << s; }
static inline uint32_t xshr(uint32_t x, uint32_t s) { return s >= 32u ? 0u : x >> s; }
static inline uint32_t clz32(uint32_t x) { return x ? (uint32_t)__builtin_clz(x) : 32u; }

/* R/random.R:1446-1462: u32 pair (hi, lo) to a float32 in (0, 1). */
static float safe_int_to_float(uint32_t hi, uint32_t lo) {
  const uint32_t hiclz = clz32(hi), loclz = clz32(lo);
  uint32_t mant = xshl(hi, hiclz) | (hiclz == 32u ? xshl(lo, loclz) : xshr(lo, 32u - hiclz));
  mant = xshr(mant, 32u - 23u - 1u) & ((1u << 23) - 1u);
  uint32_t ex = xshl(126u - (hiclz == 32u ? 32u + loclz : hiclz), 23u);
  ex &= (1u << 30) - (1u << 22);
  return bits_f32(ex | mant);
}

/* Element i of random_gumbel(key, (size), dtype, mode): mode 0 "high", 1 "highest" (float32;
 * other dtypes take "high").  Both draw a (2, size) array: row r of element i is linear
 * index r * size + i. */
double orc_gumbel_mode_at(const uint32_t key[2], int mode, int dtype, uint64_t size,
                          int partitionable, uint64_t i) {
  const uint64_t n2 = 2 * size;
  if (mode == 1 && dtype == ORC_F32) {
    const uint32_t b0 = (uint32_t)orc_bits_at(key, 32, n2, partitionable, i);
    const uint32_t b1 = (uint32_t)orc_bits_at(key, 32, n2, partitionable, size + i);
    uint32_t n0 = ~b0, n1 = ~b1;
    n0 += (n1 == 0xFFFFFFFFu) ? 1u : 0u; /* carry of the 64-bit negation */
    n1 += 1u;
    const int flip = b0 < 0x80000000u;
    const float x = flip ? safe_int_to_float(b0, b1) : safe_int_to_float(n0, n1);
    if (flip) return -(float)log_pos(-(double)(float)log1p_neg(-(double)x));
    return -(float)log_pos(-(double)(float)log_pos((double)x));
  }
  switch (dtype) {
    case ORC_F32: {
      const float h = (float)orc_uniform_at(key, ORC_F32, n2, partitionable, 0.0, 1.0, 1, i);
      const float l = (float)orc_uniform_at(key, ORC_F32, n2, partitionable, 0.0, 1.0, 1, size + i);
      const float x = h >= 0.5f ? h : (h + 0x1p-23f * l) + 0x1p-47f;
      return -(float)log_pos(-(double)(float)log1p_neg(-(double)x));
    }
    case ORC_F64: {
      const double h = orc_uniform_at(key, ORC_F64, n2, partitionable, 0.0, 1.0, 1, i);
      const double l = orc_uniform_at(key, ORC_F64, n2, partitionable, 0.0, 1.0, 1, size + i);
      const double x = h >= 0.5 ? h : (h + 0x1p-52 * l) + 0x1p-105;
      return -log_pos(-log1p_neg(-x));
    }
    default: {
      const int bf = dtype == ORC_BF16;
      const float h = (float)orc_uniform_at(key, dtype, n2, partitionable, 0.0, 1.0, 1, i);
      const float l = (float)orc_uniform_at(key, dtype, n2, partitionable, 0.0, 1.0, 1, size + i);
      /* 2^-nmant low + max(2^-(2 nmant + 1), tiny), each operation rounded to 16 bits */
      const float c = bf ? 0x1p-15f : 0x1p-14f;
      const float x = h >= 0.5f ? h : rh(rh(h + rh((bf ? 0x1p-7f : 0x1p-10f) * l, bf), bf) + c, bf);
      const float a = rh((float)log1p_neg(-(double)x), bf);
      return -rh((float)log_pos(-(double)a), bf);
    }
  }
}

/* ---- truncated normal (R/random.R:586-603) -------------------------------------------- */

/* the 16-bit float after the 16-bit value x toward +inf (up) or -inf */
static float half_step(float x, int up, int bf) {
  uint16_t b = f32_to_half_bits(x, bf);
  const uint16_t inf = bf ? 0x7F80u : 0x7C00u;
  if (isnan(x) || b == (up ? inf : (uint16_t)(0x8000u | inf))) return x;
  if ((b & 0x7FFFu) == 0) b = up ? 0x0001u : 0x8001u; /* +-0: the smallest subnormal */
  else if (up == !(b & 0x8000u)) b = (uint16_t)(b + 1); /* away from zero */
  else b = (uint16_t)(b - 1);
  return half_bits_to_f32(b, bf);
}

/* Element i of random_truncated_normal(key, lower, upper, (size), dtype), scalar bounds:
 * a = erf(lower / sqrt2), b = erf(upper / sqrt2) in dtype (erf from libm, rounded),
 * u = uniform(a, b) (fused multiply-add), sqrt2 * erf_inv(u) (fused Horner), clipped to
 * [nextafter(lower, inf), nextafter(upper, -inf)]. */
double orc_truncated_normal_at(const uint32_t key[2], int dtype, uint64_t size,
                               int partitionable, double lower, double upper, int erfinv_mode,
                               uint64_t i) {
  switch (dtype) {
    case ORC_F32: {
      const float s2 = 1.41421356237309504880f, lo = (float)lower, hi = (float)upper;
      const float a = (float)erf((double)(lo / s2)), b = (float)erf((double)(hi / s2));
      const float u = (float)orc_uniform_at(key, ORC_F32, size, partitionable, a, b, 1, i);
      const float x = s2 * orc_erfinv_f32(u, erfinv_mode);
      const float cl = nextafterf(lo, INFINITY), ch = nextafterf(hi, -INFINITY);
      const float m = isnan(x) ? x : (cl >= x ? cl : x);
      return isnan(m) ? m : (ch <= m ? ch : m);
    }
    case ORC_F64: {
      const double s2 = 1.41421356237309504880;
      const double a = erf(lower / s2), b = erf(upper / s2);
      const double u = orc_uniform_at(key, ORC_F64, size, partitionable, a, b, 1, i);
      const double x = s2 * orc_erfinv_f64(u, erfinv_mode);
      const double cl = nextafter(lower, INFINITY), ch = nextafter(upper, -INFINITY);
      const double m = isnan(x) ? x : (cl >= x ? cl : x);
      return isnan(m) ? m : (ch <= m ? ch : m);
    }
    default: {
      const int bf = dtype == ORC_BF16;
      const float s2 = rh(f64_to_f32_odd(1.41421356237309504880), bf);
      const float lo = rh(f64_to_f32_odd(lower), bf), hi = rh(f64_to_f32_odd(upper), bf);
      const float a = rh((float)erf((double)rh(lo / s2, bf)), bf);
      const float b = rh((float)erf((double)rh(hi / s2, bf)), bf);
      const float u = (float)orc_uniform_at(key, dtype, size, partitionable, a, b, 1, i);
      const float e = rh(orc_erfinv_f32(u, erfinv_mode), bf);
      const float x = rh(s2 * e, bf);
      const float cl = half_step(lo, 1, bf), ch = half_step(hi, 0, bf);
      const float m = isnan(x) ? x : (cl >= x ? cl : x);
      return isnan(m) ? m : (ch <= m ? ch : m);
    }
  }
}

int orc_gumbel_mode(const uint32_t key[2], int mode, int dtype, uint64_t size,
                    int partitionable, void* out) {
  if (dtype < ORC_F32 || dtype > ORC_BF16) return 1;
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)size; ++t)
    store_float(out, dtype, t, orc_gumbel_mode_at(key, mode, dtype, size, partitionable, (uint64_t)t));
  return 0;
}

int orc_truncated_normal(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                         double lower, double upper, int erfinv_mode, uint64_t begin,
                         uint64_t count, void* out) {
  if (dtype < ORC_F32 || dtype > ORC_BF16) return 1;
  if (begin > size || count > size - begin) return 2;
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t)
    store_float(out, dtype, t,
                orc_truncated_normal_at(key, dtype, size, partitionable, lower, upper,
                                        erfinv_mode, begin + (uint64_t)t));
  return 0;
}

/* ---- rbg / unsafe_rbg: XLA's RngBitGenerator (R/prng.R:264-426) ----------------------- */

/* Philox4x32-10 (Salmon, Moraes, Dror and Shaw, SC'11): out = the block of counter c under
 * key k. */
void orc_philox4x32(const uint32_t c[4], const uint32_t k[2], uint32_t out[4]) {
  uint32_t c0 = c[0], c1 = c[1], c2 = c[2], c3 = c[3], k0 = k[0], k1 = k[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    c0 = n0;
    c1 = (uint32_t)p1;
    c2 = n2;
    c3 = (uint32_t)p0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

/* Block b of the stream of the u32[4] key q: Philox key (q0, q1), counter = q as a 128-bit
 * number (q0 lowest) + b.  This is how the recorded rbg values of the reference
 * (tests/testthat/test-prng.R:48-54) come out of XLA's RngBitGenerator. */
static void rbg_block(const uint32_t q[4], uint64_t b, uint32_t out[4]) {
  const uint64_t lo = (uint64_t)q[1] << 32 | q[0], hi = (uint64_t)q[3] << 32 | q[2];
  const uint64_t l2 = lo + b, h2 = hi + (l2 < lo);
  const uint32_t c[4] = {(uint32_t)l2, (uint32_t)(l2 >> 32), (uint32_t)h2, (uint32_t)(h2 >> 32)};
  const uint32_t k[2] = {q[0], q[1]};
  orc_philox4x32(c, k, out);
}

/* Elements [begin, begin + count) of lax_rng_bit_generator(key, (size), uint<bits>): element
 * e of a 32-bit request is word e % 4 of block e / 4; 8/16-bit elements are the low bits of
 * the 32-bit element; 64-bit element e is words 2(e % 2), 2(e % 2) + 1 (low first) of block
 * e / 2. */
int orc_rbg_bits(const uint32_t q[4], int bit_width, uint64_t size, uint64_t begin,
                 uint64_t count, void* out) {
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64) return 1;
  if (begin > size || count > size - begin) return 2;
  ORC_PAR_FOR
  for (int64_t t = 0; t < (int64_t)count; ++t) {
    const uint64_t e = begin + (uint64_t)t;
    uint32_t w[4];
    if (bit_width == 64) {
      rbg_block(q, e / 2, w);
      ((uint64_t*)out)[t] = (uint64_t)w[2 * (e % 2)] | (uint64_t)w[2 * (e % 2) + 1] << 32;
    } else {
      rbg_block(q, e / 4, w);
      const uint32_t v = w[e % 4];
      if (bit_width == 8) ((uint8_t*)out)[t] = (uint8_t)v;
      else if (bit_width == 16) ((uint16_t*)out)[t] = (uint16_t)v;
      else ((uint32_t*)out)[t] = v;
    }
  }
  return 0;
}

/* unsafe_rbg split (R/prng.R:415-420): key i = row 10 i of the (10 num, 4) request. */
void orc_rbg_unsafe_split(const uint32_t q[4], int64_t num, uint32_t* out) {
  for (int64_t i = 0; i < num; ++i) rbg_block(q, 10 * (uint64_t)i, out + 4 * i);
}

/* unsafe_rbg fold_in (R/prng.R:423-426): key ^ row 9 of the (10, 4) request of the key
 * rbg_seed(data) = threefry_seed(data) twice = (0, data, 0, data). */
void orc_rbg_unsafe_fold_in(const uint32_t q[4], uint32_t data, uint32_t out[4]) {
  const uint32_t s[4] = {0u, data, 0u, data};
  uint32_t w[4];
  rbg_block(s, 9, w);
  for (int i = 0; i < 4; ++i) out[i] = q[i] ^ w[i];
}
