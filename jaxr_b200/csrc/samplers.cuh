// Bits -> float transforms of jaxR's samplers, fused into the cipher kernels.
//
//   uniform   R/random.R:287-304  bits >> (nbits - nmant) | bits(1.0), bitcast, - 1,
//                                 floats * (maxval - minval) + minval, max(minval, .)
//   normal    R/random.R:501-508  sqrt(2) * erf_inv(uniform(nextafter(-1, 0), 1))
//   bernoulli R/random.R:655-666  uniform(dtype(p)) < p
//   erf_inv   R/lax.R:222 lowered to chlo.erf_inv (R/lax_special.R:1327-1331): M. Giles,
//             "Approximating the erfinv function", GPU Computing Gems Jade (2011), with
//             w = -log1p(-x*x) and erf_inv(+-1) = +-inf.
//
// Every float operation is an explicitly rounded intrinsic (__fmul_rn, __fadd_rn,
// __fmaf_rn ...), so compiler contraction cannot change a result.  Where the
// reference's recorded samples show fused multiply-adds (the uniform's affine map,
// test-random.R:43 and :160; the erf_inv Horner steps), __fmaf_rn/__fma_rn is used.
// The float32 erf_inv takes log1p of the rounded float -(x*x) in double precision
// (log1p_neg) and rounds it to float, which reproduces every float32 normal the
// reference recorded.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "erfinv_tables.h"
#include "log_table.h"

namespace jxr {

// lax_max(a, b) as XLA's CPU code computes it: NaN-propagating, `a` on ties.
__device__ __forceinline__ float xla_max(float a, float b) { return (a >= b || a != a) ? a : b; }
__device__ __forceinline__ double xla_max(double a, double b) {
  return (a >= b || a != a) ? a : b;
}
// lax_min likewise.
__device__ __forceinline__ float xla_min(float a, float b) { return (a <= b || a != a) ? a : b; }
__device__ __forceinline__ double xla_min(double a, double b) {
  return (a <= b || a != a) ? a : b;
}

// ---- log1p -----------------------------------------------------------------------------

// Logarithms in double precision, branch-free, after W. J. Cody and W. Waite, "Software
// Manual for the Elementary Functions" (1980): t = 2^e m with m in [sqrt(1/2), sqrt(2)),
// log m = 2 atanh(s) = 2 (s + s^3/3 + s^5/5 + ...) with s = (m - 1) / (m + 1),
// |s| < 0.1716, ten terms.  Within 2 ulp of correctly rounded results.  The CPU oracle
// performs the same operations in the same order, so both produce the same doubles.
// log of t > 0 after Cody and Waite, plus a small correction term added before the
// exponent part; shared by log1p_neg and log_pos.  t = 0 gives -inf, t < 0 or NaN NaN,
// t = inf inf; t is a normal number in every use here (>= the float32 tiny).
__device__ __forceinline__ double log_core(double t, double corr) {
  const unsigned long long b64 = (unsigned long long)__double_as_longlong(t);
  const uint32_t hi = (uint32_t)(b64 >> 32), mh = hi & 0x000FFFFFu;
  const bool big = mh >= 0x6A09Eu;  // mantissa >= sqrt(2): use m / 2
  const int e = (int)((hi >> 20) & 0x7FFu) - 1023 + (big ? 1 : 0);
  const double m = __longlong_as_double(
      (long long)((((unsigned long long)(mh | ((big ? 1022u : 1023u) << 20))) << 32) |
                  (b64 & 0xFFFFFFFFull)));
  const double a = __dsub_rn(m, 1.0), b = __dadd_rn(m, 1.0);
  double r = (double)__frcp_rn(__double2float_rn(b));  // 1 / b to float precision
  r = __fma_rn(r, __fma_rn(-b, r, 1.0), r);            // and two Newton steps
  const double s0 = __dmul_rn(a, r);
  const double s = __fma_rn(r, __fma_rn(-b, s0, a), s0);
  const double z = __dmul_rn(s, s);
  double p = 0x1.8618618618618p-5;          // 1/21
  p = __fma_rn(p, z, 0x1.af286bca1af28p-5);  // 1/19
  p = __fma_rn(p, z, 0x1.e1e1e1e1e1e1ep-5);  // 1/17
  p = __fma_rn(p, z, 0x1.1111111111111p-4);  // 1/15
  p = __fma_rn(p, z, 0x1.3b13b13b13b14p-4);  // 1/13
  p = __fma_rn(p, z, 0x1.745d1745d1746p-4);  // 1/11
  p = __fma_rn(p, z, 0x1.c71c71c71c71cp-4);  // 1/9
  p = __fma_rn(p, z, 0x1.2492492492492p-3);  // 1/7
  p = __fma_rn(p, z, 0x1.999999999999ap-3);  // 1/5
  p = __fma_rn(p, z, 0x1.5555555555555p-2);  // 1/3
  const double s2 = __dadd_rn(s, s);
  const double lm = __fma_rn(__dmul_rn(s2, z), p, s2);
  const double LN2_HI = 0x1.62e42fefa3800p-1, LN2_LO = 0x1.ef35793c76730p-45;
  const double de = (double)e;
  double res = __fma_rn(de, LN2_HI, __fma_rn(de, LN2_LO, __dadd_rn(lm, corr)));
  const double inf = __longlong_as_double(0x7FF0000000000000ll);
  if (!(t > 0.0)) res = (t == 0.0) ? -inf : __longlong_as_double(0x7FF8000000000000ll);
  if (t == inf) res = inf;
  return res;
}

// log1p(y) for y <= 0 (and NaN), the argument erf_inv gives it (y = -x*x), branch-free:
// t = 1 + y and the rounding error of that sum added back as (y - (t - 1)) / t.
__device__ __forceinline__ double log1p_neg(double y) {
  const double t = __dadd_rn(1.0, y);
  const double corr =
      __dmul_rn(__dsub_rn(y, __dsub_rn(t, 1.0)), (double)__frcp_rn(__double2float_rn(t)));
  return log_core(t, corr);
}

// log(x) for x > 0.
__device__ __forceinline__ double log_pos(double x) { return log_core(x, 0.0); }

// ---- erf_inv --------------------------------------------------------------------------

// Giles' float32 erf_inv given w0 = -log1p(-x*x) rounded to float (no +-1 handling).
__device__ __forceinline__ float erfinv_f32_w(float x, float w0) {
  float p, w;
  if (w0 < 5.0f) {
    w = __fsub_rn(w0, 2.5f);
    p = 2.81022636e-08f;
    p = __fmaf_rn(p, w, 3.43273939e-07f);
    p = __fmaf_rn(p, w, -3.5233877e-06f);
    p = __fmaf_rn(p, w, -4.39150654e-06f);
    p = __fmaf_rn(p, w, 0.00021858087f);
    p = __fmaf_rn(p, w, -0.00125372503f);
    p = __fmaf_rn(p, w, -0.00417768164f);
    p = __fmaf_rn(p, w, 0.246640727f);
    p = __fmaf_rn(p, w, 1.50140941f);
  } else {
    w = __fsub_rn(__fsqrt_rn(w0), 3.0f);
    p = -0.000200214257f;
    p = __fmaf_rn(p, w, 0.000100950558f);
    p = __fmaf_rn(p, w, 0.00134934322f);
    p = __fmaf_rn(p, w, -0.00367342844f);
    p = __fmaf_rn(p, w, 0.00573950773f);
    p = __fmaf_rn(p, w, -0.0076224613f);
    p = __fmaf_rn(p, w, 0.00943887047f);
    p = __fmaf_rn(p, w, 1.00167406f);
    p = __fmaf_rn(p, w, 2.83297682f);
  }
  return __fmul_rn(p, x);
}

__device__ __forceinline__ float erfinv_f32(float x) {
  const float y = -__fmul_rn(x, x);
  const float w0 = -__double2float_rn(log1p_neg((double)y));
  if (fabsf(x) == 1.0f) return __fmul_rn(x, __int_as_float(0x7F800000));
  return erfinv_f32_w(x, w0);
}

// Giles' float64 erf_inv: p(w0) with erf_inv(x) = p x, for w0 = -log1p(-x*x).  The central
// piece (w0 < 6.25, i.e. |x| < 0.99903: all but about 1e-3 of a normal sampler's draws) and
// the two tail pieces are separate functions so that a kernel can evaluate several draws'
// central pieces in one branch-free stretch and the tails only where needed.
__device__ __forceinline__ double giles_f64_central(double w0) {
  double p;
  const double w = __dsub_rn(w0, 3.125);
  p = -3.6444120640178196996e-21;
  p = __fma_rn(p, w, -1.685059138182016589e-19);
  p = __fma_rn(p, w, 1.2858480715256400167e-18);
  p = __fma_rn(p, w, 1.115787767802518096e-17);
  p = __fma_rn(p, w, -1.333171662854620906e-16);
  p = __fma_rn(p, w, 2.0972767875968561637e-17);
  p = __fma_rn(p, w, 6.6376381343583238325e-15);
  p = __fma_rn(p, w, -4.0545662729752068639e-14);
  p = __fma_rn(p, w, -8.1519341976054721522e-14);
  p = __fma_rn(p, w, 2.6335093153082322977e-12);
  p = __fma_rn(p, w, -1.2975133253453532498e-11);
  p = __fma_rn(p, w, -5.4154120542946279317e-11);
  p = __fma_rn(p, w, 1.051212273321532285e-09);
  p = __fma_rn(p, w, -4.1126339803469836976e-09);
  p = __fma_rn(p, w, -2.9070369957882005086e-08);
  p = __fma_rn(p, w, 4.2347877827932403518e-07);
  p = __fma_rn(p, w, -1.3654692000834678645e-06);
  p = __fma_rn(p, w, -1.3882523362786468719e-05);
  p = __fma_rn(p, w, 0.0001867342080340571352);
  p = __fma_rn(p, w, -0.00074070253416626697512);
  p = __fma_rn(p, w, -0.0060336708714301490533);
  p = __fma_rn(p, w, 0.24015818242558961693);
  p = __fma_rn(p, w, 1.6536545626831027356);
  return p;
}

__device__ __forceinline__ double giles_f64_tail(double w0) {
  double p, w;
  if (w0 < 16.0) {
    w = __dsub_rn(__dsqrt_rn(w0), 3.25);
    p = 2.2137376921775787049e-09;
    p = __fma_rn(p, w, 9.0756561938885390979e-08);
    p = __fma_rn(p, w, -2.7517406297064545428e-07);
    p = __fma_rn(p, w, 1.8239629214389227755e-08);
    p = __fma_rn(p, w, 1.5027403968909827627e-06);
    p = __fma_rn(p, w, -4.013867526981545969e-06);
    p = __fma_rn(p, w, 2.9234449089955446044e-06);
    p = __fma_rn(p, w, 1.2475304481671778723e-05);
    p = __fma_rn(p, w, -4.7318229009055733981e-05);
    p = __fma_rn(p, w, 6.8284851459573175448e-05);
    p = __fma_rn(p, w, 2.4031110387097893999e-05);
    p = __fma_rn(p, w, -0.0003550375203628474796);
    p = __fma_rn(p, w, 0.00095328937973738049703);
    p = __fma_rn(p, w, -0.0016882755560235047313);
    p = __fma_rn(p, w, 0.0024914420961078508066);
    p = __fma_rn(p, w, -0.0037512085075692412107);
    p = __fma_rn(p, w, 0.005370914553590063617);
    p = __fma_rn(p, w, 1.0052589676941592334);
    p = __fma_rn(p, w, 3.0838856104922207635);
  } else {
    w = __dsub_rn(__dsqrt_rn(w0), 5.0);
    p = -2.7109920616438573243e-11;
    p = __fma_rn(p, w, -2.5556418169965252055e-10);
    p = __fma_rn(p, w, 1.5076572693500548083e-09);
    p = __fma_rn(p, w, -3.7894654401267369937e-09);
    p = __fma_rn(p, w, 7.6157012080783393804e-09);
    p = __fma_rn(p, w, -1.4960026627149240478e-08);
    p = __fma_rn(p, w, 2.9147953450901080826e-08);
    p = __fma_rn(p, w, -6.7711997758452339498e-08);
    p = __fma_rn(p, w, 2.2900482228026654717e-07);
    p = __fma_rn(p, w, -9.9298272942317002539e-07);
    p = __fma_rn(p, w, 4.5260625972231537039e-06);
    p = __fma_rn(p, w, -1.9681778105531670567e-05);
    p = __fma_rn(p, w, 7.5995277030017761139e-05);
    p = __fma_rn(p, w, -0.00021503011930044477347);
    p = __fma_rn(p, w, -0.00013871931833623122026);
    p = __fma_rn(p, w, 1.0103004648645343977);
    p = __fma_rn(p, w, 4.8499064014085844221);
  }
  return p;
}

__device__ __forceinline__ double erfinv_f64_w(double x, double w0) {
  double p;
  if (w0 < 6.25) p = giles_f64_central(w0);
  else p = giles_f64_tail(w0);
  return __dmul_rn(p, x);
}

__device__ __forceinline__ double erfinv_f64(double x) {
  const double w0 = -log1p_neg(-__dmul_rn(x, x));
  if (fabs(x) == 1.0) return __dmul_rn(x, __longlong_as_double(0x7FF0000000000000ll));
  return erfinv_f64_w(x, w0);
}

// ---- the float64 normal sampler's logarithm ----------------------------------------------
//
// -log(t) for a normal number t in (0, 1], table-driven (P. T. P. Tang, "Table-driven
// implementation of the logarithm function in IEEE floating-point arithmetic", ACM TOMS
// 16(4), 1990): t = 2^k z with z in [0.75, 1.5), the top 7 bits of z above 0.75 pick
// (inv, -log inv) with inv ~ 1 / z (log_table.h, made by make_log_table.py), and
// log t = k log 2 - log inv + log1p(z inv - 1), |z inv - 1| < 2^-8, the log1p a degree-7
// Taylor polynomial.  Integer work, one 16-byte L1-resident load and 11 float64
// operations, against ~27 float64 operations and 6 conversions or reciprocals of
// log1p_neg: the float64 normal sampler spends most of its time here.  Its absolute error
// is below 4e-16 (1 + |log t|), which moves a float64 normal by far less than the 1e-12
// relative that normals are held to; it is not bit-identical with log1p_neg.
__device__ const double2 kLogTabF64[JXR_LOG_TABLE_N] = {JXR_LOG_TABLE};

// log t, plus cnum / t when kCorr (the rounding error of a sum that made t, added back as
// log1p does); 1 / t for that term comes from the table entry's 1 / c and 2^-k, within
// 2^-7 relative, which is far below what a term of at most 2^-53 needs.
template <bool kCorr>
__device__ __forceinline__ double log_tab_core(double t, double cnum) {
  const uint32_t hi = (uint32_t)__double2hiint(t), lo = (uint32_t)__double2loint(t);
  const int k = (int)(hi - 0x3FE80000u) >> 20;  // arithmetic shift: z = t 2^-k in [0.75, 1.5)
  const uint32_t zhi = hi - ((uint32_t)k << 20);
  const double z = __hiloint2double((int)zhi, (int)lo);
  const double2 e = __ldg(&kLogTabF64[(zhi - 0x3FE80000u) >> 13]);
  const double r = __fma_rn(z, e.x, -1.0);
  double p = 0x1.2492492492492p-3;            //  1/7
  p = __fma_rn(p, r, -0x1.5555555555555p-3);  // -1/6
  p = __fma_rn(p, r, 0x1.999999999999ap-3);   //  1/5
  p = __fma_rn(p, r, -0.25);
  p = __fma_rn(p, r, 0x1.5555555555555p-2);   //  1/3
  p = __fma_rn(p, r, -0.5);
  const double l1p = __fma_rn(__dmul_rn(r, r), p, r);
  double s = __dadd_rn(e.y, l1p);
  if constexpr (kCorr) {
    const double inv_t = __dmul_rn(e.x, __hiloint2double((int)((uint32_t)(1023 - k) << 20), 0));
    s = __fma_rn(cnum, inv_t, s);
  }
  // k as a double without a conversion instruction: (2^52 + 2^31 + k) - (2^52 + 2^31)
  const double kd =
      __dsub_rn(__hiloint2double(0x43300000, (int)(0x80000000u + (uint32_t)k)), 0x1.000008p52);
  const double LN2_HI = 0x1.62e42fefa3800p-1, LN2_LO = 0x1.ef35793c76730p-45;
  return __fma_rn(kd, LN2_HI, __fma_rn(kd, LN2_LO, s));
}

// -log(t) for a normal t in (0, 1] (the float64 normal sampler's w).
__device__ __forceinline__ double neg_log_tab(double t) { return -log_tab_core<false>(t, 0.0); }

// log(t) for a normal t > 0, and log1p(y) for -1 < y <= 0 (1 + y normal), table-driven:
// the float32 and 16-bit samplers' logarithms.  Their results are rounded to float, and
// over all 2^23 float32 draws this rounds to the same float as log_pos / log1p_neg (the
// GPU tests compare every draw with the oracle): the double result is within ~1e-16 of
// the exact logarithm, while every exact value sits at least 1.2e-14 (relative) from a
// float rounding boundary.
__device__ __forceinline__ double log_tab(double t) { return log_tab_core<false>(t, 0.0); }
__device__ __forceinline__ double log1p_neg_tab(double y) {
  const double t = __dadd_rn(1.0, y);
  return log_tab_core<true>(t, __dsub_rn(y, __dsub_rn(t, 1.0)));
}

// The float32 erf_inv of the default lowering for |x| < 1 (the float32 and 16-bit normal
// samplers' open interval), with w from log1p_neg_tab: the same floats as erfinv_f32 there.
__device__ __forceinline__ float erfinv_f32_open(float x) {
  const float y = -__fmul_rn(x, x);
  return erfinv_f32_w(x, -__double2float_rn(log1p_neg_tab((double)y)));
}

// erf_inv of the default lowering for |x| < 1 (the normal sampler's open interval), with
// w = -log(1 - x*x) from neg_log_tab: x*x is rounded as the reference rounds it, and
// 1 - x*x is exact where it matters (x*x >= 1/2).
__device__ __forceinline__ double erfinv_f64_open(double x) {
  return erfinv_f64_w(x, neg_log_tab(__dsub_rn(1.0, __dmul_rn(x, x))));
}

// ---- accurate erf_inv (jax_accurate_erf_inv; R/lax_special.R:1022-1082) -----------------
//
// JAX's erf_inv_core(x, q = 1 - |x|) without its far-tail pieces: w = -log(q (1 + |x|)),
// which has no cancellation near |x| = 1.  Below the first split (float32 w < 3.5, float64
// w < 4.5) the result is x * P(w - c1); above it z = sqrt(w) is carried as z_h (the top
// half of its mantissa, so that z_h^2 is exact) plus z_l = (w - z_h^2) / (z + z_h), and
// the result is sign(x) (z_h + (z_l + P(z - shift))).  Each piece's coefficients are
// selected per element, as the reference selects them, and P is a fused Horner
// evaluation from the highest coefficient down.  The float32 logarithm is taken in double
// and rounded once.  |x| > 1 or NaN gives NaN, |x| = 1 gives x * inf.

__device__ __forceinline__ float erfinv_acc_f32(float x) {
  constexpr float P1[JXR_ERFINV32_P1_N] = {JXR_ERFINV32_P1};
  constexpr float P2[JXR_ERFINV32_P2_N] = {JXR_ERFINV32_P2};
  static_assert(JXR_ERFINV32_P1_N == JXR_ERFINV32_P2_N, "equal-length pieces");
  const float ax = fabsf(x);
  const float q = __fsub_rn(1.0f, ax);
  const float w = -__double2float_rn(log_pos((double)__fmul_rn(q, __fadd_rn(1.0f, ax))));
  const bool first = w < 3.5f;
  const float w_safe = first ? 1.0f : w;
  const float z = __fsqrt_rn(w_safe);
  const float z_h = __uint_as_float(__float_as_uint(z) & 0xFFFFF000u);
  const float z_l = __fdiv_rn(__fsub_rn(w_safe, __fmul_rn(z_h, z_h)), __fadd_rn(z, z_h));
  const float t = first ? __fsub_rn(w, 1.75f) : __fsub_rn(z, 3.0f);
  float p = first ? P1[JXR_ERFINV32_P1_N - 1] : P2[JXR_ERFINV32_P1_N - 1];
#pragma unroll
  for (int i = JXR_ERFINV32_P1_N - 2; i >= 0; --i) p = __fmaf_rn(p, t, first ? P1[i] : P2[i]);
  const float mag = __fadd_rn(z_h, __fadd_rn(z_l, p));
  const float r = first ? __fmul_rn(x, p) : (x < 0.0f ? -mag : mag);
  if (!(ax <= 1.0f)) return __int_as_float(0x7FC00000);
  if (ax == 1.0f) return __fmul_rn(x, __int_as_float(0x7F800000));
  return r;
}

__device__ __forceinline__ double erfinv_acc_f64(double x) {
  constexpr double P1[JXR_ERFINV64_P1_N] = {JXR_ERFINV64_P1};
  constexpr double P2[JXR_ERFINV64_P2_N] = {JXR_ERFINV64_P2};
  constexpr double P3[JXR_ERFINV64_P3_N] = {JXR_ERFINV64_P3};
  static_assert(JXR_ERFINV64_P1_N == JXR_ERFINV64_P2_N && JXR_ERFINV64_P1_N == JXR_ERFINV64_P3_N,
                "equal-length pieces");
  const double ax = fabs(x);
  const double q = __dsub_rn(1.0, ax);
  const double w = -log_pos(__dmul_rn(q, __dadd_rn(1.0, ax)));
  const int piece = w < 4.5 ? 0 : (w < 16.0 ? 1 : 2);
  const double w_safe = piece == 0 ? 1.0 : w;
  const double z = __dsqrt_rn(w_safe);
  const double z_h = __longlong_as_double(__double_as_longlong(z) & (long long)0xFFFFFFFFF8000000ull);
  const double z_l = __ddiv_rn(__dsub_rn(w_safe, __dmul_rn(z_h, z_h)), __dadd_rn(z, z_h));
  const double t = piece == 0 ? __dsub_rn(w, 2.25) : __dsub_rn(z, piece == 1 ? 3.0 : 5.0);
  constexpr int N = JXR_ERFINV64_P1_N;
  double p = piece == 0 ? P1[N - 1] : (piece == 1 ? P2[N - 1] : P3[N - 1]);
#pragma unroll
  for (int i = N - 2; i >= 0; --i)
    p = __fma_rn(p, t, piece == 0 ? P1[i] : (piece == 1 ? P2[i] : P3[i]));
  const double mag = __dadd_rn(z_h, __dadd_rn(z_l, p));
  const double r = piece == 0 ? __dmul_rn(x, p) : (x < 0.0 ? -mag : mag);
  if (!(ax <= 1.0)) return __longlong_as_double(0x7FF8000000000000ll);
  if (ax == 1.0) return __dmul_rn(x, __longlong_as_double(0x7FF0000000000000ll));
  return r;
}

// erf_inv of the reference's default lowering, or (kAcc) of jax_accurate_erf_inv's
template <bool kAcc>
__device__ __forceinline__ float erfinv32(float x) {
  if constexpr (kAcc) return erfinv_acc_f32(x);
  else return erfinv_f32(x);
}
template <bool kAcc>
__device__ __forceinline__ double erfinv64(double x) {
  if constexpr (kAcc) return erfinv_acc_f64(x);
  else return erfinv_f64(x);
}

// ---- 16-bit float helpers (raw bits in, raw bits out, arithmetic exact then rounded once) -

template <bool BF>
__device__ __forceinline__ float h2f(uint16_t h) {
  if constexpr (BF) return __uint_as_float((uint32_t)h << 16);
  else return __half2float(__ushort_as_half(h));
}
template <bool BF>
__device__ __forceinline__ uint16_t f2h(float f) {
  if constexpr (BF) return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  else return __half_as_ushort(__float2half_rn(f));
}
template <bool BF>
__device__ __forceinline__ uint16_t d2h(double d) {
  if constexpr (BF) return __bfloat16_as_ushort(__double2bfloat16(d));
  else return __half_as_ushort(__double2half(d));
}
// round a float that is exact (or rounded once to float) to the 16-bit type and back
template <bool BF>
__device__ __forceinline__ float rh(float f) { return h2f<BF>(f2h<BF>(f)); }

// ---- the transforms ---------------------------------------------------------------------
// Each has Bits (the unsigned draw it consumes: 32, 64, 16 or 8 bits), Out (what it
// stores) and operator()(Bits) -> Out.

template <int W> struct UintOf;
template <> struct UintOf<8> { using T = uint8_t; };
template <> struct UintOf<16> { using T = uint16_t; };
template <> struct UintOf<32> { using T = uint32_t; };
template <> struct UintOf<64> { using T = uint64_t; };

template <int W>
struct OpBits {
  static constexpr int kBits = W;
  using Bits = typename UintOf<W>::T;
  using Out = Bits;
  __device__ __forceinline__ Out operator()(Bits b) const { return b; }
};

__device__ __forceinline__ float unit_f32(uint32_t b) {
  return __fsub_rn(__uint_as_float((b >> 9) | 0x3F800000u), 1.0f);
}
__device__ __forceinline__ double unit_f64(uint64_t b) {
  return __dsub_rn(__longlong_as_double((long long)((b >> 12) | 0x3FF0000000000000ull)), 1.0);
}
// float16 draws 16 bits: shift 6, one = 0x3C00; bfloat16 has nmant = 7 < 8 and draws
// 8 bits, widened to 16: shift 1, one = 0x3F80.
template <bool BF>
__device__ __forceinline__ float unit_h(uint32_t b) {
  const uint16_t fb = BF ? (uint16_t)((b >> 1) | 0x3F80u) : (uint16_t)((b >> 6) | 0x3C00u);
  return __fsub_rn(h2f<BF>(fb), 1.0f);  // exact: the result is a 16-bit float in [0, 1)
}

template <bool kFused>
struct OpUniformF32 {
  static constexpr int kBits = 32;
  using Bits = uint32_t;
  using Out = float;
  float mn, d;  // minval and maxval - minval, in float32
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float f = unit_f32(b);
    const float r = kFused ? __fmaf_rn(f, d, mn) : __fadd_rn(__fmul_rn(f, d), mn);
    return xla_max(mn, r);
  }
};

template <bool kFused>
struct OpUniformF64 {
  static constexpr int kBits = 64;
  using Bits = uint64_t;
  using Out = double;
  double mn, d;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const double f = unit_f64(b);
    const double r = kFused ? __fma_rn(f, d, mn) : __dadd_rn(__dmul_rn(f, d), mn);
    return xla_max(mn, r);
  }
};

template <bool BF, bool kFused>
struct OpUniformH {
  static constexpr int kBits = BF ? 8 : 16;
  using Bits = typename UintOf<kBits>::T;
  using Out = uint16_t;
  float mn, d;  // values of 16-bit floats
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float f = unit_h<BF>(b);
    float r;
    if (kFused) r = h2f<BF>(d2h<BF>(__fma_rn((double)f, (double)d, (double)mn)));
    else r = rh<BF>(__fadd_rn(rh<BF>(__fmul_rn(f, d)), mn));
    return f2h<BF>(xla_max(mn, r));
  }
};

// u = uniform(nextafter(-1, 0), 1): maxval - minval rounds to exactly 2 in every dtype,
// so u = 2 f + lo is exact and the fused and unfused forms agree.
template <bool kAcc = false>
struct OpNormalF32T {
  static constexpr int kBits = 32;
  static constexpr int kGroups = 1;  // 4 blocks per thread: the transform needs the registers
  using Bits = uint32_t;
  using Out = float;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float lo = -0x1.fffffep-1f;  // -1 + 2^-24
    const float u = xla_max(lo, __fmaf_rn(unit_f32(b), 2.0f, lo));
    if constexpr (kAcc) return __fmul_rn(1.41421354f, erfinv_acc_f32(u));
    else return __fmul_rn(1.41421354f, erfinv_f32_open(u));  // |u| < 1
  }
};
using OpNormalF32 = OpNormalF32T<false>;

// A float32 sampler whose output depends only on bits >> 9 (the 23 mantissa bits of its
// unit float), read back from the table of its 2^23 results (32 MiB, built on the device by
// the sampler's own op, so identical to evaluating it): the cipher plus one L2 load.
struct OpTableF32 {
  static constexpr int kBits = 32;
  using Bits = uint32_t;
  using Out = float;
  const float* __restrict__ table;
  __device__ __forceinline__ Out operator()(Bits b) const { return __ldg(table + (b >> 9)); }
};

// A float16 (bfloat16) sampler whose output depends only on the top 10 (7) bits of its
// 16-bit (8-bit) draw -- every op built on unit_h -- read back from the table of its
// 1024 (128) results, built on the device by the op itself: 2 KiB at most, so the
// gathers hit L1.
template <int kDrawBits>
struct OpTableH {
  static constexpr int kBits = kDrawBits;
  static constexpr int kShift = kDrawBits == 16 ? 6 : 1;
  static constexpr int kEntries = 1 << (kDrawBits - kShift);
  using Bits = typename UintOf<kBits>::T;
  using Out = uint16_t;
  const uint16_t* __restrict__ table;
  __device__ __forceinline__ Out operator()(Bits b) const { return __ldg(table + (b >> kShift)); }
};

// The table gathers are bound by L1TEX throughput while the integer pipe has room, and
// evaluating an op directly is bound by the integer pipe: the single-key kernel evaluates
// kDirect of a thread's 16 outputs directly (op.direct, the op the table was built from,
// so the values are identical) and gathers the others.  Other kernels use the
// table for every element.
template <class Op, int kDirectOutputs = 4>
struct OpTableHybridF32 {
  static constexpr int kBits = 32;
  static constexpr int kGroups = 4;                    // 16 outputs per thread and tile
  static constexpr int kDirect = kDirectOutputs;       // of which evaluated directly
  using Bits = uint32_t;
  using Out = float;
  const float* __restrict__ table;
  Op op;
  __device__ __forceinline__ Out operator()(Bits b) const { return __ldg(table + (b >> 9)); }
  __device__ __forceinline__ Out direct(Bits b) const { return op(b); }
};

template <bool kAcc = false>
struct OpNormalF64T {
  static constexpr int kBits = 64;
  static constexpr int kGroups = 2;
  using Bits = uint64_t;
  using Out = double;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const double lo = -0x1.fffffffffffffp-1;  // -1 + 2^-53
    const double u = xla_max(lo, __fma_rn(unit_f64(b), 2.0, lo));
    // |u| < 1: the default erf_inv takes its logarithm from neg_log_tab
    if constexpr (kAcc) return __dmul_rn(1.4142135623730951, erfinv_acc_f64(u));
    else return __dmul_rn(1.4142135623730951, erfinv_f64_open(u));
  }
  // N draws at once (default erf_inv): the uniforms and logarithms, then every draw's
  // central piece in one branch-free stretch -- N independent polynomial chains that the
  // scheduler interleaves, where one branch per draw would run them one after another --
  // and the tail piece only where a draw needs it.  The same operations as operator(),
  // so the same results.
  static constexpr bool kBatch = !kAcc;
  template <int N>
  __device__ __forceinline__ void batch(const Bits* b, Out* out) const {
    const double lo = -0x1.fffffffffffffp-1;
    double u[N], w[N];
    bool tail = false;
#pragma unroll
    for (int k = 0; k < N; ++k) {
      u[k] = xla_max(lo, __fma_rn(unit_f64(b[k]), 2.0, lo));
      w[k] = neg_log_tab(__dsub_rn(1.0, __dmul_rn(u[k], u[k])));
      tail |= !(w[k] < 6.25);
    }
#pragma unroll
    for (int k = 0; k < N; ++k)
      out[k] = __dmul_rn(1.4142135623730951, __dmul_rn(giles_f64_central(w[k]), u[k]));
    if (tail) {
#pragma unroll
      for (int k = 0; k < N; ++k)
        if (!(w[k] < 6.25))
          out[k] = __dmul_rn(1.4142135623730951, __dmul_rn(giles_f64_tail(w[k]), u[k]));
    }
  }
};
using OpNormalF64 = OpNormalF64T<false>;

// erf_inv of a 16-bit float is evaluated in float32 and rounded back.
template <bool BF, bool kAcc = false>
struct OpNormalH {
  static constexpr int kBits = BF ? 8 : 16;
  static constexpr int kGroups = 1;
  using Bits = typename UintOf<kBits>::T;
  using Out = uint16_t;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float lo = BF ? -0x1.fep-1f : -0x1.ffcp-1f;  // -1 + 2^-8, -1 + 2^-11
    const float u = xla_max(lo, rh<BF>(__fmaf_rn(unit_h<BF>(b), 2.0f, lo)));
    float e;  // |u| < 1
    if constexpr (kAcc) e = rh<BF>(erfinv_acc_f32(u));
    else e = rh<BF>(erfinv_f32_open(u));
    return f2h<BF>(__fmul_rn(rh<BF>(1.41421354f), e));
  }
};

// uniform(key, shape, dtype(p), 0, 1) is the unit float itself (f * 1 + 0 = f and
// max(0, f) = f), so the draw is unit(bits) < p in dtype(p).
struct OpBernoulliF32 {
  static constexpr int kBits = 32;
  using Bits = uint32_t;
  using Out = uint8_t;
  float p;
  __device__ __forceinline__ Out operator()(Bits b) const { return unit_f32(b) < p; }
};
struct OpBernoulliF64 {
  static constexpr int kBits = 64;
  using Bits = uint64_t;
  using Out = uint8_t;
  double p;
  __device__ __forceinline__ Out operator()(Bits b) const { return unit_f64(b) < p; }
};
template <bool BF>
struct OpBernoulliH {
  static constexpr int kBits = BF ? 8 : 16;
  using Bits = typename UintOf<kBits>::T;
  using Out = uint8_t;
  float p;  // value of a 16-bit float
  __device__ __forceinline__ Out operator()(Bits b) const { return unit_h<BF>(b) < p; }
};

// ---- log-transform samplers (R/random.R:1422-1516) -------------------------------------
//
//   exponential  -log1p(-u),              u = uniform(0, 1)
//   gumbel       -log(-log(u)),           u = uniform(tiny, 1)          (mode "low")
//   logistic     log(x) - log1p(-x),      x = uniform(tiny, 1)
//   laplace      sign(u) log1p(-|u|),     u = uniform(-1 + 2^-(nmant+1), 1)
// Each float op of the reference's chain is rounded to the dtype once: the logarithms
// are evaluated in double (log_core) and rounded to float32 (then, for 16-bit dtypes,
// to 16 bits, as XLA evaluates 16-bit transcendentals in float32).

enum { kExponential = 0, kGumbel = 1, kLogistic = 2, kLaplace = 3 };

template <int kKind, int D>
struct OpLogSampler;

template <int kKind>
struct OpLogSampler<kKind, 0> {  // float32
  static constexpr int kBits = 32;
  static constexpr int kGroups = 1;
  using Bits = uint32_t;
  using Out = float;
  OpUniformF32<true> uni;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float u = uni(b);
    if constexpr (kKind == kExponential) {
      return -__double2float_rn(log1p_neg_tab(-(double)u));
    } else if constexpr (kKind == kGumbel) {
      const float a = __double2float_rn(log_tab((double)u));
      return -__double2float_rn(log_tab(-(double)a));
    } else if constexpr (kKind == kLogistic) {
      const float a = __double2float_rn(log_tab((double)u));
      const float c = __double2float_rn(log1p_neg_tab(-(double)u));
      return __fsub_rn(a, c);
    } else {
      const float l = __double2float_rn(log1p_neg_tab(-(double)fabsf(u)));
      return u < 0.0f ? -l : l;
    }
  }
};

template <int kKind>
struct OpLogSampler<kKind, 1> {  // float64
  static constexpr int kBits = 64;
  static constexpr int kGroups = 2;
  using Bits = uint64_t;
  using Out = double;
  OpUniformF64<true> uni;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const double u = uni(b);
    if constexpr (kKind == kExponential) {
      return -log1p_neg(-u);
    } else if constexpr (kKind == kGumbel) {
      return -log_pos(-log_pos(u));
    } else if constexpr (kKind == kLogistic) {
      return __dsub_rn(log_pos(u), log1p_neg(-u));
    } else {
      const double l = log1p_neg(-fabs(u));
      return u < 0.0 ? -l : l;
    }
  }
};

template <int kKind, bool BF>
struct OpLogSamplerH {  // float16 / bfloat16: float32 arithmetic rounded to 16 bits
  static constexpr int kBits = BF ? 8 : 16;
  static constexpr int kGroups = 1;
  using Bits = typename UintOf<kBits>::T;
  using Out = uint16_t;
  OpUniformH<BF, true> uni;
  __device__ __forceinline__ static float lg(double v) { return rh<BF>(__double2float_rn(v)); }
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float u = h2f<BF>(uni(b));
    float r;
    if constexpr (kKind == kExponential) {
      r = -lg(log1p_neg_tab(-(double)u));
    } else if constexpr (kKind == kGumbel) {
      r = -lg(log_tab(-(double)lg(log_tab((double)u))));
    } else if constexpr (kKind == kLogistic) {
      r = rh<BF>(__fsub_rn(lg(log_tab((double)u)), lg(log1p_neg_tab(-(double)u))));
    } else {
      const float l = lg(log1p_neg_tab(-(double)fabsf(u)));
      r = u < 0.0f ? -l : l;
    }
    return f2h<BF>(r);
  }
};
template <int kKind>
struct OpLogSampler<kKind, 2> : OpLogSamplerH<kKind, false> {};
template <int kKind>
struct OpLogSampler<kKind, 3> : OpLogSamplerH<kKind, true> {};

// ---- randint (R/random.R:306-359): two draws of the split key combined exactly ---------

// hi, lo: nbits-bit draws; span, mult as the reference computes them per element.
template <class U>
__device__ __forceinline__ U randint_offset(U hi, U lo, U span) {
  U m = (U)(((U)1 << (sizeof(U) * 4)) % span);
  m = (U)(m * m) % span;
  return (U)((U)((hi % span) * m) + (lo % span)) % span;
}

// ---- truncated normal (R/random.R:586-603) ----------------------------------------------
//
// u = uniform(a, b) with a = erf(lower / sqrt 2), b = erf(upper / sqrt 2), then
// sqrt(2) erf_inv(u) clipped to [nextafter(lower, inf), nextafter(upper, -inf)].  a, b and
// the clip bounds are parameters (computed once per call on the host).

template <int D, bool kAcc = false>
struct OpTruncNormal;

template <bool kAcc>
struct OpTruncNormal<0, kAcc> {  // float32
  static constexpr int kBits = 32;
  static constexpr int kGroups = 1;
  using Bits = uint32_t;
  using Out = float;
  OpUniformF32<true> uni;
  float lo, hi;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float x = __fmul_rn(1.41421354f, erfinv32<kAcc>(uni(b)));
    return xla_min(hi, xla_max(lo, x));
  }
};

template <bool kAcc>
struct OpTruncNormal<1, kAcc> {  // float64
  static constexpr int kBits = 64;
  static constexpr int kGroups = 2;
  using Bits = uint64_t;
  using Out = double;
  OpUniformF64<true> uni;
  double lo, hi;
  __device__ __forceinline__ Out operator()(Bits b) const {
    const double x = __dmul_rn(1.4142135623730951, erfinv64<kAcc>(uni(b)));
    return xla_min(hi, xla_max(lo, x));
  }
};

template <bool BF, bool kAcc>
struct OpTruncNormalH {
  static constexpr int kBits = BF ? 8 : 16;
  static constexpr int kGroups = 1;
  using Bits = typename UintOf<kBits>::T;
  using Out = uint16_t;
  OpUniformH<BF, true> uni;
  float lo, hi;  // values of 16-bit floats
  __device__ __forceinline__ Out operator()(Bits b) const {
    const float e = rh<BF>(erfinv32<kAcc>(h2f<BF>(uni(b))));
    const float x = rh<BF>(__fmul_rn(rh<BF>(1.41421354f), e));
    return f2h<BF>(xla_min(hi, xla_max(lo, x)));
  }
};
template <bool kAcc>
struct OpTruncNormal<2, kAcc> : OpTruncNormalH<false, kAcc> {};
template <bool kAcc>
struct OpTruncNormal<3, kAcc> : OpTruncNormalH<true, kAcc> {};

// ---- gumbel modes "high" and "highest" (R/random.R:1465-1489) ----------------------------
//
// Both draw a (2, n) array and combine element i of row 0 with element i of row 1.
// "high": high, low uniforms in [0, 1); x = high if high >= 0.5, else
// high + 2^-nmant low + max(2^-(2 nmant + 1), tiny); result -log(-log1p(-x)).

__device__ __forceinline__ float gumbel_high_f32(float high, float low) {
  const float x = high >= 0.5f ? high : __fadd_rn(__fadd_rn(high, __fmul_rn(0x1p-23f, low)), 0x1p-47f);
  const float a = __double2float_rn(log1p_neg(-(double)x));
  return -__double2float_rn(log_pos(-(double)a));
}
__device__ __forceinline__ double gumbel_high_f64(double high, double low) {
  const double x =
      high >= 0.5 ? high : __dadd_rn(__dadd_rn(high, __dmul_rn(0x1p-52, low)), 0x1p-105);
  return -log_pos(-log1p_neg(-x));
}
template <bool BF>
__device__ __forceinline__ float gumbel_high_h(float high, float low) {
  // f16: 2^-10 low + max(2^-21, 2^-14); bf16: 2^-7 low + max(2^-15, 2^-126)
  const float x = high >= 0.5f ? high
                               : rh<BF>(__fadd_rn(rh<BF>(__fadd_rn(high, rh<BF>(__fmul_rn(BF ? 0x1p-7f : 0x1p-10f, low)))),
                                                  BF ? 0x1p-15f : 0x1p-14f));
  const float a = rh<BF>(__double2float_rn(log1p_neg(-(double)x)));
  return -rh<BF>(__double2float_rn(log_pos(-(double)a)));
}

// XLA shift semantics: amounts of 32 or more give 0.
__device__ __forceinline__ uint32_t xshl(uint32_t x, uint32_t s) { return s >= 32u ? 0u : x << s; }
__device__ __forceinline__ uint32_t xshr(uint32_t x, uint32_t s) { return s >= 32u ? 0u : x >> s; }

// The 64-bit fixed-point fraction hi:lo as a float32 in (0, 1), keeping the leading 24
// significant bits (R/random.R:1446-1462).
__device__ __forceinline__ float safe_int_to_float(uint32_t hi, uint32_t lo) {
  const uint32_t hiclz = (uint32_t)__clz(hi), loclz = (uint32_t)__clz(lo);
  uint32_t mant = xshl(hi, hiclz) | (hiclz == 32u ? xshl(lo, loclz) : xshr(lo, 32u - hiclz));
  mant = (mant >> 8) & 0x7FFFFFu;
  const uint32_t ex = ((126u - (hiclz == 32u ? 32u + loclz : hiclz)) << 23) & 0x3FC00000u;
  return __uint_as_float(ex | mant);
}

// "highest" (float32): b0, b1 are 32-bit draws of rows 0 and 1; values below 1/2 use
// 1 - bits (the 64-bit negation) through log1p, the others log.
__device__ __forceinline__ float gumbel_highest_f32(uint32_t b0, uint32_t b1) {
  const bool flip = b0 < 0x80000000u;
  const uint32_t n1 = ~b1, n0 = ~b0 + (n1 == 0xFFFFFFFFu ? 1u : 0u);
  const float x = flip ? safe_int_to_float(b0, b1) : safe_int_to_float(n0, n1 + 1u);
  if (flip) {
    const float a = __double2float_rn(log1p_neg(-(double)x));
    return -__double2float_rn(log_pos(-(double)a));
  }
  const float a = __double2float_rn(log_pos((double)x));
  return -__double2float_rn(log_pos(-(double)a));
}

}  // namespace jxr
