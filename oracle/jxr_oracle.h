/*
 * CPU oracle for the threefry2x32 random-bits path of jaxR.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a scalar C restatement of the reference
 * algorithm, used as the checker by tests/, by __graft_entry__.smoke() and as
 * the timed CPU baseline leg of bench.py.  The product (libjxrng) never links,
 * loads or calls it, and there is no CPU fallback anywhere in the product.
 *
 * Every function cites the reference lines (paths within the jaxR project) it
 * restates.  Element-wise "_at" functions compute one output element from its
 * linear index, so the oracle can check arbitrary positions of requests far
 * larger than it could generate in full.
 */
#ifndef JXR_ORACLE_H
#define JXR_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes shared with include/jxrng.h */
enum { ORC_F32 = 0, ORC_F64 = 1, ORC_F16 = 2, ORC_BF16 = 3 };

/* Threefry-2x32, 20 rounds (R/prng.R:51-86). */
void orc_threefry2x32(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t out[2]);

/* Element-wise primitive over n broadcast elements (R/prng.R:88-99). */
void orc_threefry2x32_arr(const uint32_t* k0, const uint32_t* k1, const uint32_t* c0,
                          const uint32_t* c1, uint32_t* x0, uint32_t* x1, int64_t n);

/* threefry_2x32 hash of a uint32 count vector with odd-length zero padding
 * (R/prng.R:102-120). */
void orc_threefry_2x32(const uint32_t key[2], const uint32_t* count, int64_t n, uint32_t* out);

/* Seed -> key (R/prng.R:160-170 after R/prng.R:504-519).  With x64 off the
 * seed is first wrapped to int32, as an R number becomes a canonical int. */
void orc_seed(int64_t seed, int x64, uint32_t out[2]);

/* split into num keys, out is uint32[num][2] (R/prng.R:173-191). */
void orc_split(const uint32_t key[2], int64_t num, int partitionable, uint32_t* out);

/* fold_in of a uint32 datum (R/prng.R:194). */
void orc_fold_in(const uint32_t key[2], uint32_t data, uint32_t out[2]);

/* One element of random_bits(key, bit_width, shape) with `size` elements in
 * total, at C-order linear index i (R/prng.R:202-262).  Returns the value
 * zero-extended to 64 bits. */
uint64_t orc_bits_at(const uint32_t key[2], int bit_width, uint64_t size, int partitionable,
                     uint64_t i);

/* Full arrays: out has `count` elements of width bit_width, elements
 * [begin, begin+count) of a request of `size` elements.  OpenMP-parallel. */
int orc_random_bits(const uint32_t key[2], int bit_width, uint64_t size, int partitionable,
                    uint64_t begin, uint64_t count, void* out);

/* erf_inv as lowered by the reference's default path: M. Giles, "Approximating
 * the erfinv function" (GPU Computing Gems Jade, 2011), with the logarithm
 * taken as -log1p(-x*x) and erf_inv(+-1) = +-inf (R/lax_special.R:1327-1331
 * emits chlo.erf_inv).  fma selects a fused Horner evaluation.  The logarithm is
 * log1p_neg below, evaluated in double (and, for float32, rounded once). */
/* mode bit 1 (ORC_ERFINV_ACCURATE): the accurate erf_inv of jax_accurate_erf_inv instead
 * (R/lax_special.R:1022-1082, JAX's erf_inv_core without the far-tail pieces); bit 0
 * still selects fused Horner steps. */
enum { ORC_ERFINV_ACCURATE = 2 };
float orc_erfinv_f32(float x, int fma);
double orc_erfinv_f64(double x, int fma);
void orc_erfinv_arr(const void* x, int64_t n, int dtype, int fma, void* out);

/* log1p(y) for y <= 0 and log(x) for x > 0 as the kernels evaluate them (Cody and Waite
 * reduction). */
double orc_log1p_neg(double y);
double orc_log_pos(double x);

/* Samplers (R/random.R:288-304, :502-508, :656-666).  dtype is an ORC_ code;
 * 16-bit results are returned as their raw bits in a uint16_t array.
 * minval/maxval are given in double and converted to dtype first, as
 * lax_convert_element_type does.  mul_add_fma selects a fused
 * floats*(max-min)+min: the reference's jaxpr has a separate multiply and add,
 * but its recorded samples (tests/testthat/test-random.R:43, :160) are those of
 * the fused form, which XLA's CPU code generator contracts to. */
int orc_uniform(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                double minval, double maxval, int mul_add_fma, uint64_t begin,
                uint64_t count, void* out);
int orc_normal(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
               int erfinv_fma, uint64_t begin, uint64_t count, void* out);
int orc_bernoulli(const uint32_t key[2], int p_dtype, double p, uint64_t size,
                  int partitionable, uint64_t begin, uint64_t count, uint8_t* out);

/* Element-wise versions of the samplers at linear index i. */
double orc_uniform_at(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                      double minval, double maxval, int mul_add_fma, uint64_t i);
double orc_normal_at(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                     int erfinv_fma, uint64_t i);

/* Log-transform samplers (R/random.R:1422-1516): kind 0 exponential, 1 gumbel (mode
 * "low"), 2 logistic, 3 laplace, in dtype (ORC_ code). */
enum { ORC_EXPONENTIAL = 0, ORC_GUMBEL = 1, ORC_LOGISTIC = 2, ORC_LAPLACE = 3 };
int orc_sample(const uint32_t key[2], int kind, int dtype, uint64_t size, int partitionable,
               uint64_t begin, uint64_t count, void* out);
double orc_sample_at(const uint32_t key[2], int kind, int dtype, uint64_t size,
                     int partitionable, uint64_t i);

/* random_gumbel modes "high" (0) and "highest" (1, float32) (R/random.R:1465-1489) and
 * random_truncated_normal with scalar bounds (R/random.R:586-603). */
/* The float32 samplers of n given 32-bit draws: kind 0..3 exponential, gumbel (mode
 * "low"), logistic, laplace; 4 the normal (fused Horner steps). */
void orc_sample_f32_from_bits(const uint32_t* bits, int64_t n, int kind, float* out);
int orc_gumbel_mode(const uint32_t key[2], int mode, int dtype, uint64_t size,
                    int partitionable, void* out);
double orc_gumbel_mode_at(const uint32_t key[2], int mode, int dtype, uint64_t size,
                          int partitionable, uint64_t i);
int orc_truncated_normal(const uint32_t key[2], int dtype, uint64_t size, int partitionable,
                         double lower, double upper, int erfinv_mode, uint64_t begin,
                         uint64_t count, void* out);
double orc_truncated_normal_at(const uint32_t key[2], int dtype, uint64_t size,
                               int partitionable, double lower, double upper, int erfinv_mode,
                               uint64_t i);

/* rbg / unsafe_rbg (R/prng.R:264-426): XLA's RngBitGenerator as Philox4x32-10 with key
 * (q0, q1) and the key q as 128-bit counter, advanced per block of four 32-bit outputs. */
void orc_philox4x32(const uint32_t c[4], const uint32_t k[2], uint32_t out[4]);
int orc_rbg_bits(const uint32_t q[4], int bit_width, uint64_t size, uint64_t begin,
                 uint64_t count, void* out);
void orc_rbg_unsafe_split(const uint32_t q[4], int64_t num, uint32_t* out);
void orc_rbg_unsafe_fold_in(const uint32_t q[4], uint32_t data, uint32_t out[4]);

/* Number of OpenMP threads used by the array functions (0 = default). */
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
