/* jaxR's .Call shim over libjxrng: the routines jxrng.R calls for the eager threefry path
 * (random_bits, random_split, random_fold_in, random_uniform, random_normal,
 * random_bernoulli), registered as src/pjrt.cpp:799-826 registers jaxR's own.
 *
 * Conventions (those of src/pjrt.cpp):
 *  - Host scratch comes from R_alloc, which R releases on return and on Rf_error; the
 *    shim core (jxrng_shim.c) frees its device buffers before it returns, so an Rf_error
 *    after a failed call leaks nothing (src/pjrt.cpp:568-570).
 *  - Keys arrive as the key data's uint32 words in R doubles (array_host of a
 *    uint32[..., 2] jax array, row-major); counts as doubles, exact up to 2^53.
 *  - Results go back in jaxR's host representation (jaxr_buffer_to_host,
 *    src/pjrt.cpp:663-722): numbers as doubles, booleans as logicals.  Float16 and
 *    bfloat16 results come back as their 16-bit patterns, which jxrng.R bitcasts; 64-bit
 *    bits as list(hi, lo) of their 32-bit halves, which jxrng.R joins as R/prng.R:220-224
 *    does (doubles cannot hold every uint64).
 *  - Called from the R main thread only, like every jaxR routine (src/callbacks.cpp:10-15).
 *
 * Build beside jaxR (R's headers, libjxrng.so and the CUDA runtime):
 *   R CMD SHLIB -o jxrngR.so jxrng_r.c jxrng_shim.c -I../../include -L.. -ljxrng -lcudart */
#include <R.h>
#include <Rinternals.h>
#include <R_ext/Rdynload.h>

#include <stdint.h>
#include <string.h>

#include "jxrng.h"
#include "jxrng_shim.h"

static void stop_on(int rc) {
  if (rc != JXR_OK) Rf_error("%s", jxs_error());
}

/* the key words of `key_words` (a double vector, two words per key) as uint32 */
static int64_t keys_from_r(SEXP key_words, uint32_t** keys) {
  if (TYPEOF(key_words) != REALSXP) Rf_error("jxrng: key words must be a double vector");
  const R_xlen_t nw = XLENGTH(key_words);
  uint32_t* k = (uint32_t*)R_alloc(nw ? (size_t)nw : 1, sizeof(uint32_t));
  stop_on(jxs_key_words(REAL(key_words), (int64_t)nw, k));
  *keys = k;
  return (int64_t)(nw / 2);
}

static uint64_t count_from_r(SEXP x, const char* what) {
  uint64_t v = 0;
  stop_on(jxs_count(Rf_asReal(x), what, &v));
  return v;
}

/* nkeys * per as an R vector length */
static R_xlen_t r_length(int64_t nkeys, uint64_t per) {
  if (per && (uint64_t)nkeys > (uint64_t)R_XLEN_T_MAX / per)
    Rf_error("jxrng: %lld keys x %.0f elements exceed R's longest vector", (long long)nkeys,
             (double)per);
  return (R_xlen_t)((uint64_t)nkeys * per);
}

static void* host_scratch(R_xlen_t n, uint64_t elem_bytes) {
  size_t bytes = 0;
  stop_on(jxs_bytes((uint64_t)n, elem_bytes, &bytes));
  return R_alloc(bytes + 1, 1);
}

static int dtype_code(SEXP dtype) {
  const int dt = Rf_asInteger(dtype);
  if (dt < JXR_F32 || dt > JXR_BF16) Rf_error("jxrng: dtype code must be 0..3, got %d", dt);
  return dt;
}

/* host results of a float dtype -> doubles (16-bit types: their bit patterns) */
static SEXP floats_to_r(const void* host, R_xlen_t n, int dt) {
  SEXP out = PROTECT(Rf_allocVector(REALSXP, n));
  double* o = REAL(out);
  const unsigned char* p = (const unsigned char*)host;
  for (R_xlen_t i = 0; i < n; ++i) {
    if (dt == JXR_F32) {
      float v;
      memcpy(&v, p + 4 * i, 4);
      o[i] = v;
    } else if (dt == JXR_F64) {
      memcpy(o + i, p + 8 * i, 8);
    } else {
      uint16_t v;
      memcpy(&v, p + 2 * i, 2);
      o[i] = v;
    }
  }
  UNPROTECT(1);
  return out;
}

/* random_bits(key, shape) of each key: key_words (2 per key), size = prod(shape), layout
 * (1 = jax_threefry_partitionable), bit_width 8/16/32/64. */
SEXP jxr_r_random_bits(SEXP key_words, SEXP size, SEXP layout, SEXP bit_width) {
  uint32_t* keys;
  const int64_t nkeys = keys_from_r(key_words, &keys);
  const uint64_t n = count_from_r(size, "size");
  const int bw = Rf_asInteger(bit_width);
  if (bw != 8 && bw != 16 && bw != 32 && bw != 64)
    Rf_error("jxrng: requires 8-, 16-, 32- or 64-bit field width, got %d", bw);
  const R_xlen_t len = r_length(nkeys, n);
  void* host = host_scratch(len, (uint64_t)bw / 8);
  stop_on(jxs_random_bits(keys, nkeys, n, Rf_asInteger(layout), bw, host));
  const unsigned char* p = (const unsigned char*)host;
  if (bw == 64) {
    SEXP hi = PROTECT(Rf_allocVector(REALSXP, len));
    SEXP lo = PROTECT(Rf_allocVector(REALSXP, len));
    for (R_xlen_t i = 0; i < len; ++i) {
      uint64_t w;
      memcpy(&w, p + 8 * i, 8);
      REAL(hi)[i] = (double)(uint32_t)(w >> 32);
      REAL(lo)[i] = (double)(uint32_t)w;
    }
    SEXP out = PROTECT(Rf_allocVector(VECSXP, 2));
    SET_VECTOR_ELT(out, 0, hi);
    SET_VECTOR_ELT(out, 1, lo);
    UNPROTECT(3);
    return out;
  }
  SEXP out = PROTECT(Rf_allocVector(REALSXP, len));
  double* o = REAL(out);
  for (R_xlen_t i = 0; i < len; ++i) {
    if (bw == 8) {
      o[i] = p[i];
    } else if (bw == 16) {
      uint16_t w;
      memcpy(&w, p + 2 * i, 2);
      o[i] = w;
    } else {
      uint32_t w;
      memcpy(&w, p + 4 * i, 4);
      o[i] = w;
    }
  }
  UNPROTECT(1);
  return out;
}

/* random_uniform(key, shape, dtype, minval, maxval) with scalar bounds; dtype a JXR_F* code */
SEXP jxr_r_uniform(SEXP key_words, SEXP size, SEXP layout, SEXP dtype, SEXP minval,
                   SEXP maxval) {
  uint32_t* keys;
  const int64_t nkeys = keys_from_r(key_words, &keys);
  const uint64_t n = count_from_r(size, "size");
  const int dt = dtype_code(dtype);
  const R_xlen_t len = r_length(nkeys, n);
  void* host = host_scratch(len, dt == JXR_F64 ? 8 : dt == JXR_F32 ? 4 : 2);
  stop_on(jxs_uniform(keys, nkeys, n, Rf_asInteger(layout), dt, Rf_asReal(minval),
                      Rf_asReal(maxval), host));
  return floats_to_r(host, len, dt);
}

/* random_normal(key, shape, dtype) for a real dtype; accurate = jax_accurate_erf_inv */
SEXP jxr_r_normal(SEXP key_words, SEXP size, SEXP layout, SEXP dtype, SEXP accurate) {
  uint32_t* keys;
  const int64_t nkeys = keys_from_r(key_words, &keys);
  const uint64_t n = count_from_r(size, "size");
  const int dt = dtype_code(dtype);
  const R_xlen_t len = r_length(nkeys, n);
  void* host = host_scratch(len, dt == JXR_F64 ? 8 : dt == JXR_F32 ? 4 : 2);
  stop_on(jxs_normal(keys, nkeys, n, Rf_asInteger(layout), dt, Rf_asLogical(accurate) == TRUE,
                     host));
  return floats_to_r(host, len, dt);
}

/* random_bernoulli(key, p, shape), mode "low", scalar p of dtype p_dtype */
SEXP jxr_r_bernoulli(SEXP key_words, SEXP size, SEXP layout, SEXP p_dtype, SEXP p) {
  uint32_t* keys;
  const int64_t nkeys = keys_from_r(key_words, &keys);
  const uint64_t n = count_from_r(size, "size");
  const int dt = dtype_code(p_dtype);
  const R_xlen_t len = r_length(nkeys, n);
  uint8_t* host = (uint8_t*)host_scratch(len, 1);
  stop_on(jxs_bernoulli(keys, nkeys, n, Rf_asInteger(layout), dt, Rf_asReal(p), host));
  SEXP out = PROTECT(Rf_allocVector(LGLSXP, len));
  for (R_xlen_t i = 0; i < len; ++i) LOGICAL(out)[i] = host[i] != 0;
  UNPROTECT(1);
  return out;
}

/* random_split(key, num) of each key: 2 * num words per key */
SEXP jxr_r_split(SEXP key_words, SEXP num, SEXP layout) {
  uint32_t* keys;
  const int64_t nkeys = keys_from_r(key_words, &keys);
  const uint64_t m = count_from_r(num, "num");
  const R_xlen_t len = r_length(nkeys, m);
  uint32_t* host = (uint32_t*)host_scratch(len, 8);
  stop_on(jxs_split(keys, nkeys, m, Rf_asInteger(layout), host));
  SEXP out = PROTECT(Rf_allocVector(REALSXP, 2 * len));
  for (R_xlen_t i = 0; i < 2 * len; ++i) REAL(out)[i] = host[i];
  UNPROTECT(1);
  return out;
}

/* random_fold_in(key, data): data a double vector of uint32 values (one, or one per key) */
SEXP jxr_r_fold_in(SEXP key_words, SEXP data) {
  uint32_t* keys;
  const int64_t nkeys = keys_from_r(key_words, &keys);
  if (TYPEOF(data) != REALSXP) Rf_error("jxrng: fold_in data must be a double vector");
  const R_xlen_t nd = XLENGTH(data);
  uint32_t* d = (uint32_t*)R_alloc(nd ? (size_t)nd : 1, sizeof(uint32_t));
  for (R_xlen_t i = 0; i < nd; ++i) {
    uint64_t v = 0;
    stop_on(jxs_count(REAL(data)[i], "fold_in data", &v));
    if (v > 0xFFFFFFFFull) Rf_error("jxrng: fold_in data %.0f out of bounds for uint32", REAL(data)[i]);
    d[i] = (uint32_t)v;
  }
  const int64_t n = nkeys > (int64_t)nd ? nkeys : (int64_t)nd;
  uint32_t* host = (uint32_t*)host_scratch((R_xlen_t)n, 8);
  stop_on(jxs_fold_in(keys, nkeys, d, (int64_t)nd, host));
  SEXP out = PROTECT(Rf_allocVector(REALSXP, 2 * (R_xlen_t)n));
  for (R_xlen_t i = 0; i < 2 * (R_xlen_t)n; ++i) REAL(out)[i] = host[i];
  UNPROTECT(1);
  return out;
}

/* set-up, once per session: jxr_prepare_device(what) on the current device */
SEXP jxr_r_prepare(SEXP what) {
  stop_on(jxs_prepare((uint32_t)Rf_asInteger(what)));
  return R_NilValue;
}

static const R_CallMethodDef jxrng_calls[] = {
    {"jxr_r_random_bits", (DL_FUNC)&jxr_r_random_bits, 4},
    {"jxr_r_uniform", (DL_FUNC)&jxr_r_uniform, 6},
    {"jxr_r_normal", (DL_FUNC)&jxr_r_normal, 5},
    {"jxr_r_bernoulli", (DL_FUNC)&jxr_r_bernoulli, 5},
    {"jxr_r_split", (DL_FUNC)&jxr_r_split, 3},
    {"jxr_r_fold_in", (DL_FUNC)&jxr_r_fold_in, 2},
    {"jxr_r_prepare", (DL_FUNC)&jxr_r_prepare, 1},
    {NULL, NULL, 0}};

void R_init_jxrngR(DllInfo* dll) {
  R_registerRoutines(dll, NULL, jxrng_calls, NULL, NULL);
  R_useDynamicSymbols(dll, FALSE);
}
