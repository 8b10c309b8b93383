/* The R-independent core of the .Call shim: argument checks, device buffers and the
 * libjxrng calls (see jxrng_shim.h).  Plain C99 over the CUDA runtime's C API. */
#include "jxrng_shim.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <cuda_runtime.h>

#include "jxrng.h"

static __thread char g_msg[512];
static __thread int g_own_msg = 0; /* 1: g_msg holds the message; 0: libjxrng's last error */

static int shim_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof g_msg, fmt, ap);
  va_end(ap);
  g_own_msg = 1;
  return code;
}

/* a libjxrng status: its message stays in jxr_last_error() */
static int lib_status(int rc) {
  if (rc != JXR_OK) g_own_msg = 0;
  return rc;
}

const char* jxs_error(void) { return g_own_msg ? g_msg : jxr_last_error(); }

int jxs_count(double x, const char* what, uint64_t* out) {
  if (!(x >= 0.0) || x > 9007199254740992.0 || x != floor(x))
    return shim_fail(JXR_ERR_INVALID_ARGUMENT,
                     "jxrng: %s must be a whole number in [0, 2^53], got %.17g", what, x);
  *out = (uint64_t)x;
  return JXR_OK;
}

int jxs_key_words(const double* words, int64_t nwords, uint32_t* out) {
  if (nwords < 0 || nwords % 2)
    return shim_fail(JXR_ERR_INVALID_ARGUMENT,
                     "jxrng: threefry2x32 key data has two words per key, got %lld words",
                     (long long)nwords);
  for (int64_t i = 0; i < nwords; ++i) {
    const double w = words[i];
    if (!(w >= 0.0) || w > 4294967295.0 || w != floor(w))
      return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: key word %lld is not a uint32 (%.17g)",
                       (long long)i, w);
    out[i] = (uint32_t)w;
  }
  return JXR_OK;
}

int jxs_bytes(uint64_t n, uint64_t elem_bytes, size_t* out) {
  if (elem_bytes && n > (uint64_t)SIZE_MAX / elem_bytes)
    return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: %llu elements of %llu bytes overflow",
                     (unsigned long long)n, (unsigned long long)elem_bytes);
  *out = (size_t)(n * elem_bytes);
  return JXR_OK;
}

/* nkeys * per elements of elem_bytes each, checked */
static int total_bytes(int64_t nkeys, uint64_t per, uint64_t elem_bytes, size_t* out) {
  if (nkeys < 0) return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: negative key count");
  if (per && (uint64_t)nkeys > UINT64_MAX / per)
    return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: %lld keys x %llu elements overflow",
                     (long long)nkeys, (unsigned long long)per);
  return jxs_bytes((uint64_t)nkeys * per, elem_bytes, out);
}

static int dtype_bytes(int dtype, uint64_t* out) {
  switch (dtype) {
    case JXR_F32: *out = 4; return JXR_OK;
    case JXR_F64: *out = 8; return JXR_OK;
    case JXR_F16:
    case JXR_BF16: *out = 2; return JXR_OK;
  }
  return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: dtype code must be 0..3, got %d", dtype);
}

/* Device buffers of one call: keys (and data) up front, the result, all freed by
 * release(). */
typedef struct {
  void* keys;
  void* data;
  void* out;
} Bufs;

static void release(Bufs* b) {
  if (b->keys) cudaFree(b->keys);
  if (b->data) cudaFree(b->data);
  if (b->out) cudaFree(b->out);
  b->keys = b->data = b->out = NULL;
}

static int cuda_fail(Bufs* b, cudaError_t e, const char* what) {
  release(b);
  cudaGetLastError(); /* clear a sticky-free error for the next call */
  return shim_fail(JXR_ERR_CUDA, "jxrng: %s: %s", what, cudaGetErrorString(e));
}

/* allocates b->keys (and b->data when ndata_bytes) and b->out, and uploads the keys */
static int stage_in(Bufs* b, const void* keys, size_t key_bytes, const void* data,
                    size_t data_bytes, size_t out_bytes) {
  cudaError_t e;
  b->keys = b->data = b->out = NULL;
  if ((e = cudaMalloc(&b->keys, key_bytes ? key_bytes : 1)) != cudaSuccess)
    return cuda_fail(b, e, "cudaMalloc (keys)");
  if (data_bytes && (e = cudaMalloc(&b->data, data_bytes)) != cudaSuccess)
    return cuda_fail(b, e, "cudaMalloc (data)");
  if ((e = cudaMalloc(&b->out, out_bytes ? out_bytes : 1)) != cudaSuccess)
    return cuda_fail(b, e, "cudaMalloc (result)");
  if (key_bytes && (e = cudaMemcpy(b->keys, keys, key_bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
    return cuda_fail(b, e, "copying the keys to the device");
  if (data_bytes && (e = cudaMemcpy(b->data, data, data_bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
    return cuda_fail(b, e, "copying the data to the device");
  return JXR_OK;
}

/* after the launch: rc from libjxrng, then the result down (the copy waits for the kernel,
 * both on the legacy default stream) and every buffer freed */
static int stage_out(Bufs* b, int rc, void* host_out, size_t out_bytes) {
  if (rc != JXR_OK) {
    release(b);
    return lib_status(rc);
  }
  cudaError_t e = out_bytes ? cudaMemcpy(host_out, b->out, out_bytes, cudaMemcpyDeviceToHost)
                            : cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(b, e, "copying the result to the host");
  release(b);
  return JXR_OK;
}

int jxs_random_bits(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout,
                    int bit_width, void* host_out) {
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64)
    return shim_fail(JXR_ERR_INVALID_ARGUMENT,
                     "jxrng: requires 8-, 16-, 32- or 64-bit field width, got %d", bit_width);
  size_t bytes = 0;
  int rc = total_bytes(nkeys, size, (uint64_t)bit_width / 8, &bytes);
  if (rc) return rc;
  /* staged through the library's own device buffers: chunks generated and copied while
   * the next is generated */
  return lib_status(jxr_random_bits_host(keys, nkeys, size, 0, size, layout, bit_width, host_out));
}

int jxs_uniform(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout, int dtype,
                double minval, double maxval, void* host_out) {
  uint64_t esz = 0;
  size_t bytes = 0;
  Bufs b;
  int rc = dtype_bytes(dtype, &esz);
  if (rc || (rc = total_bytes(nkeys, size, esz, &bytes))) return rc;
  if ((rc = stage_in(&b, keys, 8 * (size_t)nkeys, NULL, 0, bytes))) return rc;
  rc = jxr_uniform((const uint32_t*)b.keys, nkeys, size, 0, size, layout, dtype, minval, maxval, 0,
                   b.out, NULL);
  return stage_out(&b, rc, host_out, bytes);
}

int jxs_normal(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout, int dtype,
               int accurate, void* host_out) {
  uint64_t esz = 0;
  size_t bytes = 0;
  Bufs b;
  int rc = dtype_bytes(dtype, &esz);
  if (rc || (rc = total_bytes(nkeys, size, esz, &bytes))) return rc;
  if ((rc = stage_in(&b, keys, 8 * (size_t)nkeys, NULL, 0, bytes))) return rc;
  /* the library's erf_inv choice is per host thread: set for this call, then put back */
  const int prev = jxr_set_accurate_erf_inv(accurate != 0);
  rc = jxr_normal((const uint32_t*)b.keys, nkeys, size, 0, size, layout, dtype, b.out, NULL);
  jxr_set_accurate_erf_inv(prev);
  return stage_out(&b, rc, host_out, bytes);
}

int jxs_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout, int p_dtype,
                  double p, uint8_t* host_out) {
  uint64_t esz = 0;
  size_t bytes = 0;
  Bufs b;
  int rc = dtype_bytes(p_dtype, &esz);
  if (rc || (rc = total_bytes(nkeys, size, 1, &bytes))) return rc;
  if ((rc = stage_in(&b, keys, 8 * (size_t)nkeys, NULL, 0, bytes))) return rc;
  rc = jxr_bernoulli((const uint32_t*)b.keys, nkeys, size, 0, size, layout, p_dtype, p,
                     (uint8_t*)b.out, NULL);
  return stage_out(&b, rc, host_out, bytes);
}

int jxs_split(const uint32_t* keys, int64_t nkeys, uint64_t num, int layout, uint32_t* host_out) {
  size_t bytes = 0;
  Bufs b;
  int rc = total_bytes(nkeys, num, 8, &bytes);
  if (rc) return rc;
  if (num > (uint64_t)INT64_MAX) return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: num too large");
  if ((rc = stage_in(&b, keys, 8 * (size_t)nkeys, NULL, 0, bytes))) return rc;
  rc = jxr_split((const uint32_t*)b.keys, nkeys, (int64_t)num, layout, (uint32_t*)b.out, NULL);
  return stage_out(&b, rc, host_out, bytes);
}

int jxs_fold_in(const uint32_t* keys, int64_t nkeys, const uint32_t* data, int64_t ndata,
                uint32_t* host_out) {
  if (nkeys < 0 || ndata < 0)
    return shim_fail(JXR_ERR_INVALID_ARGUMENT, "jxrng: negative key or data count");
  const int64_t n = nkeys > ndata ? nkeys : ndata;
  if ((nkeys != n && nkeys != 1) || (ndata != n && ndata != 1))
    return shim_fail(JXR_ERR_INVALID_ARGUMENT,
                     "jxrng: fold_in of %lld keys with %lld data values: each must be %lld or 1",
                     (long long)nkeys, (long long)ndata, (long long)n);
  if (n == 0) return JXR_OK;
  size_t bytes = 0;
  Bufs b;
  int rc = total_bytes(n, 1, 8, &bytes);
  if (rc) return rc;
  if ((rc = stage_in(&b, keys, 8 * (size_t)nkeys, data, 4 * (size_t)ndata, bytes))) return rc;
  rc = jxr_fold_in((const uint32_t*)b.keys, nkeys, (const uint32_t*)b.data, ndata,
                   (uint32_t*)b.out, NULL);
  return stage_out(&b, rc, host_out, bytes);
}

int jxs_prepare(uint32_t what) { return lib_status(jxr_prepare_device(what, NULL)); }
