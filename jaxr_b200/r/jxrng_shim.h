/* The R-independent core of jaxR's .Call shim over libjxrng (jxrng_r.c holds the R glue).
 *
 * jaxR's arrays live on its XLA CPU device, i.e. in host memory, so each call takes its
 * keys and returns its result in host memory, computing on the current CUDA device in
 * between: keys up, the libjxrng kernel, the result down.  Every function here
 *  - returns 0 (JXR_OK) or a libjxrng status code, with jxs_error() giving the message;
 *  - allocates its device buffers with cudaMalloc and frees them before it returns, on
 *    success and on every failure, so the R glue may call Rf_error (a longjmp) right after
 *    a failed call without leaking (jaxR's own rule for .Call code, src/pjrt.cpp:568-570);
 *  - waits for its work (results are in host_out on return).
 * Counts arrive from R as doubles (R has no 64-bit integers): jxs_count admits only finite,
 * integral values in [0, 2^53], beyond which doubles stop being exact. */
#ifndef JXRNG_SHIM_H
#define JXRNG_SHIM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The message of this thread's last failure (the shim's own, or libjxrng's). */
const char* jxs_error(void);

/* An R count (a double) as an integer: finite, integral and in [0, 2^53], else
 * JXR_ERR_INVALID_ARGUMENT naming `what`. */
int jxs_count(double x, const char* what, uint64_t* out);

/* Key words given as R doubles (each an integer in [0, 2^32)) as uint32; nwords is even
 * (two words per threefry2x32 key). */
int jxs_key_words(const double* words, int64_t nwords, uint32_t* out);

/* Host bytes of n elements of `elem_bytes` bytes, checked against size_t overflow. */
int jxs_bytes(uint64_t n, uint64_t elem_bytes, size_t* out);

/* random_bits of each of nkeys keys (R/prng.R:201-262): host_out receives
 * uint{bit_width}[nkeys][size], little-endian. */
int jxs_random_bits(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout,
                    int bit_width, void* host_out);

/* random_uniform (R/random.R:287-304), dtype a JXR_F* code; 16-bit results are raw bits. */
int jxs_uniform(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout, int dtype,
                double minval, double maxval, void* host_out);

/* random_normal for a real dtype (R/random.R:501-508); accurate selects
 * jax_accurate_erf_inv's erf_inv for this call. */
int jxs_normal(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout, int dtype,
               int accurate, void* host_out);

/* random_bernoulli, mode "low" (R/random.R:655-666): host_out receives uint8 0/1. */
int jxs_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, int layout, int p_dtype,
                  double p, uint8_t* host_out);

/* random_split of each key into num keys (R/prng.R:172-191): uint32[nkeys][num][2]. */
int jxs_split(const uint32_t* keys, int64_t nkeys, uint64_t num, int layout, uint32_t* host_out);

/* random_fold_in (R/prng.R:193-194): n = max(nkeys, ndata) keys, each of nkeys and ndata
 * being n or 1: uint32[n][2]. */
int jxs_fold_in(const uint32_t* keys, int64_t nkeys, const uint32_t* data, int64_t ndata,
                uint32_t* host_out);

/* Set-up of the current device (jxr_prepare_device): loads libjxrng's module and builds
 * the samplers' lookup tables named in `what` (JXR_PREPARE_* bits). */
int jxs_prepare(uint32_t what);

#ifdef __cplusplus
}
#endif
#endif /* JXRNG_SHIM_H */
