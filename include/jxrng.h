/*
 * jxrng: B200 (sm_100a) kernels for jaxR's threefry2x32 random-bits path.
 *
 * A plain C ABI: pointers, sizes and status codes, no C++ or torch types, so the
 * R `.Call` shim, an XLA typed-FFI handler or Python ctypes can bind it alike.
 *
 * Conventions
 *  - Every entry point returns JXR_OK (0) or a status code; jxr_last_error()
 *    returns a message for the last failure on the calling host thread.
 *  - Arrays named `keys`, `out`, `x` ... are DEVICE pointers on the current
 *    CUDA device, owned by the caller.  Work is enqueued on `stream` (a
 *    cudaStream_t; NULL = the legacy default stream) and is asynchronous unless
 *    the entry point says otherwise.
 *  - A key is two uint32 words (k0, k1); `keys` holds `nkeys` keys, key j at
 *    keys[2j], keys[2j+1].  Key-batched entry points write one row per key
 *    (row-major, key-major), which is what vmap over a key batch produces.
 *  - Requests are given by `size`, the element count of one key's full request
 *    (the product of its shape), and the range [begin, begin + count) of it to
 *    produce.  Elements are in C order, exactly as the reference's outputs, so
 *    a caller can shard a request over devices by element range and each
 *    device writes its own slab; begin = 0, count = size is the whole request.
 *  - layout selects jax_threefry_partitionable: JXR_LAYOUT_PARTITIONABLE (the
 *    reference's default) or JXR_LAYOUT_ORIGINAL.
 *  - Entry points allocate no device memory and do not wait for the stream unless
 *    their comment says so: jxr_prepare_device (set-up), jxr_free_caches, the HOST-memory
 *    entry points jxr_random_bits_host / _host_static, and jxr_shuffle /
 *    jxr_shuffle_lanes / jxr_argsort_float, which synchronise to read a bounds-check flag
 *    (their scratch comes from the caller).
 *
 * Reference interfaces replaced (paths within the jaxR project):
 *  - threefry2x32_p and its lowering           R/prng.R:48-99
 *  - prng_threefry_2x32 (hash of counts)        R/prng.R:101-120
 *  - prng_threefry_seed                         R/prng.R:159-170
 *  - prng_threefry_split (both layouts)         R/prng.R:172-191
 *  - prng_threefry_fold_in                      R/prng.R:193-194
 *  - prng_threefry_random_bits (both layouts)   R/prng.R:201-262
 *  - rnd_uniform                                R/random.R:287-304
 *  - rnd_normal_real / lax_erf_inv              R/random.R:501-508, R/lax.R:222
 *  - rnd_bernoulli (mode "low")                 R/random.R:655-666
 * The reference reaches these through .Call(jaxr_compile/jaxr_execute)
 * (src/pjrt.cpp:255, :725) on the XLA CPU plugin; a .Call shim over this ABI
 * replaces them.
 */
#ifndef JXRNG_H
#define JXRNG_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JXR_ABI_VERSION 1

/* status codes */
enum {
  JXR_OK = 0,
  JXR_ERR_INVALID_ARGUMENT = 1, /* bad size, range, dtype, layout, bit width, pointer */
  JXR_ERR_NOT_IMPLEMENTED = 2,  /* e.g. a request of more than 2^64 elements */
  JXR_ERR_CUDA = 3,             /* a CUDA runtime call failed; message has the CUDA error */
  JXR_ERR_NO_DEVICE = 4         /* no sm_100 device is current */
};

/* layouts: the value of jax_threefry_partitionable */
enum { JXR_LAYOUT_ORIGINAL = 0, JXR_LAYOUT_PARTITIONABLE = 1 };

/* key implementations (R/prng.R:430-440) */
enum { JXR_IMPL_THREEFRY = 0, JXR_IMPL_RBG = 1, JXR_IMPL_UNSAFE_RBG = 2 };

/* floating dtypes (16-bit results are stored as their raw bits) */
enum { JXR_F32 = 0, JXR_F64 = 1, JXR_F16 = 2, JXR_BF16 = 3 };

/* flags for jxr_uniform: the reference's recorded samples (tests/testthat/
 * test-random.R:43, :160) are those of a fused floats*(maxval-minval)+minval;
 * this flag asks for a separately rounded multiply and add instead. */
enum { JXR_FLAG_UNFUSED_MUL_ADD = 1 };

/* jax_accurate_erf_inv (R/config.R:18; R/lax_special.R:1326-1331 lowers erf_inv to JAX's
 * erf_inv_core, R/lax_special.R:1022-1082, when it is set): for the calling host thread,
 * selects the erf_inv that jxr_normal, jxr_normal_from_bits, jxr_normal_bernoulli, the
 * jxr_truncated_normal family and jxr_erf_inv evaluate.  Off (0) by default, as in the
 * reference; the setter returns the previous value.  The choice is made when a call
 * launches its kernels. */
int jxr_set_accurate_erf_inv(int enable);
int jxr_get_accurate_erf_inv(void);

/* Set-up of the current device, the one call that allocates on purpose; do it once per
 * device, before any stream capture and before a host framework reserves the GPU for its
 * own memory pool.  Synchronous: waits for `stream`; refused (JXR_ERR_INVALID_ARGUMENT)
 * while `stream` is being captured into a CUDA graph.
 *  - Every call loads this library's module on the device (CUDA loads modules and their
 *    kernels lazily, on first use), looks up the array of jxr_random_bits_host_static and
 *    loads every kernel that entry point launches: the module's fixed 16 MiB + 32 KiB
 *    array and that code are created then, not inside a later call.
 *  - `what` (JXR_PREPARE_* bits, 0 for none) names the samplers whose lookup tables to
 *    build: per sampler a float32 table of its 2^23 possible results (32 MiB) and the
 *    float16 / bfloat16 tables of its 1024 / 128 results (2 KiB + 256 B).  Every float32
 *    sample depends only on bits >> 9 of its draw, every 16-bit one on the top 10 / 7
 *    bits, so a table holds the sampler's exact results.
 * Sampling entry points never allocate, build a table or wait: a prepared table is read
 * by requests of 2^22 or more float32 samples (jxr_normal, jxr_sample and their _from_bits
 * forms) or 2^16 or more 16-bit samples, which then run about twice as fast; without it
 * every sample is evaluated directly, with identical results. */
enum {
  JXR_PREPARE_TABLE_NORMAL = 1u << 0,          /* normal, default erf_inv */
  JXR_PREPARE_TABLE_NORMAL_ACCURATE = 1u << 1, /* normal under jax_accurate_erf_inv */
  JXR_PREPARE_TABLE_EXPONENTIAL = 1u << 2,     /* jxr_sample kinds 0..3, in order */
  JXR_PREPARE_TABLE_GUMBEL = 1u << 3,
  JXR_PREPARE_TABLE_LOGISTIC = 1u << 4,
  JXR_PREPARE_TABLE_LAPLACE = 1u << 5,
  JXR_PREPARE_ALL = 0x3F
};
int jxr_prepare_device(uint32_t what, void* stream);

/* Frees the current device's caches: the samplers' tables that jxr_prepare_device built,
 * jxr_random_bits_host's staging buffers, streams and events, and the cached address of
 * jxr_random_bits_host_static's array (looked up again by the next call).  Waits for the
 * device first.  Call it before cudaDeviceReset or to return the memory. */
int jxr_free_caches(void);

/* ABI version (JXR_ABI_VERSION) and the last error of this host thread. */
int jxr_abi_version(void);
const char* jxr_last_error(void);

/* Seeds to keys on the host (R/prng.R:159-170 after R/prng.R:504-519): with x64
 * off an R number wraps to int32 and k0 is 0; with x64 on k0 is the high word.
 * keys_out: HOST uint32[2 * n]. */
int jxr_seed(const int64_t* seeds, int64_t n, int x64, uint32_t* keys_out);

/* threefry2x32_p on n broadcast elements (R/prng.R:88-99). */
int jxr_threefry2x32(const uint32_t* k0, const uint32_t* k1, const uint32_t* c0,
                     const uint32_t* c1, uint32_t* x0, uint32_t* x1, int64_t n,
                     void* stream);

/* prng_threefry_2x32(key, count) for each of nkeys keys over one uint32 count
 * vector of n elements, with odd-n zero padding (R/prng.R:101-120).
 * out: uint32[nkeys][n]. */
int jxr_threefry_2x32(const uint32_t* keys, int64_t nkeys, const uint32_t* count, int64_t n,
                      uint32_t* out, void* stream);

/* random_split of each key into num keys (R/prng.R:172-191).
 * out: uint32[nkeys][num][2]. */
int jxr_split(const uint32_t* keys, int64_t nkeys, int64_t num, int layout, uint32_t* out,
              void* stream);

/* random_fold_in (R/prng.R:193-194): out key i = fold_in(keys[i or 0], data[i or 0]),
 * n = max(nkeys, ndata); nkeys and ndata are each n or 1. out: uint32[n][2]. */
int jxr_fold_in(const uint32_t* keys, int64_t nkeys, const uint32_t* data, int64_t ndata,
                uint32_t* out, void* stream);

/* random_bits (R/prng.R:201-262): bit_width 8, 16, 32 or 64; out holds
 * uint{bit_width}[nkeys][count], elements [begin, begin+count) of each key's
 * size-element request. */
int jxr_random_bits(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                    uint64_t count, int layout, int bit_width, void* out, void* stream);

/* random_uniform (R/random.R:287-304) in dtype with scalar bounds given as double
 * and converted to dtype first. out: dtype[nkeys][count]. */
int jxr_uniform(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                uint64_t count, int layout, int dtype, double minval, double maxval,
                uint32_t flags, void* out, void* stream);

/* random_normal for a real dtype (R/random.R:501-508): sqrt(2) * erf_inv(u) with u
 * uniform on [nextafter(-1, 0), 1). out: dtype[nkeys][count].  Large float32 / 16-bit
 * requests read the sampler's table when jxr_prepare_device has built it (same results). */
int jxr_normal(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
               uint64_t count, int layout, int dtype, void* out, void* stream);

/* random_bernoulli, mode "low" (R/random.R:655-666): uniform(dtype(p)) < p.
 * out: uint8 (0/1)[nkeys][count]. */
int jxr_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                  uint64_t count, int layout, int p_dtype, double p, uint8_t* out,
                  void* stream);

/* random_normal(key, shape, dtype) and random_bernoulli(key, p, shape) of the SAME
 * key and shape in one pass: both draw the same bits, so the cipher runs once.
 * normal_out: dtype[nkeys][count]; bern_out: uint8[nkeys][count]. */
int jxr_normal_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                         uint64_t count, int layout, int dtype, double p, void* normal_out,
                         uint8_t* bern_out, void* stream);

/* The sampler transforms alone, applied element-wise to caller-provided random
 * bits (the second half of rnd_uniform / rnd_normal_real, R/random.R:297-304,
 * :505-507): bits are uint32 for F32, uint64 for F64, uint16 for F16 and uint8
 * for BF16, as rnd_bits draws them. */
int jxr_uniform_from_bits(const void* bits, int64_t n, int dtype, double minval,
                          double maxval, uint32_t flags, void* out, void* stream);
int jxr_normal_from_bits(const void* bits, int64_t n, int dtype, void* out, void* stream);

/* Array-valued parameters, applied to unit draws u = uniform(key, shape, dtype, 0, 1)
 * (which are the unit floats themselves), all arrays of n elements of dtype:
 *  - uniform with per-element bounds (R/random.R:297-303, bounds broadcast by the
 *    caller): out = max(minval, u * (maxval - minval) + minval);
 *  - bernoulli with per-element p (R/random.R:656-666): mode "low" (u_hi == NULL)
 *    out = u_lo < p; mode "high" out = u_hi * 2^-nmant < p - u_lo, where u_lo and
 *    u_hi are the two halves of uniform(key, (2, shape)).  out: uint8 0/1. */
int jxr_uniform_affine(const void* unit, const void* minval, const void* maxval, int64_t n,
                       int dtype, uint32_t flags, void* out, void* stream);
/* jxr_uniform_affine over nrows rows of n unit draws (unit, out: dtype[nrows][n], a key
 * batch's rows) with one row of bounds (minval, maxval: dtype[n]) for every row, in one
 * launch. */
int jxr_uniform_affine_rows(const void* unit, const void* minval, const void* maxval,
                            int64_t nrows, int64_t n, int dtype, uint32_t flags, void* out,
                            void* stream);
int jxr_bernoulli_from_uniform(const void* u_lo, const void* u_hi, const void* p, int64_t n,
                               int dtype, uint8_t* out, void* stream);

/* The log-transform samplers (R/random.R:1422-1516) fused like jxr_uniform, kind:
 * 0 exponential -log1p(-u); 1 gumbel (mode "low") -log(-log(u)), u from (tiny, 1);
 * 2 logistic log(x) - log1p(-x), x from (tiny, 1); 3 laplace sign(u) log1p(-|u|),
 * u from (-1 + 2^-(nmant+1), 1).  out: dtype[nkeys][count].  Large float32 / 16-bit
 * requests read the sampler's table when jxr_prepare_device has built it (same results). */
int jxr_sample(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
               uint64_t count, int layout, int kind, int dtype, void* out, void* stream);
/* The same transforms of n random_bits values (the dtype's draw width: 32/64/16/8 bits for
 * float32/float64/float16/bfloat16), e.g. the bits of an rbg key. */
int jxr_sample_from_bits(const void* bits, int64_t n, int kind, int dtype, void* out,
                         void* stream);

/* randint (R/random.R:306-359) with scalar bounds in one pass, partitionable layout:
 * keys_hi / keys_lo are the two halves of split(key) for each of nkeys keys (u32[nkeys][2]
 * each); minval / maxval are the bounds clipped to the sampling dtype (nbits = 32 or 64,
 * signed if is_signed), sign- or zero-extended; out_of_range says maxval exceeded the
 * dtype's maximum.  Writes the low out_bits of each sample, out: [nkeys][count]. */
int jxr_randint(const uint32_t* keys_hi, const uint32_t* keys_lo, int64_t nkeys, uint64_t size,
                uint64_t begin, uint64_t count, int nbits, int is_signed, int64_t minval,
                int64_t maxval, int out_of_range, int out_bits, void* out, void* stream);

/* randint (R/random.R:306-359) from its two draws: hi and lo are nbits-bit (32 or 64)
 * random_bits of the two halves of split(key); minval/maxval are the bounds already
 * clipped and converted to the sampling dtype (signed if is_signed), sign- or
 * zero-extended to int64; out_of_range flags where maxval exceeded that dtype's maximum.
 * Each parameter array has stride 0 (one value for all) or 1.  Writes the low out_bits of
 * minval + ((hi % span) * (2^nbits % span) + lo % span) % span. */
int jxr_randint_combine(const void* hi, const void* lo, int64_t n, int nbits, int is_signed,
                        const int64_t* minval, int64_t minval_stride, const int64_t* maxval,
                        int64_t maxval_stride, const uint8_t* out_of_range, int64_t oor_stride,
                        int out_bits, void* out, void* stream);

/* gumbel modes "high" and "highest" (R/random.R:1465-1489) from the two rows of a (2, n)
 * draw of one key: mode 0 ("high") takes uniforms of dtype, mode 1 ("highest", float32
 * only) 32-bit random_bits.  out: dtype[n]. */
int jxr_gumbel_rows(const void* row0, const void* row1, int64_t n, int mode, int dtype,
                    void* out, void* stream);

/* random_truncated_normal (R/random.R:586-603) with scalar bounds: uniform(erf(lower/sqrt2),
 * erf(upper/sqrt2)), sqrt(2) erf_inv, clipped to the open interval; the two erf values are
 * computed on the host once per call. */
int jxr_truncated_normal(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                         uint64_t count, int layout, int dtype, double lower, double upper,
                         void* out, void* stream);
/* jxr_truncated_normal with caller-provided scratch (device memory, 16-byte aligned):
 * float32 requests of 2^25 or more samples with at least 32 MiB of scratch build, in the
 * call, the table of the sampler at all 2^23 values it can take (each sample depends
 * only on bits >> 9 of its draw) and read most samples from it; float16 / bfloat16
 * requests of 2^16 or more samples with at least 2 KiB of scratch do the same with their
 * 1024 / 128 possible results.  The results are those of jxr_truncated_normal, which
 * every other request calls. */
int jxr_truncated_normal_scratch(const uint32_t* keys, int64_t nkeys, uint64_t size,
                                 uint64_t begin, uint64_t count, int layout, int dtype,
                                 double lower, double upper, void* scratch, size_t scratch_bytes,
                                 void* out, void* stream);
int jxr_truncated_normal_from_bits(const void* bits, int64_t n, int dtype, double lower,
                                   double upper, void* out, void* stream);

/* random_truncated_normal with per-element bounds: unit is the uniform(0, 1) draw of the
 * key (dtype[n]); lower and upper are dtype arrays with stride 0 (one value) or 1.  The erf
 * of the bounds is evaluated on the device (CUDA's erf in double, rounded to dtype). */
int jxr_truncated_normal_from_unit(const void* unit, const void* lower, int64_t lower_stride,
                                   const void* upper, int64_t upper_stride, int64_t n, int dtype,
                                   void* out, void* stream);

/* The shuffle of random_permutation (rnd_shuffle, R/random.R:402-413) over an array of
 * shape (outer, n, inner), shuffling each 1-D slice along the middle axis (outer = inner = 1
 * for a vector).  Writes perm[f] = the flat index of the source element that lands at flat
 * position f (total = outer * n * inner < 2^31).  Each of the ceil(3 log(total) /
 * log(2^32 - 1)) rounds splits the key, draws 32-bit sort keys and sorts stably: radix
 * passes over the keys' top bits, then every run of equal top bits sorted in shared memory
 * (the span sort).  scratch (256-byte aligned) holds jxr_shuffle_scratch_bytes(total)
 * bytes.  Synchronises `stream` to read back the sort's flags; if a run was longer than
 * the span sort takes (which uniformly random keys make vanishingly unlikely), the shuffle
 * is repeated with radix passes alone before the call returns.  impl: the key's
 * implementation (JXR_IMPL_*; key is u32[2] for threefry2x32, u32[4] for rbg and
 * unsafe_rbg). */
size_t jxr_shuffle_scratch_bytes(int64_t total);
int jxr_shuffle(const uint32_t* key, int impl, int64_t outer, int64_t n, int64_t inner,
                int layout, uint32_t* perm, void* scratch, size_t scratch_bytes, void* stream);
/* rnd_shuffle under vmap with rbg or unsafe_rbg keys (R/random.R:402-413 with the batching
 * rule of rng_bit_generator, R/prng.R:300-313: every lane's bits come from the first lane's
 * key, lane i taking row i of one (nlanes, shape) request).  key is the first lane's u32[4]
 * key; perm (nlanes x total) gets, per lane, the flat source index of each position of an
 * (outer, n, inner) array shuffled along the middle axis, as jxr_shuffle does for one key.
 * scratch (256-byte aligned) holds jxr_shuffle_lanes_scratch_bytes(nlanes, total) bytes.
 * Synchronises `stream` to read back the sort's flags. */
size_t jxr_shuffle_lanes_scratch_bytes(int64_t nlanes, int64_t total);
int jxr_shuffle_lanes(const uint32_t* key, int impl, int64_t nlanes, int64_t outer, int64_t n,
                      int64_t inner, int layout, uint32_t* perm, void* scratch,
                      size_t scratch_bytes, void* stream);
/* The longest span (elements) the span sort of jxr_shuffle takes, for the calling host
 * thread: 4096 by default, 0 = radix passes only, anything in [0, 4096] accepted; returns
 * the previous value, or -1 (and the message for jxr_last_error) for a value outside that
 * range.  Shorter caps exercise the repeat by radix passes; the results are identical
 * either way. */
int jxr_set_shuffle_span_cap(int cap);

/* jnp_take along the middle axis: out[o][i][:] = src[o][idx[i]][:], rows of row_bytes bytes,
 * src of shape (outer, n_src, row), out (outer, n_idx, row).  An index >= n_src is skipped
 * and, if err (device int) is given, sets *err = 4. */
int jxr_take(const void* src, int64_t outer, int64_t n_src, const uint32_t* idx, int64_t n_idx,
             int64_t row_bytes, void* out, int* err, void* stream);

/* random_choice with p (R/random.R:440-459).  With replacement: from unit = uniform(0, 1)
 * draws (dtype float32/float64, n of them) and the cumulative sums cuml (m >= 1, dtype),
 * out[i] = searchsorted_left(cuml, cuml[m-1] * (1 - unit[i])) as int32 or int64
 * (out_bits).  Without replacement: x = gumbel draws, jxr_add_log adds log(p) in place,
 * and jxr_argsort_float (stable; descending for top_k, ties to the lower index) orders
 * them; -0 sorts as +0.  scratch: 256-byte aligned, jxr_argsort_scratch_bytes(n) bytes. */
int jxr_choice_p_from_unit(const void* unit, int64_t n, int dtype, const void* cuml, int64_t m,
                           int out_bits, void* out, void* stream);
int jxr_add_log(void* x, const void* p, int64_t n, int dtype, void* stream);
size_t jxr_argsort_scratch_bytes(int64_t n);
int jxr_argsort_float(const void* x, int64_t n, int dtype, int descending, uint32_t* idx,
                      void* scratch, size_t scratch_bytes, void* stream);

/* The rbg and unsafe_rbg implementations (R/prng.R:382-426): XLA's RngBitGenerator,
 * Philox4x32-10 with key (k0, k1) and 128-bit counter k0 | k1 << 32 | k2 << 64 | k3 << 96
 * advanced by one per block of four 32-bit outputs (key: a device u32[4]).
 * jxr_rbg_bits: elements [begin, begin + count) of a size-element request of bit_width-bit
 * values (8/16 take the low bits of one 32-bit output per element, 64 two outputs, low
 * first); new_key (device u32[4], may be NULL) receives the state after the whole request.
 * jxr_rbg_blocks: blocks first + i * stride, i < n, 4 words each (unsafe_rbg split).
 * jxr_rbg_unsafe_fold_in: keys[i] ^ row 9 of the (10, 4) request of rbg_seed(data[i]);
 * keys u32[nkeys][4], data u32[ndata], broadcasting; lanes_from_first != 0 draws output i
 * from row 9 + 10 i of data[0]'s request (rng_bit_generator under vmap). */
int jxr_rbg_bits(const uint32_t* key, uint64_t size, uint64_t begin, uint64_t count, int bit_width,
                 void* out, uint32_t* new_key, void* stream);
int jxr_rbg_blocks(const uint32_t* key, uint64_t first, uint64_t stride, int64_t n, uint32_t* out,
                   void* stream);
int jxr_rbg_unsafe_fold_in(const uint32_t* keys, int64_t nkeys, const uint32_t* data, int64_t ndata,
                           int lanes_from_first, uint32_t* out, void* stream);

/* random_bits over several GPUs from one process (the R session): device i of ndev
 * computes elements [size * i / ndev, size * (i + 1) / ndev) of the request of one
 * threefry key (keys[i]: that key's u32[2] on device i), on streams[i] (or the default
 * stream).  With gather_to < 0 device i writes its slab to outs[i] (its own memory); with
 * gather_to = g, every device's kernel stores its slab straight into gather_out (size
 * elements on device g) through peer access over NVLink.  Asynchronous: synchronise the
 * streams to wait.  The current device is left as it was. */
int jxr_random_bits_multi(const int* devices, int ndev, const uint32_t* const* keys, uint64_t size,
                          int layout, int bit_width, void* const* outs, int gather_to,
                          void* gather_out, void* const* streams);

/* Complex normals (R/random.R:489-499): out (complex64 / complex128, interleaved) =
 * (re[i] + i im[i]) / divisor, each part divided in the real dtype (float32/float64). */
int jxr_complex_from_parts(const void* re, const void* im, int64_t n, int dtype, double divisor,
                           void* out, void* stream);

/* Cumulative sum of m float32/float64 values, added left to right in the dtype (the
 * probabilities of random_choice, R/random.R:446). */
int jxr_cumsum(const void* x, int64_t m, int dtype, void* out, void* stream);

/* lax_erf_inv (R/lax.R:222, lowered as chlo.erf_inv at R/lax_special.R:1327-1331),
 * element-wise for F32 or F64. */
int jxr_erf_inv(const void* x, int64_t n, int dtype, void* out, void* stream);

/* random_bits into HOST memory: generates on the current device in 64 MiB chunks into
 * device staging buffers and copies each chunk to host_out while the next one is
 * generated.  Synchronous: returns when host_out holds the result.  host_out should be
 * pinned (cudaHostAlloc or cudaHostRegister) for full PCIe bandwidth.  The staging
 * buffers (2 x 64 MiB), a device copy of the keys and two streams are created on the
 * first call on a device and kept for later calls; calls on one device run one at a
 * time. */
int jxr_random_bits_host(const uint32_t* keys_host, int64_t nkeys, uint64_t size,
                         uint64_t begin, uint64_t count, int layout, int bit_width,
                         void* host_out);

/* ---- measurement hook (for bench.py's roofline; not part of the sampling API) ----
 * Throughput probe: launches (number of SMs) x ctas_per_sm CTAs of 256 threads that
 * each push 8 register-resident blocks through `iters` threefry20 passes (no counters,
 * loads or stores) and returns in *blocks_out the number of cipher blocks that launch
 * computes; sink needs (number of SMs) x ctas_per_sm x 256 uint32.  Timing it gives the
 * cipher's integer-pipe ceiling on this GPU (the roofline of the bits kernels). */
int jxr_probe_cipher(uint64_t iters, int ctas_per_sm, uint32_t* sink, uint64_t* blocks_out,
                     void* stream);

/* Device memory shared between the processes of one node, so that a bits kernel on one
 * GPU can write its shard of a request straight into another GPU's buffer over NVLink
 * (plain stores through a peer mapping), for callers who want a whole request on one
 * device.  jxr_ipc_export: a 64-byte handle for the
 * allocation holding dev_ptr and dev_ptr's offset into it.  jxr_ipc_open: map a handle
 * exported by another process (peer access enabled lazily); add the offset to the
 * returned base.  jxr_ipc_close: unmap.  No counterpart in the reference, which runs on
 * one device (src/pjrt.cpp:751). */
int jxr_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset);
int jxr_ipc_open(const void* handle, void** base_out);
int jxr_ipc_close(void* base);

/* random_bits into HOST memory without allocating anything.  Some callers cannot
 * allocate device memory while they run: a host framework that has reserved (nearly)
 * all of the GPU for its own memory pool, as XLA's PJRT client does when it runs an FFI
 * handler, where a cudaMalloc fails or stalls the device behind the framework's back.
 * This variant of jxr_random_bits_host uses no cudaMalloc, cudaFree or any other
 * allocating call: its device scratch is one array of fixed size compiled into the
 * library (4096 keys + a 16 MiB staging buffer, 16 MiB + 32 KiB in all), held on every
 * GPU that loads the library until the process exits.  It has no counterpart in the
 * reference.
 *  - nkeys may be at most 4096; larger batches are rejected with
 *    JXR_ERR_INVALID_ARGUMENT.  count is produced in 16 MiB chunks, any length.
 *  - Work is ordered on `stream` (NULL = legacy default stream) and the call returns
 *    when host_out holds the result, also when it fails part way.
 *  - Set-up: the array exists once the library's module is loaded on the device, and
 *    CUDA loads modules lazily, on the library's first use there.  If a call of this
 *    entry point is that first use, the module (its code and this array) is created
 *    inside the call, i.e. allocated.  So call jxr_prepare_device once per device at
 *    set-up, before the framework reserves its memory pool and before any stream capture:
 *    it loads the module and this entry point's kernels and looks up the array's device
 *    address (cudaGetSymbolAddress).  Otherwise the first call on a device does that.
 *  - Every call on a device shares the one array, which keeps the last call's contents
 *    (nothing in it needs to start at zero: keys and staging are rewritten before they
 *    are read).  Calls that overlap on the GPU would race on it; the library holds a lock
 *    per device for the whole of each call (which ends with its stream synchronised), so
 *    calls from several host threads of one process take turns. */
int jxr_random_bits_host_static(const uint32_t* keys_host, int64_t nkeys, uint64_t size,
                                uint64_t begin, uint64_t count, int layout, int bit_width,
                                void* host_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* JXRNG_H */
