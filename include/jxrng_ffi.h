/* XLA typed-FFI handlers over libjxrng (libjxrng_ffi.so), for ffi_register_target /
 * ffi_call (R/ffi.R:58-81, :241-319).  Each takes one argument, threefry2x32 key data
 * uint32[*batch, 2], and its result buffers; the attribute "partitionable" (bool, default
 * true) selects the counter layout; jxr_ffi_uniform also reads "minval" and "maxval", the
 * normal handlers "accurate_erf_inv" (bool), the bernoulli handlers "p" (a float32 or
 * float64 scalar, default 0.5 float32; its dtype is that of the compared uniform).
 *
 *   jxr_ffi_random_bits       platform "cuda": random_bits into a u8/u16/u32/u64 result
 *   jxr_ffi_random_bits_cpu   platform "cpu":  the same with host buffers (the GPU
 *                                              computes, through
 *                                              jxr_random_bits_host_static)
 *   jxr_ffi_uniform           platform "cuda": random_uniform, f32/f64/f16/bf16 result
 *   jxr_ffi_normal            platform "cuda": random_normal, f32/f64/f16/bf16 result
 *   jxr_ffi_bernoulli         platform "cuda": random_bernoulli (mode "low"), bool result
 *   jxr_ffi_normal_bernoulli  platform "cuda": random_normal(key, shape, dtype) and
 *                                              random_bernoulli(key, p, shape) of the same
 *                                              key, two results, one pass
 *
 * None of them allocates device memory or waits for XLA's stream.  They replace no
 * function of the reference: they are how its FFI interface would bind this library
 * inside jit (R/random.R:280-304, :482-508, :643-666 are what they compute).  The types
 * are those of XLA's FFI C API (xla/ffi/api/c_api.h). */
#ifndef JXRNG_FFI_H
#define JXRNG_FFI_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct XLA_FFI_Error XLA_FFI_Error;
typedef struct XLA_FFI_CallFrame XLA_FFI_CallFrame;

XLA_FFI_Error* jxr_ffi_random_bits(XLA_FFI_CallFrame* call_frame);
XLA_FFI_Error* jxr_ffi_random_bits_cpu(XLA_FFI_CallFrame* call_frame);
XLA_FFI_Error* jxr_ffi_uniform(XLA_FFI_CallFrame* call_frame);
XLA_FFI_Error* jxr_ffi_normal(XLA_FFI_CallFrame* call_frame);
XLA_FFI_Error* jxr_ffi_bernoulli(XLA_FFI_CallFrame* call_frame);
XLA_FFI_Error* jxr_ffi_normal_bernoulli(XLA_FFI_CallFrame* call_frame);

#ifdef __cplusplus
}
#endif
#endif
