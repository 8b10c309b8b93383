// XLA typed-FFI handlers over libjxrng: the kernels made callable from jit-compiled jaxR
// programs through ffi_register_target / ffi_call (R/ffi.R:58-81, :241-319), written
// against XLA's FFI C API (the subset in xla_ffi_abi.h, or xla/ffi/api/c_api.h itself
// when JXR_FFI_XLA_HEADER is defined).
//
//   jxr_ffi_random_bits       platform "cuda"  key u32[..., 2] and the result on the
//                                              device, launched on XLA's stream
//   jxr_ffi_random_bits_cpu   platform "cpu"   key and result in host memory (the CPU PJRT
//                                              plugin jaxR runs on); the GPU computes the
//                                              bits through jxr_random_bits_host_static,
//                                              which allocates nothing
//   jxr_ffi_uniform           platform "cuda"  float result, attributes minval, maxval
//   jxr_ffi_normal            platform "cuda"  float result, attribute accurate_erf_inv
//   jxr_ffi_bernoulli         platform "cuda"  bool (pred) result, attribute p
//   jxr_ffi_normal_bernoulli  platform "cuda"  two results of one key and shape, a float
//                                              normal and a bool bernoulli(p) from the same
//                                              draws, in one pass
//
// One argument, the key buffer (threefry2x32 data, u32[*batch, 2]: one key per batch row,
// as ffi_call's vmap methods deliver them); the results, whose dtype gives the bit width
// or the float type and whose element count divided by the number of keys gives each
// key's request.  Attribute "partitionable" (a bool scalar; the value of
// jax_threefry_partitionable, default true) selects the counter layout, and
// "accurate_erf_inv" (a bool scalar; jax_accurate_erf_inv, default false) the normal's
// erf_inv.  Attribute "p" (a float32 or float64 scalar, default 0.5 float32) is the
// bernoulli probability; its dtype is the dtype of the uniform it is compared with
// (R/random.R:655-666), as the dtype of p is in the reference.  Errors come back as XLA
// FFI errors carrying the library's message.  No handler allocates device memory or waits
// for XLA's stream.

#include <cstring>

#include "jxrng.h"
#ifdef JXR_FFI_XLA_HEADER
#include "xla/ffi/api/c_api.h"
#else
#include "xla_ffi_abi.h"
#endif

namespace {

XLA_FFI_Error* error(const XLA_FFI_Api* api, XLA_FFI_Error_Code code, const char* msg) {
  XLA_FFI_Error_Create_Args a;
  std::memset(&a, 0, sizeof(a));
  a.struct_size = XLA_FFI_Error_Create_Args_STRUCT_SIZE;
  a.message = msg;
  a.errc = code;
  return api->XLA_FFI_Error_Create(&a);
}

// XLA first calls a handler with a metadata extension to learn its API version and traits.
bool answer_metadata(XLA_FFI_CallFrame* cf) {
  XLA_FFI_Extension_Base* ext = cf->extension_start;
  if (!ext || ext->type != XLA_FFI_Extension_Metadata) return false;
  XLA_FFI_Metadata* m = reinterpret_cast<XLA_FFI_Metadata_Extension*>(ext)->metadata;
  m->api_version.major_version = XLA_FFI_API_MAJOR;
  m->api_version.minor_version = XLA_FFI_API_MINOR;
  m->traits = 0;
  return true;
}

struct Frame {
  const XLA_FFI_Buffer* key = nullptr;
  const XLA_FFI_Buffer* out = nullptr;   // the (first) result
  const XLA_FFI_Buffer* out2 = nullptr;  // the second result, where the handler has one
  int64_t nkeys = 0, out_elems = 0;
  int layout = JXR_LAYOUT_PARTITIONABLE;
  int accurate_erf_inv = 0;
  double minval = 0.0, maxval = 1.0;
  double p = 0.5;
  int p_dtype = JXR_F32;
};

int64_t elements(const XLA_FFI_Buffer* b) {
  int64_t n = 1;
  for (int64_t i = 0; i < b->rank; ++i) n *= b->dims[i];
  return n;
}

bool name_is(const XLA_FFI_ByteSpan* s, const char* name) {
  return s->len == std::strlen(name) && std::memcmp(s->ptr, name, s->len) == 0;
}

double scalar_value(const XLA_FFI_Scalar* sc) {
  switch (sc->dtype) {
    case XLA_FFI_DataType_PRED: return *static_cast<const uint8_t*>(sc->value) ? 1.0 : 0.0;
    case XLA_FFI_DataType_S32: return *static_cast<const int32_t*>(sc->value);
    case XLA_FFI_DataType_S64: return (double)*static_cast<const int64_t*>(sc->value);
    case XLA_FFI_DataType_F32: return *static_cast<const float*>(sc->value);
    case XLA_FFI_DataType_F64: return *static_cast<const double*>(sc->value);
    default: return 0.0;
  }
}

// Checks and decodes the frame: one u32[..., 2] key buffer, `nrets` result buffers of one
// element count, scalar attributes.  Returns nullptr on success.
XLA_FFI_Error* decode(XLA_FFI_CallFrame* cf, int nrets, Frame* f) {
  const XLA_FFI_Api* api = cf->api;
  if (cf->args.size != 1 || cf->args.types[0] != XLA_FFI_ArgType_BUFFER)
    return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT, "jxrng: expected one key buffer argument");
  if (cf->rets.size != nrets)
    return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                 nrets == 1 ? "jxrng: expected one result buffer"
                            : "jxrng: expected two result buffers (normal, bernoulli)");
  for (int i = 0; i < nrets; ++i)
    if (cf->rets.types[i] != XLA_FFI_RetType_BUFFER)
      return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT, "jxrng: results must be buffers");
  f->key = static_cast<const XLA_FFI_Buffer*>(cf->args.args[0]);
  f->out = static_cast<const XLA_FFI_Buffer*>(cf->rets.rets[0]);
  if (nrets == 2) {
    f->out2 = static_cast<const XLA_FFI_Buffer*>(cf->rets.rets[1]);
    if (elements(f->out2) != elements(f->out))
      return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                   "jxrng: the two results must have the same number of elements");
  }
  if (f->key->dtype != XLA_FFI_DataType_U32 || f->key->rank < 1 ||
      f->key->dims[f->key->rank - 1] != 2)
    return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                 "jxrng: the key must be threefry2x32 key data, uint32[..., 2]");
  f->nkeys = elements(f->key) / 2;
  f->out_elems = elements(f->out);
  if (f->nkeys < 1 || f->out_elems % f->nkeys)
    return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                 "jxrng: the result's element count is not a multiple of the number of keys");
  for (int64_t i = 0; i < cf->attrs.size; ++i) {
    if (cf->attrs.types[i] != XLA_FFI_AttrType_SCALAR) continue;
    const auto* sc = static_cast<const XLA_FFI_Scalar*>(cf->attrs.attrs[i]);
    const XLA_FFI_ByteSpan* name = cf->attrs.names[i];
    if (name_is(name, "partitionable"))
      f->layout = scalar_value(sc) != 0.0 ? JXR_LAYOUT_PARTITIONABLE : JXR_LAYOUT_ORIGINAL;
    else if (name_is(name, "accurate_erf_inv")) f->accurate_erf_inv = scalar_value(sc) != 0.0;
    else if (name_is(name, "minval")) f->minval = scalar_value(sc);
    else if (name_is(name, "maxval")) f->maxval = scalar_value(sc);
    else if (name_is(name, "p")) {
      if (sc->dtype != XLA_FFI_DataType_F32 && sc->dtype != XLA_FFI_DataType_F64)
        return error(api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                     "jxrng: attribute p must be a float32 or float64 scalar");
      f->p = scalar_value(sc);
      f->p_dtype = sc->dtype == XLA_FFI_DataType_F64 ? JXR_F64 : JXR_F32;
    }
  }
  return nullptr;
}

bool is_bool(XLA_FFI_DataType t) { return t == XLA_FFI_DataType_PRED || t == XLA_FFI_DataType_U8; }

int bits_of(XLA_FFI_DataType t) {
  switch (t) {
    case XLA_FFI_DataType_U8: return 8;
    case XLA_FFI_DataType_U16: return 16;
    case XLA_FFI_DataType_U32: return 32;
    case XLA_FFI_DataType_U64: return 64;
    default: return 0;
  }
}

int float_code(XLA_FFI_DataType t) {
  switch (t) {
    case XLA_FFI_DataType_F32: return JXR_F32;
    case XLA_FFI_DataType_F64: return JXR_F64;
    case XLA_FFI_DataType_F16: return JXR_F16;
    case XLA_FFI_DataType_BF16: return JXR_BF16;
    default: return -1;
  }
}

XLA_FFI_Error* stream_of(XLA_FFI_CallFrame* cf, void** stream) {
  XLA_FFI_Stream_Get_Args a;
  std::memset(&a, 0, sizeof(a));
  a.struct_size = XLA_FFI_Stream_Get_Args_STRUCT_SIZE;
  a.ctx = cf->ctx;
  XLA_FFI_Error* e = cf->api->XLA_FFI_Stream_Get(&a);
  *stream = a.stream;
  return e;
}

XLA_FFI_Error* status(const XLA_FFI_Api* api, int rc) {
  if (rc == JXR_OK) return nullptr;
  const XLA_FFI_Error_Code code = rc == JXR_ERR_INVALID_ARGUMENT ? XLA_FFI_Error_Code_INVALID_ARGUMENT
                                  : rc == JXR_ERR_NOT_IMPLEMENTED ? XLA_FFI_Error_Code_UNIMPLEMENTED
                                                                  : XLA_FFI_Error_Code_INTERNAL;
  return error(api, code, jxr_last_error());
}

enum Kind { kBits, kBitsHost, kUniform, kNormal, kBernoulli, kNormalBernoulli };

XLA_FFI_Error* handle(XLA_FFI_CallFrame* cf, Kind kind) {
  if (answer_metadata(cf)) return nullptr;
  if (cf->stage != XLA_FFI_ExecutionStage_EXECUTE) return nullptr;
  Frame f;
  if (XLA_FFI_Error* e = decode(cf, kind == kNormalBernoulli ? 2 : 1, &f)) return e;
  const uint64_t size = (uint64_t)(f.out_elems / f.nkeys);
  const uint32_t* keys = static_cast<const uint32_t*>(f.key->data);
  void* out = f.out->data;
  if (kind == kBitsHost) {
    const int bits = bits_of(f.out->dtype);
    if (!bits)
      return error(cf->api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                   "jxrng: random bits need an unsigned 8/16/32/64-bit result");
    return status(cf->api, jxr_random_bits_host_static(keys, f.nkeys, size, 0, size, f.layout,
                                                       bits, out, nullptr));
  }
  void* stream = nullptr;
  if (XLA_FFI_Error* e = stream_of(cf, &stream)) return e;
  if (kind == kBits) {
    const int bits = bits_of(f.out->dtype);
    if (!bits)
      return error(cf->api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                   "jxrng: random bits need an unsigned 8/16/32/64-bit result");
    return status(cf->api, jxr_random_bits(keys, f.nkeys, size, 0, size, f.layout, bits, out,
                                           stream));
  }
  if (kind == kBernoulli) {
    if (!is_bool(f.out->dtype))
      return error(cf->api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                   "jxrng: random_bernoulli needs a bool (pred) result");
    return status(cf->api, jxr_bernoulli(keys, f.nkeys, size, 0, size, f.layout, f.p_dtype, f.p,
                                         static_cast<uint8_t*>(out), stream));
  }
  const int dt = float_code(f.out->dtype);
  if (dt < 0)
    return error(cf->api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                 "jxrng: the samplers need a float32/float64/float16/bfloat16 result");
  if (kind == kUniform)
    return status(cf->api, jxr_uniform(keys, f.nkeys, size, 0, size, f.layout, dt, f.minval,
                                       f.maxval, 0, out, stream));
  if (kind == kNormalBernoulli && !is_bool(f.out2->dtype))
    return error(cf->api, XLA_FFI_Error_Code_INVALID_ARGUMENT,
                 "jxrng: the second result (the bernoulli draws) must be bool (pred)");
  // the library's erf_inv setting is per host thread: set for this call, then restored
  const int prev = jxr_set_accurate_erf_inv(f.accurate_erf_inv);
  const int rc =
      kind == kNormal
          ? jxr_normal(keys, f.nkeys, size, 0, size, f.layout, dt, out, stream)
          : jxr_normal_bernoulli(keys, f.nkeys, size, 0, size, f.layout, dt, f.p, out,
                                 static_cast<uint8_t*>(f.out2->data), stream);
  jxr_set_accurate_erf_inv(prev);
  return status(cf->api, rc);
}

}  // namespace

extern "C" {

XLA_FFI_Error* jxr_ffi_random_bits(XLA_FFI_CallFrame* cf) { return handle(cf, kBits); }
XLA_FFI_Error* jxr_ffi_random_bits_cpu(XLA_FFI_CallFrame* cf) { return handle(cf, kBitsHost); }
XLA_FFI_Error* jxr_ffi_uniform(XLA_FFI_CallFrame* cf) { return handle(cf, kUniform); }
XLA_FFI_Error* jxr_ffi_normal(XLA_FFI_CallFrame* cf) { return handle(cf, kNormal); }
XLA_FFI_Error* jxr_ffi_bernoulli(XLA_FFI_CallFrame* cf) { return handle(cf, kBernoulli); }
XLA_FFI_Error* jxr_ffi_normal_bernoulli(XLA_FFI_CallFrame* cf) {
  return handle(cf, kNormalBernoulli);
}

}  // extern "C"
