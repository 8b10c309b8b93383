"""Drives the XLA typed-FFI handlers of libjxrng_ffi.so the way XLA's runtime does, with
a call frame laid out as XLA's FFI C API (xla/ffi/api/c_api.h, API 0.3) declares it and a
minimal API table: error creation and the stream query.  No XLA
runtime is needed, so the handlers are tested where no PJRT plugin is installed."""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
FFI_LIB = os.path.join(os.path.dirname(HERE), "jaxr_b200", "libjxrng_ffi.so")

# data types (XLA_FFI_DataType)
PRED, S32, S64, U8, U16, U32, U64, F16, F32, F64, BF16 = 1, 4, 5, 6, 7, 8, 9, 10, 11, 12, 16
ARG_BUFFER = RET_BUFFER = 1
ATTR_SCALAR = 3
STAGE_EXECUTE = 3
EXT_METADATA = 1


class ExtBase(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("type", C.c_int), ("next", C.c_void_p)]


class ApiVersion(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("major_version", C.c_int), ("minor_version", C.c_int)]


class Metadata(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("api_version", ApiVersion),
                ("traits", C.c_uint32), ("state_type_id", C.c_int64)]


class MetadataExt(C.Structure):
    _fields_ = [("extension_base", ExtBase), ("metadata", C.POINTER(Metadata))]


class Buffer(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("dtype", C.c_int), ("data", C.c_void_p), ("rank", C.c_int64),
                ("dims", C.POINTER(C.c_int64))]


class ByteSpan(C.Structure):
    _fields_ = [("ptr", C.c_char_p), ("len", C.c_size_t)]


class Scalar(C.Structure):
    _fields_ = [("dtype", C.c_int), ("value", C.c_void_p)]


class Args(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("size", C.c_int64), ("types", C.POINTER(C.c_int)),
                ("args", C.POINTER(C.c_void_p))]


class Attrs(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("size", C.c_int64), ("types", C.POINTER(C.c_int)),
                ("names", C.POINTER(C.POINTER(ByteSpan))), ("attrs", C.POINTER(C.c_void_p))]


class CallFrame(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("api", C.c_void_p), ("ctx", C.c_void_p), ("stage", C.c_int),
                ("args", Args), ("rets", Args), ("attrs", Attrs), ("future", C.c_void_p)]


class ErrorCreateArgs(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("message", C.c_char_p), ("errc", C.c_int)]


class StreamGetArgs(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("ctx", C.c_void_p), ("stream", C.c_void_p)]


_FN = C.c_void_p  # a function pointer slot of the API table
_API_FIELDS = ["Error_Create", "Error_GetMessage", "Error_Destroy", "Handler_Register",
               "Stream_Get", "Type_Register", "ExecutionContext_Get", "State_Set", "State_Get",
               "DeviceMemory_Allocate", "DeviceMemory_Free", "ThreadPool_Schedule",
               "ThreadPool_NumThreads", "Future_Create", "Future_SetAvailable",
               "Future_SetError", "RunId_Get", "DeviceOrdinal_Get"]


class Api(C.Structure):
    _fields_ = ([("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                 ("api_version", ApiVersion), ("internal_api", C.c_void_p)] +
                [(f, _FN) for f in _API_FIELDS])


class FfiError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"XLA FFI error {code}: {message}")
        self.code = code
        self.message = message


class Runtime:
    """The API table and error store a handler sees; `stream` is what Stream_Get returns."""

    def __init__(self):
        self.errors = {}
        self.stream = None

        @C.CFUNCTYPE(C.c_void_p, C.POINTER(ErrorCreateArgs))
        def error_create(a):
            key = len(self.errors) + 1
            self.errors[key] = (a.contents.errc, a.contents.message.decode())
            return key

        @C.CFUNCTYPE(C.c_void_p, C.POINTER(StreamGetArgs))
        def stream_get(a):
            a.contents.stream = self.stream
            return None

        self._keep = (error_create, stream_get)
        self.api = Api()
        self.api.struct_size = C.sizeof(Api)
        self.api.api_version.struct_size = C.sizeof(ApiVersion)
        self.api.api_version.major_version = 0
        self.api.api_version.minor_version = 3
        self.api.Error_Create = C.cast(error_create, C.c_void_p)
        self.api.Stream_Get = C.cast(stream_get, C.c_void_p)

    def call(self, handler, key, out, attrs=(), stage=STAGE_EXECUTE, metadata=None):
        """Call `handler` with one argument buffer and the result buffer(s) `out` (one
        tuple, or a list of tuples for several results), each a tuple (dtype, data
        pointer, dims), and scalar attributes [(name, dtype, ctypes value)] sorted by name
        as XLA sorts them."""
        keep = []

        def buf(spec):
            dtype, ptr, dims = spec
            d = (C.c_int64 * len(dims))(*dims)
            b = Buffer(C.sizeof(Buffer), None, dtype, ptr, len(dims), d)
            keep.extend([d, b])
            return C.cast(C.pointer(b), C.c_void_p)

        f = CallFrame()
        f.struct_size = C.sizeof(CallFrame)
        f.api = C.cast(C.pointer(self.api), C.c_void_p)
        f.stage = stage
        at = (C.c_int * 1)(ARG_BUFFER)
        av = (C.c_void_p * 1)(buf(key))
        outs = out if isinstance(out, list) else [out]
        rt = (C.c_int * len(outs))(*([RET_BUFFER] * len(outs)))
        rv = (C.c_void_p * len(outs))(*[buf(o) for o in outs])
        f.args = Args(C.sizeof(Args), None, 1, at, av)
        f.rets = Args(C.sizeof(Args), None, len(outs), rt, rv)
        attrs = sorted(attrs)
        n = len(attrs)
        tt = (C.c_int * max(n, 1))(*([ATTR_SCALAR] * n))
        names = (C.POINTER(ByteSpan) * max(n, 1))()
        vals = (C.c_void_p * max(n, 1))()
        for i, (name, dtype, value) in enumerate(attrs):
            raw = name.encode()
            span = ByteSpan(raw, len(raw))
            sc = Scalar(dtype, C.cast(C.pointer(value), C.c_void_p))
            keep.extend([raw, span, sc, value])
            names[i] = C.pointer(span)
            vals[i] = C.cast(C.pointer(sc), C.c_void_p)
        f.attrs = Attrs(C.sizeof(Attrs), None, n, tt, names, vals)
        keep.extend([at, av, rt, rv, tt, names, vals])
        if metadata is not None:
            ext = MetadataExt(ExtBase(C.sizeof(MetadataExt), EXT_METADATA, None),
                              C.pointer(metadata))
            keep.append(ext)
            f.extension_start = C.cast(C.pointer(ext), C.c_void_p)
        rc = handler(C.addressof(f))
        if rc:
            code, msg = self.errors[rc]
            raise FfiError(code, msg)


HANDLERS = ("jxr_ffi_random_bits", "jxr_ffi_random_bits_cpu", "jxr_ffi_uniform", "jxr_ffi_normal",
            "jxr_ffi_bernoulli", "jxr_ffi_normal_bernoulli")


def load():
    lib = C.CDLL(FFI_LIB)
    for name in HANDLERS:
        fn = getattr(lib, name)
        fn.argtypes = [C.c_void_p]
        fn.restype = C.c_void_p
    return lib
