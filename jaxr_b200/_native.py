"""Loader of libjxrng.so, the sm_100a kernels behind include/jxrng.h.

The library is built in-tree (jaxr_b200/libjxrng.so) by `jaxr_b200.build.build()`.
There is no CPU fallback: if the library is missing, or no sm_100 device is current,
every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjxrng.so")

# include/jxrng.h
JXR_OK = 0
JXR_ERR_INVALID_ARGUMENT = 1
JXR_ERR_NOT_IMPLEMENTED = 2
JXR_ERR_CUDA = 3
JXR_ERR_NO_DEVICE = 4
LAYOUT_ORIGINAL = 0
LAYOUT_PARTITIONABLE = 1
F32, F64, F16, BF16 = 0, 1, 2, 3
FLAG_UNFUSED_MUL_ADD = 1

_u32p = ctypes.c_void_p
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_dbl = ctypes.c_double
_u32 = ctypes.c_uint32
_sz = ctypes.c_size_t

# name -> argument types; every entry point returns int status
SIGNATURES = {
    "jxr_seed": [ctypes.POINTER(ctypes.c_int64), _i64, _int, ctypes.POINTER(ctypes.c_uint32)],
    "jxr_threefry2x32": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp],
    "jxr_threefry_2x32": [_vp, _i64, _vp, _i64, _vp, _vp],
    "jxr_split": [_vp, _i64, _i64, _int, _vp, _vp],
    "jxr_fold_in": [_vp, _i64, _vp, _i64, _vp, _vp],
    "jxr_random_bits": [_vp, _i64, _u64, _u64, _u64, _int, _int, _vp, _vp],
    "jxr_uniform": [_vp, _i64, _u64, _u64, _u64, _int, _int, _dbl, _dbl, _u32, _vp, _vp],
    "jxr_normal": [_vp, _i64, _u64, _u64, _u64, _int, _int, _vp, _vp],
    "jxr_bernoulli": [_vp, _i64, _u64, _u64, _u64, _int, _int, _dbl, _vp, _vp],
    "jxr_normal_bernoulli": [_vp, _i64, _u64, _u64, _u64, _int, _int, _dbl, _vp, _vp, _vp],
    "jxr_uniform_from_bits": [_vp, _i64, _int, _dbl, _dbl, _u32, _vp, _vp],
    "jxr_normal_from_bits": [_vp, _i64, _int, _vp, _vp],
    "jxr_uniform_affine": [_vp, _vp, _vp, _i64, _int, _u32, _vp, _vp],
    "jxr_uniform_affine_rows": [_vp, _vp, _vp, _i64, _i64, _int, _u32, _vp, _vp],
    "jxr_bernoulli_from_uniform": [_vp, _vp, _vp, _i64, _int, _vp, _vp],
    "jxr_sample": [_vp, _i64, _u64, _u64, _u64, _int, _int, _int, _vp, _vp],
    "jxr_randint": [_vp, _vp, _i64, _u64, _u64, _u64, _int, _int, _i64, _i64, _int, _int, _vp,
                    _vp],
    "jxr_randint_combine": [_vp, _vp, _i64, _int, _int, _vp, _i64, _vp, _i64, _vp, _i64, _int,
                            _vp, _vp],
    "jxr_gumbel_rows": [_vp, _vp, _i64, _int, _int, _vp, _vp],
    "jxr_truncated_normal": [_vp, _i64, _u64, _u64, _u64, _int, _int, _dbl, _dbl, _vp, _vp],
    "jxr_truncated_normal_from_unit": [_vp, _vp, _i64, _vp, _i64, _i64, _int, _vp, _vp],
    "jxr_shuffle_scratch_bytes": [_i64],
    "jxr_shuffle": [_vp, _int, _i64, _i64, _i64, _int, _vp, _vp, ctypes.c_size_t, _vp],
    "jxr_take": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp],
    "jxr_choice_p_from_unit": [_vp, _i64, _int, _vp, _i64, _int, _vp, _vp],
    "jxr_add_log": [_vp, _vp, _i64, _int, _vp],
    "jxr_argsort_scratch_bytes": [_i64],
    "jxr_argsort_float": [_vp, _i64, _int, _int, _vp, _vp, ctypes.c_size_t, _vp],
    "jxr_rbg_bits": [_vp, _u64, _u64, _u64, _int, _vp, _vp, _vp],
    "jxr_rbg_blocks": [_vp, _u64, _u64, _i64, _vp, _vp],
    "jxr_rbg_unsafe_fold_in": [_vp, _i64, _vp, _i64, _int, _vp, _vp],
    "jxr_sample_from_bits": [_vp, _i64, _int, _int, _vp, _vp],
    "jxr_truncated_normal_scratch": [_vp, _i64, _u64, _u64, _u64, _int, _int, _dbl, _dbl, _vp,
                                     _sz, _vp, _vp],
    "jxr_truncated_normal_from_bits": [_vp, _i64, _int, _dbl, _dbl, _vp, _vp],
    "jxr_random_bits_multi": [_vp, _int, _vp, _u64, _int, _int, _vp, _int, _vp, _vp],
    "jxr_complex_from_parts": [_vp, _vp, _i64, _int, _dbl, _vp, _vp],
    "jxr_cumsum": [_vp, _i64, _int, _vp, _vp],
    "jxr_erf_inv": [_vp, _i64, _int, _vp, _vp],
    "jxr_set_accurate_erf_inv": [_int],
    "jxr_free_caches": [],
    "jxr_prepare_device": [_u32, _vp],
    "jxr_get_accurate_erf_inv": [],
    "jxr_set_shuffle_span_cap": [_int],
    "jxr_shuffle_lanes_scratch_bytes": [_i64, _i64],
    "jxr_shuffle_lanes": [_vp, _int, _i64, _i64, _i64, _i64, _int, _vp, _vp, ctypes.c_size_t, _vp],
    "jxr_random_bits_host": [_vp, _i64, _u64, _u64, _u64, _int, _int, _vp],
    "jxr_probe_cipher": [_u64, _int, _vp, ctypes.POINTER(ctypes.c_uint64), _vp],
    "jxr_random_bits_host_static": [_vp, _i64, _u64, _u64, _u64, _int, _int, _vp, _vp],
    "jxr_ipc_export": [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)],
    "jxr_ipc_open": [_vp, ctypes.POINTER(ctypes.c_void_p)],
    "jxr_ipc_close": [_vp],
}


class NativeError(RuntimeError):
    """A status code other than JXR_OK from libjxrng."""

    def __init__(self, fn, code, message):
        super().__init__(f"{fn} failed ({code}): {message}")
        self.fn = fn
        self.code = code
        self.message = message


_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (loads it once; raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -c 'import jaxr_b200.build as b; "
                    "b.build()'` (nvcc, sm_100a). There is no CPU fallback.")
            L = ctypes.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
            L.jxr_abi_version.restype = ctypes.c_int
            L.jxr_last_error.restype = ctypes.c_char_p
            L.jxr_shuffle_scratch_bytes.restype = ctypes.c_size_t
            L.jxr_shuffle_lanes_scratch_bytes.restype = ctypes.c_size_t
            L.jxr_argsort_scratch_bytes.restype = ctypes.c_size_t
            _lib = L
    return _lib


def call(name, *args):
    """Call entry point `name`; raise NativeError on a non-zero status."""
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != JXR_OK:
        msg = L.jxr_last_error().decode(errors="replace")
        raise NativeError(name, rc, msg)
    return rc


def exported_symbols():
    return ["jxr_abi_version", "jxr_last_error"] + list(SIGNATURES)
