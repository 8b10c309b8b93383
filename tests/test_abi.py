"""The C ABI library: it loads and exports every entry point include/jxrng.h declares
(no compute call: that needs a GPU)."""

import ctypes
import os
import re

from jaxr_b200 import _native
from jaxr_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    text = open(os.path.join(ROOT, "include", "jxrng.h")).read()
    return sorted(set(re.findall(r"^(?:int|size_t|const char\*)\s+(jxr_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    build.build()
    lib = ctypes.CDLL(_native.LIB_PATH)
    names = declared()
    assert len(names) >= 18
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(_native.exported_symbols()) == names


def test_abi_version_and_host_seed():
    L = _native.lib()
    assert L.jxr_abi_version() == 1
    seeds = (ctypes.c_int64 * 3)(0, -1, (1 << 40) + 5)
    out = (ctypes.c_uint32 * 6)()
    assert L.jxr_seed(seeds, 3, 1, out) == 0
    assert list(out) == [0, 0, 0xFFFFFFFF, 0xFFFFFFFF, 256, 5]
    assert L.jxr_seed(seeds, 3, 0, out) == 0
    assert list(out) == [0, 0, 0, 0xFFFFFFFF, 0, 5]


def test_invalid_arguments_fail_before_any_device_work():
    L = _native.lib()
    # bad layout / range / bit width are rejected with a message, no device touched
    rc = L.jxr_random_bits(None, 1, 10, 5, 6, 1, 32, None, None)
    assert rc == _native.JXR_ERR_INVALID_ARGUMENT
    assert b"outside a request" in L.jxr_last_error()
    rc = L.jxr_random_bits(None, 1, 10, 0, 10, 7, 32, None, None)
    assert rc == _native.JXR_ERR_INVALID_ARGUMENT and b"layout" in L.jxr_last_error()
    rc = L.jxr_uniform(None, 1, 10, 0, 10, 1, 9, 0.0, 1.0, 0, None, None)
    assert rc == _native.JXR_ERR_INVALID_ARGUMENT and b"dtype" in L.jxr_last_error()
    assert L.jxr_random_bits(None, 1, 10, 0, 0, 1, 32, None, None) == 0  # empty request
