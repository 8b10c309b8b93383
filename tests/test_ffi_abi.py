"""The XLA FFI declarations the handlers compile against (jaxr_b200/csrc/ffi/xla_ffi_abi.h)
have the layouts, enum values and table slots of XLA's own FFI C API: a C++ translation
unit includes both and static_asserts every offset, size and value the handlers use.
Needs XLA's header (xla/ffi/api/c_api.h, e.g. jaxR's vendored copy under inst/include) in
$XLA_FFI_INCLUDE_DIR; skipped without it."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FFI_DIR = os.path.join(ROOT, "jaxr_b200", "csrc", "ffi")

STRUCT_FIELDS = {
    "XLA_FFI_Extension_Base": ["struct_size", "type", "next"],
    "XLA_FFI_Api_Version": ["struct_size", "extension_start", "major_version", "minor_version"],
    "XLA_FFI_Error_Create_Args": ["struct_size", "extension_start", "message", "errc"],
    "XLA_FFI_Buffer": ["struct_size", "extension_start", "dtype", "data", "rank", "dims"],
    "XLA_FFI_ByteSpan": ["ptr", "len"],
    "XLA_FFI_Scalar": ["dtype", "value"],
    "XLA_FFI_TypeId": ["type_id"],
    "XLA_FFI_Args": ["struct_size", "extension_start", "size", "types", "args"],
    "XLA_FFI_Rets": ["struct_size", "extension_start", "size", "types", "rets"],
    "XLA_FFI_Attrs": ["struct_size", "extension_start", "size", "types", "names", "attrs"],
    "XLA_FFI_CallFrame": ["struct_size", "extension_start", "api", "ctx", "stage", "args",
                          "rets", "attrs", "future"],
    "XLA_FFI_Stream_Get_Args": ["struct_size", "extension_start", "ctx", "stream"],
    "XLA_FFI_Metadata": ["struct_size", "api_version", "traits", "state_type_id"],
    "XLA_FFI_Metadata_Extension": ["extension_base", "metadata"],
}
# the API table: our declaration stops at the last slot the handlers call
API_SLOTS = ["struct_size", "extension_start", "api_version", "internal_api",
             "XLA_FFI_Error_Create", "XLA_FFI_Error_GetMessage", "XLA_FFI_Error_Destroy",
             "XLA_FFI_Handler_Register", "XLA_FFI_Stream_Get"]
ENUMS = ["XLA_FFI_Extension_Metadata", "XLA_FFI_Error_Code_OK",
         "XLA_FFI_Error_Code_INVALID_ARGUMENT", "XLA_FFI_Error_Code_RESOURCE_EXHAUSTED",
         "XLA_FFI_Error_Code_UNIMPLEMENTED", "XLA_FFI_Error_Code_INTERNAL",
         "XLA_FFI_DataType_INVALID", "XLA_FFI_DataType_PRED", "XLA_FFI_DataType_S32",
         "XLA_FFI_DataType_S64", "XLA_FFI_DataType_U8", "XLA_FFI_DataType_U16",
         "XLA_FFI_DataType_U32", "XLA_FFI_DataType_U64", "XLA_FFI_DataType_F16",
         "XLA_FFI_DataType_F32", "XLA_FFI_DataType_F64", "XLA_FFI_DataType_BF16",
         "XLA_FFI_ArgType_BUFFER", "XLA_FFI_RetType_BUFFER", "XLA_FFI_AttrType_ARRAY",
         "XLA_FFI_AttrType_DICTIONARY", "XLA_FFI_AttrType_SCALAR", "XLA_FFI_AttrType_STRING",
         "XLA_FFI_ExecutionStage_INSTANTIATE", "XLA_FFI_ExecutionStage_PREPARE",
         "XLA_FFI_ExecutionStage_INITIALIZE", "XLA_FFI_ExecutionStage_EXECUTE",
         "XLA_FFI_Error_Create_Args_STRUCT_SIZE", "XLA_FFI_Stream_Get_Args_STRUCT_SIZE"]


def layout_check_source():
    lines = ["#include <cstddef>", "#include <cstdint>", "namespace mine {",
             '#include "xla_ffi_abi.h"', "}", '#include "xla/ffi/api/c_api.h"']
    lines.append("static_assert(XLA_FFI_API_MAJOR == 0 && XLA_FFI_API_MINOR == 3, \"api 0.3\");")
    for t, fields in STRUCT_FIELDS.items():
        lines.append(f"static_assert(sizeof(mine::{t}) == sizeof(::{t}), \"size of {t}\");")
        for f in fields:
            lines.append(f"static_assert(offsetof(mine::{t}, {f}) == offsetof(::{t}, {f}), "
                         f"\"{t}.{f}\");")
    for f in API_SLOTS:
        lines.append(f"static_assert(offsetof(mine::XLA_FFI_Api, {f}) == "
                     f"offsetof(::XLA_FFI_Api, {f}), \"XLA_FFI_Api.{f}\");")
    for e in ENUMS:
        lines.append(f"static_assert((long)mine::{e} == (long)::{e}, \"{e}\");")
    return "\n".join(lines) + "\n"


def test_declarations_match_xla_c_api(tmp_path):
    inc = os.environ.get("XLA_FFI_INCLUDE_DIR")
    if not inc or not os.path.exists(os.path.join(inc, "xla", "ffi", "api", "c_api.h")):
        pytest.skip("XLA's FFI header not available (set XLA_FFI_INCLUDE_DIR)")
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    src = tmp_path / "layout_check.cc"
    src.write_text(layout_check_source())
    r = subprocess.run([cxx, "-std=c++17", "-fsyntax-only", "-I" + FFI_DIR, "-I" + inc,
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


def test_handlers_build_without_xla_headers(tmp_path):
    """The handlers compile against the declarations alone (as on a machine without XLA's
    source tree)."""
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    r = subprocess.run([cxx, "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", "-I" + FFI_DIR,
                        "-I" + os.path.join(ROOT, "include"),
                        os.path.join(FFI_DIR, "jxrng_ffi.cc")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
