"""The XLA typed-FFI handlers (include/jxrng_ffi.h) driven through a call frame laid out
as XLA's FFI C API declares it (tests/ffi_frame.py): the metadata query, argument checks
and error reporting on the CPU; results against the oracle on the GPU, for the CUDA
handlers (device buffers, the runtime's stream) and the CPU one (host buffers)."""

import ctypes as C
import os
import re

import numpy as np
import pytest

import ffi_frame as ff

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.skipif(not os.path.exists(ff.FFI_LIB),
                                reason="libjxrng_ffi.so not built (no XLA FFI headers)")


@pytest.fixture(scope="module")
def lib():
    return ff.load()


def test_exports_the_declared_handlers(lib):
    text = open(os.path.join(ROOT, "include", "jxrng_ffi.h")).read()
    names = re.findall(r"^XLA_FFI_Error\* (jxr_ffi_\w+)\(", text, re.M)
    assert len(names) == 4
    for n in names:
        assert hasattr(lib, n), n


def test_metadata_query(lib):
    rt = ff.Runtime()
    md = ff.Metadata()
    md.struct_size = C.sizeof(ff.Metadata)
    key = (ff.U32, None, [2])
    rt.call(lib.jxr_ffi_random_bits, key, (ff.U32, None, [4]), metadata=md)
    assert (md.api_version.major_version, md.api_version.minor_version) == (0, 3)
    assert md.traits == 0


def test_argument_errors(lib):
    rt = ff.Runtime()
    with pytest.raises(ff.FfiError, match="uint32\\[..., 2\\]") as e:
        rt.call(lib.jxr_ffi_random_bits, (ff.U32, None, [3]), (ff.U32, None, [4]))
    assert e.value.code == 3  # INVALID_ARGUMENT
    with pytest.raises(ff.FfiError, match="uint32"):
        rt.call(lib.jxr_ffi_random_bits, (ff.S32, None, [2]), (ff.U32, None, [4]))
    with pytest.raises(ff.FfiError, match="multiple of the number of keys"):
        rt.call(lib.jxr_ffi_random_bits, (ff.U32, None, [3, 2]), (ff.U32, None, [4]))
    with pytest.raises(ff.FfiError, match="unsigned 8/16/32/64-bit"):
        rt.call(lib.jxr_ffi_random_bits_cpu, (ff.U32, None, [2]), (ff.F32, None, [4]))
    # other execution stages are no-ops
    rt.call(lib.jxr_ffi_random_bits, (ff.U32, None, [3]), (ff.U32, None, [4]), stage=0)


@pytest.mark.gpu
def test_cuda_handlers_match_the_oracle(lib):
    import torch

    from oracle import oracle as orc
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from jaxr_b200 import build
    build.build()
    rt = ff.Runtime()
    rt.stream = torch.cuda.current_stream().cuda_stream
    keys = np.stack([orc.seed(s) for s in (0, 42, 7)])
    kd = torch.from_numpy(keys).cuda()
    for part in (True, False):
        attr = [("partitionable", ff.PRED, C.c_uint8(int(part)))]
        for bw, tdt, code in ((8, torch.uint8, ff.U8), (32, torch.uint32, ff.U32),
                              (64, torch.uint64, ff.U64)):
            out = torch.empty((3, 1001), dtype=tdt, device="cuda")
            rt.call(lib.jxr_ffi_random_bits, (ff.U32, kd.data_ptr(), [3, 2]),
                    (code, out.data_ptr(), [3, 1001]), attr)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            for r in range(3):
                assert np.array_equal(got[r], orc.random_bits(keys[r], bw, 1001, part)), (bw, part)
    u = torch.empty((3, 500), dtype=torch.float32, device="cuda")
    rt.call(lib.jxr_ffi_uniform, (ff.U32, kd.data_ptr(), [3, 2]), (ff.F32, u.data_ptr(), [3, 500]),
            [("maxval", ff.F64, C.c_double(3.0)), ("minval", ff.F64, C.c_double(-2.0))])
    n = torch.empty((3, 500), dtype=torch.float64, device="cuda")
    rt.call(lib.jxr_ffi_normal, (ff.U32, kd.data_ptr(), [3, 2]), (ff.F64, n.data_ptr(), [3, 500]))
    torch.cuda.synchronize()
    for r in range(3):
        want = orc.uniform(keys[r], "float32", 500, True, -2.0, 3.0)
        assert np.array_equal(u[r].cpu().numpy().view(np.uint32), want.view(np.uint32))
        wn = orc.normal(keys[r], "float64", 500, True)
        assert np.array_equal(n[r].cpu().numpy().view(np.uint64), wn.view(np.uint64))
    # attribute accurate_erf_inv: the accurate erf_inv for this call only
    from jaxr_b200 import _native as nat
    na = torch.empty((3, 500), dtype=torch.float32, device="cuda")
    before = nat.lib().jxr_get_accurate_erf_inv()
    rt.call(lib.jxr_ffi_normal, (ff.U32, kd.data_ptr(), [3, 2]), (ff.F32, na.data_ptr(), [3, 500]),
            [("accurate_erf_inv", ff.PRED, C.c_uint8(1))])
    torch.cuda.synchronize()
    assert nat.lib().jxr_get_accurate_erf_inv() == before == 0
    for r in range(3):
        wa = orc.normal(keys[r], "float32", 500, True, accurate=True)
        assert np.array_equal(na[r].cpu().numpy().view(np.uint32), wa.view(np.uint32))


@pytest.mark.gpu
def test_cpu_handler_host_buffers(lib):
    import torch

    from oracle import oracle as orc
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    rt = ff.Runtime()
    keys = np.ascontiguousarray(np.stack([orc.seed(s) for s in (1, 2)]))
    out = np.empty((2, 70001), dtype=np.uint16)
    rt.call(lib.jxr_ffi_random_bits_cpu, (ff.U32, keys.ctypes.data, [2, 2]),
            (ff.U16, out.ctypes.data, [2, 70001]))
    for r in range(2):
        assert np.array_equal(out[r], orc.random_bits(keys[r], 16, 70001, True))
