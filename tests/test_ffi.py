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
    assert sorted(names) == sorted(ff.HANDLERS)
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
        wn = orc.normal(keys[r], "float64", 500, True)  # float64 normals: 1e-12 relative
        assert np.all(np.abs(n[r].cpu().numpy() - wn) <= 1e-12 * np.abs(wn))
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


@pytest.mark.gpu
def test_bernoulli_handlers_match_the_oracle(lib):
    """jxr_ffi_bernoulli (p's dtype from the attribute's) and jxr_ffi_normal_bernoulli (a
    float normal and a bool bernoulli of the same key from one pass), key batches of three,
    both layouts, against the oracle."""
    import torch

    from oracle import oracle as orc
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    rt = ff.Runtime()
    rt.stream = torch.cuda.current_stream().cuda_stream
    keys = np.stack([orc.seed(s) for s in (3, 2024, 11)])
    kd = torch.from_numpy(keys).cuda()
    n = 4099
    for part in (True, False):
        lay = [("partitionable", ff.PRED, C.c_uint8(int(part)))]
        for pdt, code, val in (("float32", ff.F32, C.c_float(0.3)),
                               ("float64", ff.F64, C.c_double(0.3))):
            b = torch.empty((3, n), dtype=torch.bool, device="cuda")
            rt.call(lib.jxr_ffi_bernoulli, (ff.U32, kd.data_ptr(), [3, 2]),
                    (ff.PRED, b.data_ptr(), [3, n]), lay + [("p", code, val)])
            torch.cuda.synchronize()
            for r in range(3):
                want = orc.bernoulli(keys[r], pdt, 0.3, n, part)
                assert np.array_equal(b[r].cpu().numpy(), want.astype(bool)), (pdt, part)
        for dt, tdt, code, pval in (("float64", torch.float64, ff.F64, C.c_double(0.3)),
                                    ("float32", torch.float32, ff.F32, C.c_float(0.3))):
            z = torch.empty((3, n), dtype=tdt, device="cuda")
            b = torch.empty((3, n), dtype=torch.bool, device="cuda")
            rt.call(lib.jxr_ffi_normal_bernoulli, (ff.U32, kd.data_ptr(), [3, 2]),
                    [(code, z.data_ptr(), [3, n]), (ff.PRED, b.data_ptr(), [3, n])],
                    lay + [("p", code, pval)])
            torch.cuda.synchronize()
            for r in range(3):
                wz = orc.normal(keys[r], dt, n, part)
                gz = z[r].cpu().numpy()
                if dt == "float64":  # within 1e-12 relative
                    assert np.all(np.abs(gz - wz) <= 1e-12 * np.abs(wz)), (dt, part)
                else:  # within 2 ulp
                    d = np.abs(gz.view(np.int32).astype(np.int64) - wz.view(np.int32).astype(np.int64))
                    assert d.max() <= 2, (dt, part)
                wb = orc.bernoulli(keys[r], dt, 0.3, n, part)
                assert np.array_equal(b[r].cpu().numpy(), wb.astype(bool)), (dt, part)
    with pytest.raises(ff.FfiError, match="bool"):
        rt.call(lib.jxr_ffi_bernoulli, (ff.U32, kd.data_ptr(), [3, 2]),
                (ff.F32, b.data_ptr(), [3, n]))
    with pytest.raises(ff.FfiError, match="two result buffers"):
        rt.call(lib.jxr_ffi_normal_bernoulli, (ff.U32, kd.data_ptr(), [3, 2]),
                (ff.F32, z.data_ptr(), [3, n]))


@pytest.mark.gpu
def test_normal_handler_allocates_nothing(lib):
    """A float32 normal of 2^22 samples (large enough to read the sampler's table) through
    the CUDA handler allocates no device memory, whether or not the table was prepared,
    and its samples match the oracle's at sampled positions."""
    import torch

    import jaxr_b200 as jr
    from jaxr_b200 import _native as nat
    from oracle import oracle as orc
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    rt = ff.Runtime()
    rt.stream = torch.cuda.current_stream().cuda_stream
    key = orc.seed(42)
    kd = torch.from_numpy(key.reshape(1, 2).copy()).cuda()
    n = 1 << 22
    idx = np.unique(np.random.default_rng(5).integers(0, n, 4096))
    want = orc.normal_at(key, "float32", n, True, True, idx).astype(np.float32)
    tiny = torch.empty(16, dtype=torch.float32, device="cuda")
    jr.free_caches()  # no table on this device now
    rt.call(lib.jxr_ffi_normal, (ff.U32, kd.data_ptr(), [1, 2]), (ff.F32, tiny.data_ptr(), [1, 16]))
    results = []
    for prepared in (False, True):
        if prepared:  # the set-up call, made by the caller before its framework's pool
            nat.call("jxr_prepare_device", 1, rt.stream)
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rt.call(lib.jxr_ffi_normal, (ff.U32, kd.data_ptr(), [1, 2]), (ff.F32, out.data_ptr(), [1, n]))
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, prepared
        got = out.cpu().numpy()
        d = np.abs(got[idx].view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
        assert d.max() <= 2, prepared
        results.append(got)
    assert np.array_equal(results[0].view(np.uint32), results[1].view(np.uint32))
    jr.free_caches()


@pytest.mark.gpu
def test_cpu_handler_from_two_threads(lib):
    """Two host threads calling the CPU handler at once, with different keys, each get
    their own key's bits: the no-allocation entry point it runs on shares one device array
    per GPU, and the library serialises its calls."""
    import threading

    import torch

    from oracle import oracle as orc
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    n = (1 << 23) + 7  # several 16 MiB staging chunks per call
    wants = {s: orc.random_bits(orc.seed(s), 32, n, True) for s in (21, 22)}
    errors = []

    def worker(s):
        rt = ff.Runtime()
        key = np.ascontiguousarray(orc.seed(s).reshape(1, 2))
        for _ in range(4):
            out = np.empty((1, n), dtype=np.uint32)
            try:
                rt.call(lib.jxr_ffi_random_bits_cpu, (ff.U32, key.ctypes.data, [1, 2]),
                        (ff.U32, out.ctypes.data, [1, n]))
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append(repr(e))
                return
            if not np.array_equal(out[0], wants[s]):
                errors.append(f"seed {s}: wrong bits")

    ts = [threading.Thread(target=worker, args=(s,)) for s in (21, 22)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
