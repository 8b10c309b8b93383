"""jxr_random_bits_host_static, the entry point that allocates nothing.

Callers that cannot allocate device memory while they run -- a host framework that has
reserved the GPU for its own memory pool, such as XLA's PJRT client running an FFI
handler -- use this variant of jxr_random_bits_host.  Its device scratch is one fixed
array compiled into the library, so these tests check that it gives exactly what the
allocating entry point gives, on two calls in a row (the second call finds the
previous call's data in the shared array), and that it refuses key batches larger than
that array holds; against the oracle directly; and, in a fresh process after the set-up
call (jxr_prepare_device), that calls leave the device's free memory unchanged.  The file
is named to run last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_KEYS = 4096
STAGE_WORDS = (16 << 20) // 4


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from jaxr_b200 import _native, build
    build.build()
    torch.cuda.set_device(0)
    return _native


def _call(nat, name, keys, size, begin, count, layout, bw, out, *stream):
    nat.call(name, _ptr(keys), keys.shape[0], size, begin, count, layout, bw, _ptr(out), *stream)


CASES = [(1, 32, np.uint32), (0, 32, np.uint32), (1, 64, np.uint64), (0, 64, np.uint64),
         (1, 8, np.uint8), (0, 8, np.uint8), (1, 16, np.uint16), (0, 16, np.uint16)]


def test_static_matches_allocating_entry_point(lib):
    keys = np.array([[0, 123], [7, 0xDEADBEEF]], dtype=np.uint32)
    size = 3 * STAGE_WORDS + 1234            # several staging chunks and a ragged tail
    begin, count = 17, 3 * STAGE_WORDS + 1000
    for layout, bw, npdt in CASES:
        want = np.zeros((2, count), dtype=npdt)
        _call(lib, "jxr_random_bits_host", keys, size, begin, count, layout, bw, want)
        for _ in range(2):  # two calls in a row through the shared scratch
            got = np.full((2, count), 0xAB, dtype=npdt)
            _call(lib, "jxr_random_bits_host_static", keys, size, begin, count, layout, bw, got,
                  torch.cuda.current_stream().cuda_stream)
            assert np.array_equal(got, want), (layout, bw)


def test_static_matches_the_oracle(lib):
    """The same requests against the CPU oracle directly, both layouts, every width."""
    from oracle import oracle as orc
    keys = np.array([[0, 123], [7, 0xDEADBEEF]], dtype=np.uint32)
    size = 2 * STAGE_WORDS + 77
    begin, count = 5, 2 * STAGE_WORDS + 60
    for layout, bw, npdt in CASES:
        got = np.full((2, count), 0xAB, dtype=npdt)
        _call(lib, "jxr_random_bits_host_static", keys, size, begin, count, layout, bw, got, None)
        for r in range(2):
            want = orc.random_bits(keys[r], bw, size, bool(layout), begin, count)
            assert np.array_equal(got[r], want), (layout, bw, r)


_FRESH = r"""
import ctypes, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import torch
from jaxr_b200 import _native as nat
torch.cuda.init()
torch.cuda.synchronize()
nat.call("jxr_prepare_device", 0, None)   # set-up: module, array and kernels loaded now
keys = np.array([[0, 9], [1, 2]], dtype=np.uint32)
free0 = torch.cuda.mem_get_info()[0]
for layout in (1, 0):
    for bw, dt in ((8, np.uint8), (16, np.uint16), (32, np.uint32), (64, np.uint64)):
        out = np.empty((2, (1 << 22) + 3), dtype=dt)
        nat.call("jxr_random_bits_host_static", keys.ctypes.data_as(ctypes.c_void_p), 2,
                 out.shape[1], 0, out.shape[1], layout, bw, out.ctypes.data_as(ctypes.c_void_p), None)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
print("free before", free0, "after", free1)
assert free1 == free0, (free0, free1)
print("no allocation after set-up")
"""


def test_static_allocates_nothing_after_set_up(lib, tmp_path):
    """In a fresh process: jxr_prepare_device at set-up (loading the module, its array and
    the kernels), then calls of every width and layout leave the device's free memory as
    it was."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH, root], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "no allocation after set-up" in r.stdout, (r.stdout + r.stderr)[-3000:]


def test_static_rejects_batches_beyond_its_scratch(lib):
    keys = np.zeros((MAX_KEYS + 1, 2), dtype=np.uint32)
    out = np.zeros((MAX_KEYS + 1, 4), dtype=np.uint32)
    with pytest.raises(lib.NativeError, match="at most 4096 keys"):
        _call(lib, "jxr_random_bits_host_static", keys, 4, 0, 4, 1, 32, out, None)
    keys = np.zeros((MAX_KEYS, 2), dtype=np.uint32)  # the maximum itself is accepted
    out = np.zeros((MAX_KEYS, 4), dtype=np.uint32)
    _call(lib, "jxr_random_bits_host_static", keys, 4, 0, 4, 1, 32, out, None)
    want = np.zeros_like(out)
    _call(lib, "jxr_random_bits_host", keys, 4, 0, 4, 1, 32, want)
    assert np.array_equal(out, want)
