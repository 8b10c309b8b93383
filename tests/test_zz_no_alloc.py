"""jxr_random_bits_host_static, the entry point that allocates nothing.

Callers that cannot allocate device memory while they run -- a host framework that has
reserved the GPU for its own memory pool, such as XLA's PJRT client running an FFI
handler -- use this variant of jxr_random_bits_host.  Its device scratch is one fixed
array compiled into the library, so these tests check that it gives exactly what the
allocating entry point gives, on two calls in a row (the second call finds the
previous call's data in the shared array), and that it refuses key batches larger than
that array holds.  The file is named to run last.
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


def test_static_matches_allocating_entry_point(lib):
    keys = np.array([[0, 123], [7, 0xDEADBEEF]], dtype=np.uint32)
    size = 3 * STAGE_WORDS + 1234            # several staging chunks and a ragged tail
    begin, count = 17, 3 * STAGE_WORDS + 1000
    for layout, bw, npdt in [(1, 32, np.uint32), (0, 32, np.uint32), (1, 64, np.uint64),
                             (1, 8, np.uint8)]:
        want = np.zeros((2, count), dtype=npdt)
        _call(lib, "jxr_random_bits_host", keys, size, begin, count, layout, bw, want)
        for _ in range(2):  # two calls in a row through the shared scratch
            got = np.full((2, count), 0xAB, dtype=npdt)
            _call(lib, "jxr_random_bits_host_static", keys, size, begin, count, layout, bw, got,
                  torch.cuda.current_stream().cuda_stream)
            assert np.array_equal(got, want), (layout, bw)


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
