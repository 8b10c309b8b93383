"""Parity of random_permutation / random_choice (R/random.R:361-464) with the CPU oracle,
on the GPU: the device radix sort must reproduce the stable sort of every shuffle round
exactly, for one, two and three rounds (n up to 2^22), independent slices along any axis,
both counter layouts, and key batches."""

import math

import numpy as np
import pytest
import torch

import jaxr_b200 as jr
from oracle import oracle as orc
from product_backend import flags, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from jaxr_b200 import build
    build.build()


def dev_key(k):
    return torch.tensor(np.asarray(k, dtype=np.uint32)).cuda()


def rounds(n):
    return int(math.ceil(3 * math.log(max(1, n)) / math.log(2 ** 32 - 1)))


@pytest.mark.parametrize("part", [True, False])
def test_permutation_of_n_exact(part):
    key = orc.seed(2718)
    for n in (0, 1, 2, 3, 10, 255, 256, 257, 1625, 1626, 8191, 8192, 8193, 100003):
        with flags(False, part):
            got = to_np(jr.random_permutation(dev_key(key), n))
        want = orc.permutation(key, n, partitionable=part)
        assert got.dtype == np.int32
        assert np.array_equal(got, want), (n, rounds(n))


def test_permutation_three_rounds():
    """n = 2^22: three shuffle rounds (ceil(3 * 22 ln 2 / ln(2^32 - 1)) = 3), 512 tiles per
    sort pass; compared in full with the oracle, and checked to be a permutation."""
    key = orc.seed(5)
    n = 1 << 22
    assert rounds(n) == 3
    got = to_np(jr.random_permutation(dev_key(key), n))
    want = orc.permutation(key, n)
    assert np.array_equal(got, want)
    assert np.array_equal(np.sort(got), np.arange(n, dtype=np.int32))


@pytest.mark.parametrize("dt", [torch.float32, torch.float64, torch.int8, torch.int16,
                                torch.bfloat16, torch.uint8, torch.int64])
def test_permutation_of_arrays(dt):
    key = orc.seed(9)
    x = torch.arange(60).reshape(5, 4, 3).to(dt)
    xn = x.float().numpy() if dt == torch.bfloat16 else x.numpy()
    with flags(dt in (torch.float64, torch.int64)):
        for axis in (0, 1, 2, -1):
            got = jr.random_permutation(dev_key(key), x, axis=axis)
            want = orc.permutation(key, xn, axis=axis)
            assert np.array_equal(to_np(got), want), (dt, axis)
            got = jr.random_permutation(dev_key(key), x, axis=axis, independent=True)
            want = orc.permutation(key, xn, axis=axis, independent=True)
            assert np.array_equal(to_np(got), want), (dt, axis, "independent")


def test_permutation_independent_many_segments():
    """(700, 3000) independent along axis 1: 2.1M elements, 700 segments -> two shuffle
    rounds, each a 32-bit sort then a 16-bit segment sort."""
    key = orc.seed(77)
    x = torch.arange(700 * 3000, dtype=torch.int32).reshape(700, 3000)
    got = to_np(jr.random_permutation(dev_key(key), x, axis=1, independent=True))
    want = orc.permutation(key, x.numpy(), axis=1, independent=True)
    assert np.array_equal(got, want)
    got = to_np(jr.random_permutation(dev_key(key), x, axis=0, independent=True))
    want = orc.permutation(key, x.numpy(), axis=0, independent=True)
    assert np.array_equal(got, want)


def test_permutation_key_batches():
    keys = np.stack([orc.seed(s) for s in range(3)])
    out = jr.vmap(lambda k: jr.random_permutation(k, 50))(dev_key(keys))
    for r in range(3):
        assert np.array_equal(to_np(out[r]), orc.permutation(keys[r], 50))


def test_permutation_errors():
    k = dev_key(orc.seed(0))
    with pytest.raises(jr.JaxTypeError, match="x must be an integer or at least 1-dimensional"):
        jr.random_permutation(k, 2.5)
    with pytest.raises(jr.JaxValueError, match="axis 2 is out of bounds for array of rank 1"):
        jr.random_permutation(k, torch.arange(4), axis=2)


def test_choice_variants():
    key = orc.seed(11)
    a = np.arange(40, dtype=np.int32).reshape(8, 5)
    at = torch.from_numpy(a)
    for shape in ((3,), (2, 2), ()):
        for replace in (True, False):
            got = to_np(jr.random_choice(dev_key(key), 30, shape, replace))
            want = orc.choice(key, 30, shape, replace)
            assert np.array_equal(got.ravel(), np.asarray(want).ravel()), (shape, replace)
            got = to_np(jr.random_choice(dev_key(key), at, shape, replace))
            want = orc.choice(key, a, shape, replace)
            assert np.array_equal(got.ravel(), np.asarray(want).ravel()), (shape, replace)
    p = [0.05, 0.3, 0.15, 0.0, 0.5]
    for x64 in (False, True):
        with flags(x64):
            got = to_np(jr.random_choice(dev_key(key), 5, (1000,), True, p))
        assert np.array_equal(got, orc.choice(key, 5, (1000,), True, p, x64=x64))
        assert not np.any(got == 3)
    assert to_np(jr.random_choice(dev_key(key), 10, (0,))).shape == (0,)
    with pytest.raises(jr.JaxValueError, match=r"Cannot take a larger sample \(size 5\)"):
        jr.random_choice(dev_key(key), 3, 5, replace=False)
    with pytest.raises(jr.JaxValueError, match="a must be greater than 0"):
        jr.random_choice(dev_key(key), 0, 2)
    with pytest.raises(jr.JaxValueError, match="p must be None or a 1D vector"):
        jr.random_choice(dev_key(key), 5, 2, p=[0.5, 0.5])


def test_choice_p_without_replacement():
    """gumbel + log(p), top_k: the device argsort against numpy's stable argsort of the
    same gumbel + log(p) values; zero-probability entries are never drawn."""
    key = orc.seed(3)
    p = np.array([0.1, 0.0, 0.3, 0.2, 0.15, 0.25], dtype=np.float32)
    got = to_np(jr.random_choice(dev_key(key), 6, (5,), False, p))
    g = orc.sample(key, "gumbel", "float32", 6)
    lp = np.array([np.float32(orc.lib().orc_log_pos(float(v))) if v > 0 else -np.inf for v in p],
                  dtype=np.float32)
    want = np.argsort(-(g + lp).astype(np.float32), kind="stable")[:5]
    assert np.array_equal(got, want)
    assert 1 not in got


@pytest.mark.parametrize("dt", ["float32", "float64"])
def test_argsort_float_stable(dt):
    """Descending and ascending stable argsort of floats with ties, both zeros and infinities,
    against numpy (2^20 + 3 values: 129 tiles, the last one partial)."""
    from jaxr_b200 import _native as nat
    rng = np.random.default_rng(1)
    n = (1 << 20) + 3
    x = rng.integers(-50, 50, n).astype(dt) / 4
    x[:5] = [0.0, -0.0, np.inf, -np.inf, 0.0]
    xt = torch.from_numpy(x).cuda()
    code = 0 if dt == "float32" else 1
    for desc in (0, 1):
        idx = torch.empty(n, dtype=torch.uint32, device="cuda")
        nb = nat.lib().jxr_argsort_scratch_bytes(n)
        scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
        nat.call("jxr_argsort_float", xt.data_ptr(), n, code, desc, idx.data_ptr(),
                 scratch.data_ptr(), nb, torch.cuda.current_stream().cuda_stream)
        got = to_np(idx).astype(np.int64)
        key = np.where(x == 0, 0.0, x)
        want = np.argsort(-key if desc else key, kind="stable")
        assert np.array_equal(got, want), (dt, desc)


def test_choice_key_batches():
    keys = np.stack([orc.seed(s) for s in range(3)])
    out = jr.vmap(lambda k: jr.random_choice(k, 20, (4,), False))(dev_key(keys))
    assert tuple(out.shape) == (3, 4)
    for r in range(3):
        assert np.array_equal(to_np(out[r]), orc.choice(keys[r], 20, (4,), False))


@pytest.mark.parametrize("dt", ["float32", "float64"])
def test_choice_p_long_vector(dt):
    """Choice with replacement from 100003 unnormalised probabilities: the device cumulative
    sum is taken left to right in the dtype, so every draw matches the oracle's."""
    rng = np.random.default_rng(4)
    p = rng.random(100003).astype(dt)
    p[rng.integers(0, p.size, 1000)] = 0
    key = orc.seed(12)
    with flags(dt == "float64"):
        got = to_np(jr.random_choice(dev_key(key), p.size, (50000,), True, p))
    assert np.array_equal(got, orc.choice(key, p.size, (50000,), True, p, x64=dt == "float64"))
    assert not np.any(p[got] == 0)


def _span_cap(cap):
    from jaxr_b200 import _native as nat
    prev = nat.lib().jxr_set_shuffle_span_cap(cap)
    assert prev >= 0
    return prev


@pytest.mark.parametrize("n", [4096, 4097, 393216, 393217, (1 << 20) + 7, (1 << 27) + 5,
                               (1 << 30) + 3])
def test_span_sort_matches_radix_passes(n):
    """The span sort (radix passes over the top 0, 8, 16 or 24 bits, then every run of
    equal top bits in shared memory) against the radix passes over all four digits, at the
    sizes where the number of top-bit passes changes; the result is a permutation."""
    key = dev_key(orc.seed(31))
    got = jr.random_permutation(key, n)
    prev = _span_cap(0)
    try:
        want = jr.random_permutation(key, n)
    finally:
        _span_cap(prev)
    assert torch.equal(got, want), n
    srt = torch.sort(got.to(torch.int64))[0]
    assert torch.equal(srt, torch.arange(n, dtype=torch.int64, device=srt.device))


@pytest.mark.parametrize("variant", ["original layout", "rbg key", "unsafe_rbg key"])
def test_span_sort_other_key_paths(variant):
    """Sort keys that come from the bits kernels rather than the fused key-and-count kernel
    (the original counter layout; rbg and unsafe_rbg keys): the span sort against the radix
    passes over all four digits at 2^20 + 7 elements (two top-bit passes)."""
    n = (1 << 20) + 7
    if variant == "original layout":
        key, part = dev_key(orc.seed(31)), False
    else:
        key, part = jr.random_key(31, impl=variant.split()[0]), True
    with flags(False, part):
        got = jr.random_permutation(key, n)
        prev = _span_cap(0)
        try:
            want = jr.random_permutation(key, n)
        finally:
            _span_cap(prev)
    assert torch.equal(got, want), variant
    srt = torch.sort(got.to(torch.int64))[0]
    assert torch.equal(srt, torch.arange(n, dtype=torch.int64, device=srt.device))


def test_span_sort_overflow_repeats_with_radix_passes():
    """A span longer than the cap (forced here with a cap of 64) makes the shuffle repeat
    with radix passes alone: the results stay exact against the oracle, for vectors and
    for independent slices."""
    key = orc.seed(2718)
    prev = _span_cap(64)
    try:
        for n in (50, 64, 65, 8193, 100003):
            got = to_np(jr.random_permutation(dev_key(key), n))
            assert np.array_equal(got, orc.permutation(key, n)), n
        x = torch.arange(300 * 40, dtype=torch.int32).reshape(300, 40)
        got = to_np(jr.random_permutation(dev_key(key), x, axis=1, independent=True))
        assert np.array_equal(got, orc.permutation(key, x.numpy(), axis=1, independent=True))
    finally:
        _span_cap(prev)


def test_span_cap_setter():
    from jaxr_b200 import _native as nat
    L = nat.lib()
    prev = L.jxr_set_shuffle_span_cap(4096)
    assert prev == 4096
    assert L.jxr_set_shuffle_span_cap(4097) == -1
    assert b"span cap" in L.jxr_last_error()
    assert L.jxr_set_shuffle_span_cap(-1) == -1
    assert L.jxr_set_shuffle_span_cap(prev) == 4096


def test_vmap_batched_arrays_and_probabilities():
    """vmap over (key, x) for the permutation and over (key, a) / (key, p) for choice, and
    over x, a or p alone with one key, equals the loop over the lanes."""
    keys = jr.random_split(jr.random_key(17), 3)
    x = torch.arange(3 * 4 * 5, dtype=torch.int32).reshape(3, 4, 5)
    for axis, indep in ((0, False), (1, False), (1, True)):
        out = jr.vmap(lambda k, r: jr.random_permutation(k, r, axis=axis, independent=indep))(keys, x)
        assert tuple(out.shape) == (3, 4, 5)
        for i in range(3):
            want = jr.random_permutation(keys[i], x[i], axis=axis, independent=indep)
            assert np.array_equal(to_np(out)[i], to_np(want)), (axis, indep, i)
    out = jr.vmap(lambda r: jr.random_permutation(jr.random_key(5), r))(x[:, 0, :])
    for i in range(3):
        assert np.array_equal(to_np(out)[i], to_np(jr.random_permutation(jr.random_key(5), x[i, 0])))
    a = torch.arange(3 * 7, dtype=torch.int32).reshape(3, 7)
    for replace in (True, False):
        out = jr.vmap(lambda k, r: jr.random_choice(k, r, (4,), replace))(keys, a)
        for i in range(3):
            want = jr.random_choice(keys[i], a[i], (4,), replace)
            assert np.array_equal(to_np(out)[i], to_np(want)), (replace, i)
    ns = torch.tensor([5, 9, 30], dtype=torch.int32)
    out = jr.vmap(lambda k, n: jr.random_choice(k, n, (6,)))(keys, ns)
    for i in range(3):
        assert np.array_equal(to_np(out)[i], to_np(jr.random_choice(keys[i], int(ns[i]), (6,))))
    ps = torch.tensor([[0.2, 0.3, 0.5, 0.0], [0.25, 0.25, 0.25, 0.25], [0.0, 0.0, 1.0, 0.0]])
    for replace in (True, False):
        out = jr.vmap(lambda pr: jr.random_choice(jr.random_key(8), 4, (2,), replace, pr))(ps)
        for i in range(3):
            want = jr.random_choice(jr.random_key(8), 4, (2,), replace, ps[i])
            assert np.array_equal(to_np(out)[i], to_np(want)), (replace, i)
