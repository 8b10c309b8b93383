"""Parity of the derived samplers (randint, exponential, gumbel, logistic, laplace,
truncated normal) with the CPU oracle, on the GPU through the public API.

The log-transform samplers and the scalar-bound truncated normal are bit-exact against
the oracle (both evaluate each logarithm with the same operations, in double, and round
once per reference float operation); randint is exact integer work.  The array-bound
truncated normal evaluates erf of the bounds with CUDA's erf and is held to 2 ulp
(float32 and 16-bit) / 1e-12 relative (float64).  Their agreement with the reference's
recorded values is in the golden cases (test_gpu_parity.test_golden_through_public_api).
"""

import numpy as np
import pytest
import torch

import jaxr_b200 as jr
from golden_cases import max_ulp
from oracle import oracle as orc
from product_backend import flags, to_np

pytestmark = pytest.mark.gpu

FLOATS = ["float32", "float64", "float16", "bfloat16"]
KINDS = ["exponential", "gumbel", "logistic", "laplace"]
FN = {"exponential": jr.random_exponential, "gumbel": jr.random_gumbel,
      "logistic": jr.random_logistic, "laplace": jr.random_laplace}


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from jaxr_b200 import build
    build.build()


def dev_key(k):
    return torch.tensor(np.asarray(k, dtype=np.uint32)).cuda()


def raw(t, dt):
    t = t.detach().cpu()
    if dt in ("float16", "bfloat16"):
        return t.view(torch.uint16).numpy()
    return t.numpy()


def as_float(a, dt):
    if dt == "bfloat16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    if dt == "float16":
        return a.view(np.float16)
    return a


def same_bits(got, want, dt):
    gv, wv = as_float(got, dt), as_float(want, dt)
    gn, wn = np.isnan(gv), np.isnan(wv)
    if not np.array_equal(gn, wn):
        return False
    ub = f"u{got.itemsize}"
    return np.array_equal(got[~gn].view(ub), want[~wn].view(ub))


# ---- exponential / gumbel / logistic / laplace ------------------------------------------------

@pytest.mark.parametrize("part", [True, False])
@pytest.mark.parametrize("dt", FLOATS)
@pytest.mark.parametrize("kind", KINDS)
def test_log_samplers_exact(kind, dt, part):
    key = orc.seed(1234)
    for n in (0, 1, 7, 4097, 100003):
        with flags(dt == "float64", part):
            got = raw(FN[kind](dev_key(key), (n,), dt), dt)
        want = orc.sample(key, kind, dt, n, part)
        assert got.shape == want.shape
        assert same_bits(got, want, dt), (kind, dt, part, n)


def test_log_samplers_key_batches():
    keys = np.stack([orc.seed(s) for s in (0, 1, 2)])
    for kind in KINDS:
        out = jr.vmap(lambda k: FN[kind](k, (3, 5)))(dev_key(keys))
        assert tuple(out.shape) == (3, 3, 5)
        for r in range(3):
            want = orc.sample(keys[r], kind, "float32", 15)
            assert same_bits(to_np(out[r]).ravel(), want, "float32"), kind


def test_log_samplers_large_sampled():
    """2^26 float32 samples of each kind, checked at 4096 random positions (both ends
    included), plus range properties over every sample."""
    key = orc.seed(99)
    n = 1 << 26
    rng = np.random.default_rng(5)
    idx = np.unique(np.concatenate([[0, 1, n - 2, n - 1], rng.integers(0, n, 4092)]))
    for kind in KINDS:
        out = FN[kind](dev_key(key), (n,))
        got = to_np(out[torch.from_numpy(idx).cuda()])
        want = orc.sample_at(key, kind, "float32", n, True, idx).astype(np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), kind
        assert bool(torch.isfinite(out).all())
        if kind == "exponential":
            assert float(out.min()) >= 0.0
            assert abs(float(out.double().mean()) - 1.0) < 1e-3
        if kind == "laplace":
            assert abs(float(out.double().mean())) < 1e-3


@pytest.mark.parametrize("dt", FLOATS)
@pytest.mark.parametrize("mode", ["high", "highest"])
def test_gumbel_modes_exact(mode, dt):
    key = orc.seed(31)
    for n in (0, 1, 5, 10007):
        with flags(dt == "float64"):
            got = raw(jr.random_gumbel(dev_key(key), (n,), dt, mode=mode), dt)
        want = orc.gumbel_mode(key, mode, dt, n)
        assert same_bits(got, want, dt), (mode, dt, n)


def test_gumbel_default_mode_follows_config():
    key = dev_key(orc.seed(3))
    low = to_np(jr.random_gumbel(key, (64,)))
    with jr.with_jax_config("jax_use_high_dynamic_range_gumbel", True):
        high = to_np(jr.random_gumbel(key, (64,)))
    assert np.array_equal(low, orc.sample(orc.seed(3), "gumbel", "float32", 64))
    assert np.array_equal(high, orc.gumbel_mode(orc.seed(3), "high", "float32", 64))


# ---- truncated normal -------------------------------------------------------------------------

BOUNDS = [(-1.0, 2.0), (0.5, 0.6), (-3.0, -2.0), (5.0, 6.0), (0.0, np.inf),
          (-np.inf, np.inf), (1.0, 1.0)]


@pytest.mark.parametrize("part", [True, False])
@pytest.mark.parametrize("dt", FLOATS)
def test_truncated_normal_scalar_bounds_exact(dt, part):
    key = orc.seed(77)
    for lo, hi in BOUNDS:
        for n in (1, 4097):
            with flags(dt == "float64", part):
                got = raw(jr.random_truncated_normal(dev_key(key), lo, hi, (n,), dt), dt)
            want = orc.truncated_normal(key, dt, n, lo, hi, part)
            assert same_bits(got, want, dt), (dt, lo, hi, n)
            v = as_float(got, dt).astype(np.float64)
            if lo < hi:
                assert np.all((v > lo) | (np.isinf(lo) & np.isfinite(v))), (dt, lo, hi)
                assert np.all(v < hi), (dt, lo, hi)


@pytest.mark.parametrize("dt", FLOATS)
def test_truncated_normal_array_bounds(dt):
    """Bounds broadcast over (50, 2) as in test-random.R:228; each element against the
    oracle run with that element's bounds."""
    key = orc.seed(7)
    shape = (50, 2)
    lower = np.array([-0.5, 0.0])
    upper = np.array([0.5, 0.1])
    with flags(dt == "float64"):
        out = jr.random_truncated_normal(dev_key(key), lower, upper, shape, dt)
    got = as_float(raw(out, dt), dt).astype(np.float64).reshape(shape)
    n = 100
    for j in range(2):
        col = np.array([as_float(orc.truncated_normal(key, dt, n, lower[j], upper[j], True,
                                                      begin=2 * i + j, count=1), dt)[0]
                        for i in range(50)], dtype=np.float64)
        if dt == "float64":
            assert np.allclose(got[:, j], col, rtol=1e-12, atol=0)
        elif dt == "float32":
            assert max_ulp(got[:, j].astype(np.float32), col.astype(np.float32)) <= 2
        else:  # 2 ulp of the 16-bit type, as a relative difference
            nmant = 7 if dt == "bfloat16" else 10
            diff = np.abs(got[:, j] - col) / np.maximum(np.abs(col), 1e-30)
            assert np.all(diff <= 2 * 2.0 ** -nmant)
        assert np.all(got[:, j] > lower[j]) and np.all(got[:, j] < upper[j])


# ---- randint ------------------------------------------------------------------------------------

INTS = ["int8", "int16", "int32", "uint8", "uint16", "uint32"]
INTS64 = ["int64", "uint64"]


def _randint_check(key, shape, mn, mx, dt, part=True, x64=False):
    with flags(x64, part):
        got = to_np(jr.random_randint(dev_key(key), shape, mn, mx, dt)).ravel()
    want = orc.randint(key, shape, mn, mx, dt, part)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    assert np.array_equal(got, want), (dt, mn, mx, got[:8], want[:8])
    return got


@pytest.mark.parametrize("part", [True, False])
@pytest.mark.parametrize("dt", INTS)
def test_randint_exact(dt, part):
    key = orc.seed(2024)
    bits, signed = orc.INT_INFO[dt]
    lo, hi = orc._int_range(bits, signed)
    i32 = 2**31 - 1  # bounds are int32 with x64 off
    cases = [(0, 10), (-5, 5), (lo, min(hi, i32)), (lo, min(hi + 1, i32)), (7, 7), (9, 3),
             (0, 1), (min(hi, i32) - 3, min(hi, i32))]
    for mn, mx in cases:
        if not signed and mn < 0:
            continue
        for n in (0, 1, 13, 10007):
            got = _randint_check(key, (n,), mn, mx, dt, part)
            if n and mx > mn:
                assert got.min() >= mn and got.max() < mx


@pytest.mark.parametrize("dt", INTS64 + ["int32", "uint32"])
def test_randint_x64_out_of_range_bounds(dt):
    """Under x64 the bounds are int64: maxval beyond the dtype's maximum widens the span by
    one (R/random.R:338-350); a full 2^nbits span reduces to the low draw."""
    key = orc.seed(5, True)
    bits, signed = orc.INT_INFO[dt]
    lo, hi = orc._int_range(bits, signed)
    cases = [(0, 10), (-3, 3) if signed else (0, 3), (lo, min(hi, 2**63 - 1)),
             (0, min(hi, 2**63 - 1))]
    if bits == 32:
        cases += [(lo, hi + 1), (lo - 5, hi + 100)]
    for mn, mx in cases:
        for n in (1, 4097):
            _randint_check(key, (n,), mn, mx, dt, x64=True)


def test_randint_array_bounds_and_key_batches():
    key = orc.seed(0)
    mn = np.array([0, 10, 100], dtype=np.int32)
    mx = np.array([5, 20, 1000], dtype=np.int32)
    for part in (True, False):
        _randint_check(key, (2, 3), mn, mx, "int32", part)
        _randint_check(key, (40, 3), mn, mx, "int32", part)
        _randint_check(key, (40, 3), mn, 1000, "int16", part)
    keys = np.stack([orc.seed(s) for s in range(4)])
    out = jr.vmap(lambda k: jr.random_randint(k, (6,), -5, 5))(dev_key(keys))
    for r in range(4):
        assert np.array_equal(to_np(out[r]), orc.randint(keys[r], (6,), -5, 5, "int32"))
    out = jr.vmap(lambda k: jr.random_randint(k, (2, 3), mn, mx))(dev_key(keys))
    for r in range(4):
        assert np.array_equal(to_np(out[r]).ravel(), orc.randint(keys[r], (2, 3), mn, mx, "int32"))


def test_randint_large_uniformity():
    """2^24 draws of randint(0, 10): every value within 0.5% of n / 10 (the modulo bias of a
    64-bit offset is below 2^-28)."""
    key = dev_key(orc.seed(11))
    out = jr.random_randint(key, (1 << 24,), 0, 10)
    counts = torch.bincount(out.long(), minlength=10).cpu().numpy()
    assert counts.sum() == 1 << 24
    assert np.all(np.abs(counts - (1 << 24) / 10) < 0.005 * (1 << 24) / 10)


_GRAPH_CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import jaxr_b200 as jr
from jaxr_b200 import _native as nat
n = 1 << 22
key = jr.random_key_data(jr.random_key(4242)).cuda()
out = torch.empty(n, dtype=torch.float32, device="cuda")
g = torch.cuda.CUDAGraph()
s = torch.cuda.Stream()
s.wait_stream(torch.cuda.current_stream())
with torch.cuda.stream(s):
    with torch.cuda.graph(g, stream=s):
        nat.call("jxr_sample", key.data_ptr(), 1, n, 0, n, 1, 0, 0, out.data_ptr(), s.cuda_stream)
g.replay()
torch.cuda.synchronize()
want = jr.random_exponential(key, (n,))
assert torch.equal(out.view(torch.int32), want.view(torch.int32))
del g
print("graph ok")
"""


def test_samplers_inside_a_cuda_graph():
    """A fresh process captures a float32 exponential of 2^22 outputs into a CUDA graph
    before the sampler's table exists: evaluated directly during capture (building the
    table would wait on the stream), identical to the table path afterwards."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _GRAPH_CHILD, root], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "graph ok" in r.stdout, r.stderr[-2000:]


@pytest.mark.parametrize("dt", ["complex64", "complex128"])
@pytest.mark.parametrize("part", [True, False])
def test_complex_normal_exact(dt, part):
    """Complex normals (R/random.R:489-499) against the oracle's split-then-divide-by-
    sqrt(2), at an odd size with a ragged tail (and the f32 size above the sampler table's
    threshold, so the real parts come from the table path): complex64 components
    bit-exact, complex128 ones within the float64 normal's 1e-12 relative."""
    key = orc.seed(31)
    for n in (1, 7, 1001, (1 << 22) + 5):
        with flags(dt == "complex128", part):
            got = to_np(jr.random_normal(dev_key(key), (n,), dt))
        want = orc.complex_normal(key, dt, n, part)
        assert got.dtype == want.dtype
        g, w = got.view(got.real.dtype), want.view(want.real.dtype)
        if dt == "complex64":
            assert np.array_equal(g, w), (dt, n)
        else:
            assert np.all(np.abs(g - w) <= 1e-12 * np.abs(w)), (dt, n)


def test_complex_normal_key_batches():
    keys = np.stack([orc.seed(s) for s in range(4)])
    out = to_np(jr.vmap(lambda k: jr.random_normal(k, (2, 3), "complex64"))(dev_key(keys)))
    assert out.shape == (4, 2, 3)
    for r in range(4):
        want = orc.complex_normal(keys[r], "complex64", 6).reshape(2, 3)
        assert np.array_equal(out[r].view(np.float32), want.view(np.float32))


def test_free_caches_then_rebuild():
    """jxr_free_caches releases the sampler tables and the host-copy buffers; the next
    calls rebuild them and give the same results."""
    from jaxr_b200.shard import random_bits_to_host
    key = orc.seed(5)
    n = 1 << 22
    a = to_np(jr.random_normal(dev_key(key), (n,)))
    h1 = random_bits_to_host(jr.random_key(3), (1 << 20,)).numpy().copy()
    jr.free_caches()
    jr.free_caches()  # idempotent
    b = to_np(jr.random_normal(dev_key(key), (n,)))
    h2 = random_bits_to_host(jr.random_key(3), (1 << 20,)).numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(h1, h2)
    assert np.array_equal(a[:4096], orc.normal(key, "float32", n, True, count=4096))


@pytest.mark.parametrize("kind", ["normal"] + KINDS)
def test_table_samplers_every_output(kind):
    """Requests of 2^22 or more float32 samples read the sampler's table for most outputs
    and evaluate a share of each thread's outputs directly (fixed positions in every
    tile): every output compared with the oracle, for one key in both layouts (a ragged
    tail past the last full tile) and for a batch of four keys."""
    fn = jr.random_normal if kind == "normal" else FN[kind]

    def want(k, n, part):
        if kind == "normal":
            return orc.normal(k, "float32", n, part)
        return orc.sample(k, kind, "float32", n, part)

    key = orc.seed(123)
    n = (1 << 22) + 777
    for part in (True, False):
        with flags(False, part):
            got = to_np(fn(dev_key(key), (n,)))
        assert same_bits(got, want(key, n, part), "float32"), (kind, part)
    keys = np.stack([orc.seed(s) for s in range(4)])
    m = (1 << 20) + 3
    got = to_np(jr.vmap(lambda k: fn(k, (m,)))(dev_key(keys)))
    for r in range(4):
        assert same_bits(got[r], want(keys[r], m, True), "float32"), (kind, r)


def test_truncated_normal_table_in_the_call():
    """float32 truncated normals of 2^25 or more samples build the table for their bounds in
    the call and read most samples from it: every output against the oracle, one key in
    both layouts (a ragged tail), a batch of two keys, and with the accurate erf_inv."""
    key = orc.seed(31)
    n = (1 << 25) + 777
    for part in (True, False):
        with flags(False, part):
            got = to_np(jr.random_truncated_normal(dev_key(key), -0.7, 2.25, (n,)))
        assert same_bits(got, orc.truncated_normal(key, "float32", n, -0.7, 2.25, part),
                         "float32"), part
    keys = np.stack([orc.seed(s) for s in (4, 5)])
    m = (1 << 24) + 5
    got = to_np(jr.vmap(lambda k: jr.random_truncated_normal(k, -3.0, 1.5, (m,)))(dev_key(keys)))
    for r in range(2):
        assert same_bits(got[r], orc.truncated_normal(keys[r], "float32", m, -3.0, 1.5),
                         "float32"), r
    with jr.with_jax_config("jax_accurate_erf_inv", True):
        got = to_np(jr.random_truncated_normal(dev_key(key), -0.7, 2.25, (n,)))
    assert same_bits(got, orc.truncated_normal(key, "float32", n, -0.7, 2.25, accurate=True),
                     "float32")


def test_truncated_normal_scratch_entry_point():
    """jxr_truncated_normal_scratch through the C ABI: with a table-sized scratch, with one
    too small (it falls back to jxr_truncated_normal) and below the size threshold, the
    same samples as jxr_truncated_normal."""
    from jaxr_b200 import _native as nat
    kd = dev_key(orc.seed(8)).view(1, 2)
    st = torch.cuda.current_stream().cuda_stream
    for n, scratch_words in (((1 << 25) + 3, 1 << 23), ((1 << 25) + 3, 1000), (4097, 1 << 23)):
        ref = torch.empty(n, dtype=torch.float32, device="cuda")
        nat.call("jxr_truncated_normal", kd.data_ptr(), 1, n, 0, n, 1, nat.F32, -1.0, 2.0,
                 ref.data_ptr(), st)
        got = torch.empty_like(ref)
        scratch = torch.empty(scratch_words, dtype=torch.float32, device="cuda")
        nat.call("jxr_truncated_normal_scratch", kd.data_ptr(), 1, n, 0, n, 1, nat.F32, -1.0, 2.0,
                 scratch.data_ptr(), scratch_words * 4, got.data_ptr(), st)
        assert torch.equal(got.view(torch.int32), ref.view(torch.int32)), (n, scratch_words)


@pytest.mark.parametrize("dt", ["float16", "bfloat16"])
@pytest.mark.parametrize("kind", ["normal", "normal_accurate"] + KINDS)
def test_16bit_table_samplers_every_output(kind, dt):
    """16-bit samplers of 2^16 or more samples read the table of their 1024 (float16) or
    128 (bfloat16) possible results: every output against the oracle, one key in both
    layouts and a batch of three keys."""
    def sample(k, shape):
        if kind.startswith("normal"):
            return jr.random_normal(k, shape, dt)
        return FN[kind](k, shape, dt)

    def want(k, n, part):
        if kind.startswith("normal"):
            return orc.normal(k, dt, n, part, accurate=kind == "normal_accurate")
        return orc.sample(k, kind, dt, n, part)

    def acc():
        return jr.with_jax_config("jax_accurate_erf_inv", kind == "normal_accurate")

    key = orc.seed(64)
    n = (1 << 17) + 5
    for part in (True, False):
        with flags(False, part), acc():
            got = to_np(sample(dev_key(key), (n,)))
        assert same_bits_h(got, want(key, n, part), dt), part
    keys = np.stack([orc.seed(s) for s in range(3)])
    m = (1 << 16) + 1
    with acc():
        got = to_np(jr.vmap(lambda k: sample(k, (m,)))(dev_key(keys)))
    for r in range(3):
        assert same_bits_h(got[r], want(keys[r], m, True), dt), r


def same_bits_h(got_values, want_bits, dt):
    """16-bit results (as float32 values) against the oracle's raw 16-bit patterns."""
    g = np.asarray(got_values, dtype=np.float32)
    w = np.asarray(as_float(np.asarray(want_bits), dt), dtype=np.float32)
    gn, wn = np.isnan(g), np.isnan(w)
    return np.array_equal(gn, wn) and np.array_equal(g[~gn].view(np.uint32), w[~wn].view(np.uint32))


@pytest.mark.parametrize("dt", ["float16", "bfloat16"])
def test_16bit_truncated_normal_table_in_the_call(dt):
    """16-bit truncated normals of 2^16 or more samples build the table of their bounds
    (1024 / 128 entries) in the call: every output against the oracle in both layouts."""
    key = orc.seed(65)
    n = (1 << 17) + 5
    for part in (True, False):
        with flags(False, part):
            got = to_np(jr.random_truncated_normal(dev_key(key), -0.5, 3.0, (n,), dt))
        assert same_bits_h(got, orc.truncated_normal(key, dt, n, -0.5, 3.0, part), dt), part


@pytest.mark.parametrize("kind", ["normal", "exponential", "gumbel", "logistic", "laplace"])
def test_float32_samplers_every_draw(kind):
    """Every float32 sample depends only on bits >> 9 of its draw: all 2^23 of them
    through the from-bits transforms, evaluated directly (no table is prepared), each
    bit-identical with the oracle's (its logarithms are Cody and Waite's, the kernels'
    a table-driven one: over these inputs both round to the same floats)."""
    from jaxr_b200 import _native as nat
    jr.free_caches()
    n = 1 << 23
    bits = (torch.arange(n, dtype=torch.int64) << 9).to(torch.uint32).cuda()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    if kind == "normal":
        nat.call("jxr_normal_from_bits", bits.data_ptr(), n, nat.F32, out.data_ptr(), st)
    else:
        nat.call("jxr_sample_from_bits", bits.data_ptr(), n, orc.SAMPLE_KIND[kind], nat.F32,
                 out.data_ptr(), st)
    got = to_np(out)
    want = orc.sample_f32_from_bits(bits.cpu().numpy(), kind)
    diff = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert diff.size == 0, (kind, diff[:8], got[diff[:8]], want[diff[:8]])
