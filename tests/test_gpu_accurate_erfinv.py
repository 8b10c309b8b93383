"""jax_accurate_erf_inv on the GPU (R/lax_special.R:1022-1082 via the lowering at
:1324-1331): every sampler that evaluates erf_inv -- lax_erf_inv, random_normal (real,
complex, 16-bit, the float32 table path, rbg keys), the fused normal + bernoulli and the
truncated normal (scalar and array bounds) -- bit-exact against the oracle's accurate
erf_inv, whose recorded values the golden cases pin at 0 ulp."""

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


def accurate():
    return jr.with_jax_config("jax_accurate_erf_inv", True)


def same_bits(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b, dtype=a.dtype)
    u = f"u{a.dtype.itemsize}"
    return np.array_equal(a.view(u), b.view(u))


def as_float(bits, dt):
    """The oracle's 16-bit samples (raw bits) as float32 values."""
    if dt not in ("float16", "bfloat16"):
        return bits
    b = np.asarray(bits, dtype=np.uint16)
    if dt == "bfloat16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


@pytest.mark.parametrize("dt", ["float32", "float64"])
def test_lax_erf_inv_accurate(dt):
    npdt = np.float32 if dt == "float32" else np.float64
    rng = np.random.default_rng(8)
    digits = 7 if dt == "float32" else 15
    tail = 1 - 10.0 ** -rng.uniform(1, digits, 1 << 16)
    x = np.concatenate([rng.uniform(-1, 1, 1 << 20), tail, -tail,
                        10.0 ** -rng.uniform(5, 40, 4096),
                        [0.0, -0.0, 1.0, -1.0, 1.5, -2.0, np.nan, np.inf]]).astype(npdt)
    with flags(dt == "float64"), accurate():
        got = to_np(jr.lax_erf_inv(torch.from_numpy(x).cuda()))
    assert same_bits(got, orc.erfinv(x, dt, accurate=True))
    # and the default erf_inv again once the option is off
    with flags(dt == "float64"):
        got = to_np(jr.lax_erf_inv(torch.from_numpy(x[:1000]).cuda()))
    assert same_bits(got, orc.erfinv(x[:1000], dt))


@pytest.mark.parametrize("dt", ["float32", "float64", "float16", "bfloat16"])
@pytest.mark.parametrize("part", [True, False])
def test_normal_accurate(dt, part):
    key = orc.seed(44)
    for n in (1, 1001, 65537):
        with flags(dt == "float64", part), accurate():
            got = to_np(jr.random_normal(dev_key(key), (n,), dt))
        want = as_float(orc.normal(key, dt, n, part, accurate=True), dt)
        assert same_bits(got, want), (dt, part, n)


def test_normal_accurate_float32_table_path():
    """2^22 + 3 float32 normals read the accurate sampler's own 2^23-entry table."""
    key = orc.seed(45)
    n = (1 << 22) + 3
    with accurate():
        got = to_np(jr.random_normal(dev_key(key), (n,), "float32"))
    assert same_bits(got, orc.normal(key, "float32", n, True, accurate=True))
    got = to_np(jr.random_normal(dev_key(key), (n,), "float32"))
    assert same_bits(got, orc.normal(key, "float32", n, True))


@pytest.mark.parametrize("dt", ["complex64", "complex128"])
def test_complex_normal_accurate(dt):
    key = orc.seed(46)
    with flags(dt == "complex128"), accurate():
        got = to_np(jr.random_normal(dev_key(key), (777,), dt))
    want = orc.complex_normal(key, dt, 777, accurate=True)
    real = np.float32 if dt == "complex64" else np.float64
    assert same_bits(got.view(real), want.view(real))


@pytest.mark.parametrize("x64,dt", [(True, "float64"), (False, "float32")])
def test_normal_bernoulli_fused_accurate(x64, dt):
    with flags(x64), accurate():
        k = jr.random_fold_in(jr.random_key(2024), 17)
        nrm, ber = jr.random_normal_bernoulli(k, 0.3, (129, 33), dt)
        assert same_bits(to_np(nrm), to_np(jr.random_normal(k, (129, 33), dt)))
        assert np.array_equal(to_np(ber), to_np(jr.random_bernoulli(k, 0.3, (129, 33))))
    kd = to_np(jr.random_key_data(k)).astype(np.uint32).reshape(2)
    want = orc.normal(kd, dt, 129 * 33, True, accurate=True)
    assert same_bits(to_np(nrm).ravel(), want)


@pytest.mark.parametrize("dt", ["float32", "float64", "float16", "bfloat16"])
def test_truncated_normal_accurate(dt):
    key = orc.seed(47)
    n = 4097
    with flags(dt == "float64"), accurate():
        got = to_np(jr.random_truncated_normal(dev_key(key), -3.0, 2.5, (n,), dt))
    want = as_float(orc.truncated_normal(key, dt, n, -3.0, 2.5, accurate=True), dt)
    assert same_bits(got, want)


def test_rbg_normal_accurate():
    """rbg keys draw normals through the from-bits path."""
    q = np.array([0xDEADBEEF, 0x12345678, 0x9ABCDEF0, 0x0F0F0F0F], dtype=np.uint32)
    k = jr.random_wrap_key_data(torch.tensor(q).cuda(), impl="rbg")
    with accurate():
        got = to_np(jr.random_normal(k, (1000,)))
    bits = orc.rbg_bits(q, 32, 1000)
    f = ((bits >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1)
    lo = np.float32(-1 + 2.0 ** -24)
    u = np.maximum(lo, (f.astype(np.float64) * 2 + lo).astype(np.float32))
    want = (np.float32(np.sqrt(2)) * orc.erfinv(u, "float32", accurate=True)).astype(np.float32)
    assert same_bits(got, want)
