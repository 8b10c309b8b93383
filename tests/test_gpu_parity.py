"""Parity of the sm_100a kernels with the reference (golden vectors) and the CPU oracle.

Integer bits and keys must match exactly; uniforms and bernoulli draws exactly
(bitwise); normals within 2 ulp (float32) / 1e-12 relative (float64); every float32 or
16-bit normal the reference recorded at 0 ulp, and every float64 one within its own
tests' 16 ulp (the float64 normal sampler takes its logarithm from a table-driven
method, not the oracle's).  Sizes run from the empty request to the
named workloads (C1-C5); large requests are checked at sampled positions, which the
oracle computes element by element from their counters.
"""

import numpy as np
import pytest
import torch

import jaxr_b200 as jr
from golden_cases import (check, evaluate, expected, float_dtype, load_cases, max_ulp,
                          ulp_distance)
from product_backend import ProductBackend, flags, to_np

pytestmark = pytest.mark.gpu

CASES = load_cases()
ODD_SIZES = [0, 1, 2, 3, 5, 7, 8, 9, 15, 16, 17, 255, 256, 257, 1000, 4097, 65537]


def dev_key(k):
    return torch.tensor(np.asarray(k, dtype=np.uint32)).cuda()


_SIGNED = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def take(t, idx):
    """t.reshape(-1)[idx] as numpy, for any dtype (unsigned tensors are gathered through
    their signed views)."""
    flat = t.reshape(-1)
    ti = torch.from_numpy(np.asarray(idx, dtype=np.int64)).to(flat.device)
    if flat.dtype in (torch.uint16, torch.uint32, torch.uint64):
        g = flat.view(_SIGNED[flat.element_size()])[ti].cpu().numpy()
        return g.view({2: np.uint16, 4: np.uint32, 8: np.uint64}[flat.element_size()])
    return to_np(flat[ti])


def _as_float(a, dt):
    if dt == "bfloat16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    if dt == "float16":
        return a.view(np.float16)
    return a


def same_bits(got, want, dt):
    """Bitwise equality, NaN payloads aside (any NaN equals any NaN)."""
    gv, wv = _as_float(got, dt), _as_float(want, dt)
    gn, wn = np.isnan(gv), np.isnan(wv)
    if not np.array_equal(gn, wn):
        return False
    ub = f"u{got.itemsize}"
    return np.array_equal(got[~gn].view(ub), want[~wn].view(ub))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from jaxr_b200 import build
    build.build()


# ---- golden vectors of the reference ---------------------------------------------------------

def _f64_normal(case):
    """A float64 (or complex128) normal: held to 1e-12 relative (the float64 normal's bar)
    and the reference's own 16 ulp (test-random.R:10-27), since its logarithm is not the oracle's."""
    return case["op"] in ("normal", "vmap_normal") and float_dtype(case["args"]) in (
        "float64", "complex128")


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden_through_public_api(case):
    if _f64_normal(case):
        case = dict(case, compare="ulp16", max_ulp=16)
    a = case["args"]
    be = ProductBackend(x64=bool(a.get("x64", False)), partitionable=a.get("partitionable", True))
    got = evaluate(case, be)
    ok, detail = check(case, got)
    assert ok, f"{case['name']} ({case['source']}): {detail}"
    want = expected(case)
    if _f64_normal(case):
        g = np.asarray(got).astype(want.dtype).ravel().view(want.real.dtype)
        w = np.asarray(want).ravel().view(want.real.dtype)
        assert np.all(np.abs(g - w) <= 1e-12 * np.abs(w)), case["source"]
    if want.dtype.kind == "f" and np.all(np.isfinite(want)):
        assert max_ulp(np.asarray(got).astype(want.dtype), want) <= case.get("max_ulp", 0), \
            case["source"]


def _golden(name):
    return next(c for c in CASES if c["name"] == name)


def test_vmap_over_key_batches_golden():
    # tests/testthat/test-prng.R:190-195 and test-random.R:292-297
    k0 = jr.random_PRNGKey(0)
    out = jr.vmap(lambda k: jr.random_split(k))(jr.random_split(k0, 3))
    assert np.array_equal(to_np(out), expected(_golden("vmap_split")))
    out = jr.vmap(lambda d: jr.random_fold_in(k0, d))(torch.arange(3, dtype=torch.int32))
    assert np.array_equal(to_np(out), expected(_golden("vmap_fold_in")))
    out = jr.vmap(lambda s: jr.random_key_data(jr.random_key(s)))(torch.arange(3, dtype=torch.int32))
    assert np.array_equal(to_np(out), expected(_golden("vmap_key")))
    out = jr.vmap(lambda k: jr.random_uniform(k, 3))(jr.random_split(k0, 4))
    assert max_ulp(to_np(out), expected(_golden("vmap_uniform"))) == 0
    keys = jr.random_split(jr.random_key(7), 3)
    v = jr.vmap(lambda k: jr.random_normal(k, 2))(keys)
    assert isinstance(keys, jr.PRNGKeyArray)
    want = expected(_golden("vmap_normal_exact"))
    assert np.array_equal(to_np(v).view(np.uint32), want.view(np.uint32))  # bit for bit
    for i, ki in enumerate(keys):
        assert np.array_equal(to_np(jr.random_normal(ki, 2)), to_np(v)[i])
    # vmap of bits equals a loop over the keys (test-prng.R:196-200)
    K = jr.random_key(0)
    vb = jr.vmap(lambda k: jr.random_bits(k, 2))(jr.random_split(K, 3))
    for i, ki in enumerate(jr.random_split(K, 3)):
        assert np.array_equal(to_np(vb)[i], to_np(jr.random_bits(ki, 2)))


def test_nested_vmap():
    keys = jr.random_split(jr.random_key(1), (2, 3))
    out = jr.vmap(jr.vmap(lambda k: jr.random_uniform(k, 4)))(keys)
    assert tuple(out.shape) == (2, 3, 4)
    for i in range(2):
        for j in range(3):
            assert np.array_equal(to_np(out)[i, j], to_np(jr.random_uniform(keys[i, j], 4)))


# ---- bits: exact against the oracle ------------------------------------------------------------

@pytest.mark.parametrize("part", [True, False], ids=["partitionable", "original"])
@pytest.mark.parametrize("bw", [8, 16, 32, 64])
def test_bits_exact_odd_sizes(oracle, part, bw):
    key = np.array([0x13198A2E, 0x03707344], np.uint32)
    for n in ODD_SIZES:
        with flags(bw == 64, part):
            got = to_np(jr.random_bits(dev_key(key), (n,), f"uint{bw}"))
        want = oracle.random_bits(key, bw, n, part)
        assert np.array_equal(got, want), (n, bw, part)


@pytest.mark.parametrize("part", [True, False], ids=["partitionable", "original"])
@pytest.mark.parametrize("bw", [8, 16, 32, 64])
def test_bits_ranges_through_abi(oracle, part, bw):
    """Element ranges [begin, begin + count) of a request (the shard interface)."""
    from jaxr_b200 import _native as nat
    key = np.array([7, 0xDEADBEEF], np.uint32)
    kd = dev_key(key)
    size = 100003
    whole = oracle.random_bits(key, bw, size, part)
    dt = {8: torch.uint8, 16: torch.uint16, 32: torch.uint32, 64: torch.uint64}[bw]
    for begin, count in [(0, size), (1, 17), (3, 1000), (49999, 5), (50000, 50003), (size - 1, 1),
                         (12345, 0), (4, 65536)]:
        out = torch.empty(count, dtype=dt, device="cuda")
        nat.call("jxr_random_bits", kd.data_ptr(), 1, size, begin, count,
                 int(part), bw, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert np.array_equal(to_np(out), whole[begin:begin + count]), (begin, count)


def test_bits_high_counter_words(oracle):
    """Counters past 2^32 carry into the high word (R/prng.R:130-148)."""
    from jaxr_b200 import _native as nat
    key = np.array([1, 2], np.uint32)
    kd = dev_key(key)
    size = (1 << 34) + 11
    for begin in [(1 << 32) - 7, (1 << 33) + 1, size - 300]:
        out = torch.empty(300, dtype=torch.uint32, device="cuda")
        nat.call("jxr_random_bits", kd.data_ptr(), 1, size, begin, 300, 1, 32, out.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
        want = oracle.bits_at(key, 32, size, True, range(begin, begin + 300))
        assert np.array_equal(to_np(out), want)


def test_key_batches_exact(oracle):
    keys = np.random.default_rng(3).integers(0, 2**32, size=(37, 2), dtype=np.uint64).astype(np.uint32)
    for part in (True, False):
        for n in (1, 5, 1024, 1027):
            with flags(False, part):
                got = to_np(jr.vmap(lambda k: jr.random_bits(k, n))(dev_key(keys)))
            for r in range(keys.shape[0]):
                assert np.array_equal(got[r], oracle.random_bits(keys[r], 32, n, part)), (part, n, r)


def test_split_fold_in_primitives(oracle):
    rng = np.random.default_rng(5)
    for _ in range(8):
        key = rng.integers(0, 2**32, size=2, dtype=np.uint64).astype(np.uint32)
        for part in (True, False):
            with flags(False, part):
                got = to_np(jr.random_split(dev_key(key), 7))
            assert np.array_equal(got, oracle.split(key, 7, part))
        d = int(rng.integers(0, 2**32))
        assert np.array_equal(to_np(jr.random_fold_in(dev_key(key), d)), oracle.fold_in(key, d))
    k1, k2, c1, c2 = (rng.integers(0, 2**32, size=(3, 4), dtype=np.uint64).astype(np.uint32)
                      for _ in range(4))
    x0, x1 = jr.threefry2x32(*(torch.tensor(a) for a in (k1, k2, c1, c2)))
    for idx in np.ndindex(3, 4):
        assert (int(to_np(x0)[idx]), int(to_np(x1)[idx])) == oracle.threefry2x32(
            int(k1[idx]), int(k2[idx]), int(c1[idx]), int(c2[idx]))


# ---- samplers ----------------------------------------------------------------------------------

@pytest.mark.parametrize("part", [True, False], ids=["partitionable", "original"])
@pytest.mark.parametrize("dt", ["float32", "float64", "float16", "bfloat16"])
def test_uniform_exact(oracle, part, dt):
    key = np.array([0, 42], np.uint32)
    for mn, mx in [(0.0, 1.0), (-2.0, 3.0), (1e-3, 7.5), (-1e30, 1e30)]:
        for n in (1, 7, 1024, 4099):
            with flags(dt == "float64", part):
                out = jr.random_uniform(dev_key(key), (n,), dt, mn, mx)
            got = out.detach().cpu().view(torch.uint16).numpy() if dt in ("float16", "bfloat16") \
                else to_np(out)
            want = oracle.uniform(key, dt, n, part, mn, mx)
            assert same_bits(got, want, dt), (mn, mx, n)


def test_uniform_unfused_flag(oracle):
    from jaxr_b200 import _native as nat
    key = np.array([0, 42], np.uint32)
    n = 4096
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    nat.call("jxr_uniform", dev_key(key).data_ptr(), 1, n, 0, n, 1, nat.F32, -2.0, 3.0,
             nat.FLAG_UNFUSED_MUL_ADD, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    want = oracle.uniform(key, "float32", n, True, -2.0, 3.0, fma=False)
    assert np.array_equal(to_np(out).view(np.uint32), want.view(np.uint32))


def test_normal_f32_all_reachable_uniforms(oracle):
    """The float32 normal depends only on bits >> 9: all 2^23 of them, through the
    transform entry point, against the oracle."""
    from jaxr_b200 import _native as nat
    bits = (torch.arange(1 << 23, dtype=torch.int64) << 9).to(torch.uint32).cuda()
    out = torch.empty(1 << 23, dtype=torch.float32, device="cuda")
    nat.call("jxr_normal_from_bits", bits.data_ptr(), 1 << 23, nat.F32, out.data_ptr(),
             torch.cuda.current_stream().cuda_stream)
    got = to_np(out)
    # oracle: normal of draw k is the normal of a request whose bits are k << 9; compute
    # through uniform + erfinv of the oracle at every k
    k = np.arange(1 << 23, dtype=np.uint32)
    f = ((k | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)).astype(np.float32)
    lo = np.float32(-1 + 2.0 ** -24)
    u = np.maximum(lo, (f * np.float32(2.0) + lo).astype(np.float32))
    want = (np.float32(np.sqrt(2)) * oracle.erfinv(u, "float32")).astype(np.float32)
    d = ulp_distance(got, want)
    assert d.max() <= 2, f"max {d.max()} ulp"
    assert np.count_nonzero(d) <= 64, f"{np.count_nonzero(d)} values differ"


def test_normal_samples(oracle):
    rng = np.random.default_rng(11)
    for part in (True, False):
        for dt, tol in [("float32", None), ("float64", 1e-12), ("float16", None), ("bfloat16", None)]:
            key = rng.integers(0, 2**32, size=2, dtype=np.uint64).astype(np.uint32)
            n = 20011
            with flags(dt == "float64", part):
                out = jr.random_normal(dev_key(key), (n,), dt)
            want = oracle.normal(key, dt, n, part)
            if dt in ("float16", "bfloat16"):
                assert np.array_equal(out.detach().cpu().view(torch.uint16).numpy(), want)
            elif dt == "float32":
                assert ulp_distance(to_np(out), want).max() <= 2
            else:
                got = to_np(out)
                assert np.all(np.abs(got - want) <= tol * np.abs(want))


def test_erf_inv_edges():
    x = torch.tensor([0.0, -0.0, 0.5, -0.9, 1.0, -1.0, 1.5, float("nan"), float("inf")],
                     dtype=torch.float32)
    y = to_np(jr.lax_erf_inv(x))
    assert y[0] == 0 and np.signbit(y[1]) and y[4] == np.inf and y[5] == -np.inf
    assert np.isnan(y[6]) and np.isnan(y[7]) and np.isnan(y[8])


@pytest.mark.parametrize("dt", ["float32", "float64"])
def test_erf_inv_bit_exact_with_oracle(oracle, dt):
    """lax_erf_inv on 2^20 + tail values: uniform in (-1, 1), within 1e-3..1e-15 of +-1,
    tiny and subnormal magnitudes, the exact ends and zeros; every result bit-identical
    with the oracle's."""
    npdt = np.float32 if dt == "float32" else np.float64
    rng = np.random.default_rng(3)
    digits = 7 if dt == "float32" else 15
    tail = 1 - 10.0 ** -rng.uniform(3, digits, 1 << 16)
    tiny = 10.0 ** -rng.uniform(5, 300 if dt == "float64" else 40, 1 << 12)
    x = np.concatenate([rng.uniform(-1, 1, 1 << 20), tail, -tail, tiny, -tiny,
                        [0.0, -0.0, 1.0, -1.0, np.finfo(npdt).tiny, np.finfo(npdt).eps]])
    x = x.astype(npdt)
    with flags(dt == "float64"):
        got = to_np(jr.lax_erf_inv(torch.from_numpy(x).cuda()))
    want = oracle.erfinv(x, dt)
    assert np.array_equal(got.view(f"u{npdt().itemsize}"), want.view(f"u{npdt().itemsize}"))


@pytest.mark.parametrize("part", [True, False], ids=["partitionable", "original"])
@pytest.mark.parametrize("dt", ["float32", "float64", "float16", "bfloat16"])
def test_bernoulli_exact(oracle, part, dt):
    key = np.array([0, 7], np.uint32)
    for p in (0.0, 0.3, 0.5, 0.999, 1.0):
        for n in (8, 1000, 4097):
            with flags(dt == "float64", part):
                pt = torch.tensor(p, dtype=getattr(torch, dt))
                got = to_np(jr.random_bernoulli(dev_key(key), pt, (n,)))
            want = oracle.bernoulli(key, dt, p, n, part).astype(bool)
            assert np.array_equal(got, want), (p, n)


def test_normal_bernoulli_fused_equals_separate():
    for x64, dt in ((True, "float64"), (False, "float32")):
        for part in (True, False):
            with flags(x64, part):
                k = jr.random_fold_in(jr.random_key(2024), 17)
                nrm, ber = jr.random_normal_bernoulli(k, 0.3, (129, 33), dt)
                assert np.array_equal(to_np(nrm), to_np(jr.random_normal(k, (129, 33), dt)))
                assert np.array_equal(to_np(ber), to_np(jr.random_bernoulli(k, 0.3, (129, 33))))


# ---- the named workloads C1-C5, checked at sampled positions ----------------------------------

def _sample_idx(size, n=4096, seed=0):
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, size, n, dtype=np.uint64)
    edges = np.array([0, 1, 2, 3, size // 2 - 1, size // 2, size - 2, size - 1], dtype=np.uint64)
    return np.unique(np.concatenate([idx, edges]))


def test_config1_bits_2p20(oracle):
    k = jr.random_key(0)
    got = to_np(jr.random_bits(k, (1 << 20,)))
    assert np.array_equal(got, oracle.random_bits(oracle.seed(0), 32, 1 << 20, True))


@pytest.mark.parametrize("part", [True, False], ids=["partitionable", "original"])
def test_config2_normal_8192sq(oracle, part):
    size = 8192 * 8192
    with flags(False, part):
        out = jr.random_normal(jr.random_key(42), (8192, 8192))
    assert tuple(out.shape) == (8192, 8192)
    idx = _sample_idx(size)
    got = take(out, idx)
    want = oracle.normal_at(oracle.seed(42), "float32", size, part, True, idx).astype(np.float32)
    assert ulp_distance(got, want).max() <= 2


def test_config3_vmap_uniform(oracle):
    keys = jr.random_split(jr.random_key(7), 65536)
    out = jr.vmap(lambda k: jr.random_uniform(k, (1024,), minval=-2, maxval=3))(keys)
    assert tuple(out.shape) == (65536, 1024)
    kd = to_np(keys.data)
    assert np.array_equal(kd, oracle.split(oracle.seed(7), 65536, True))
    rng = np.random.default_rng(1)
    for r in list(rng.integers(0, 65536, 24)) + [0, 65535]:
        want = oracle.uniform(kd[r], "float32", 1024, True, -2.0, 3.0)
        assert np.array_equal(to_np(out[r]).view(np.uint32), want.view(np.uint32)), r


def test_config4_bits_2p34_sampled(oracle):
    """2^34 uint32 words (64 GiB): sampled positions against the oracle, and shards of
    the request equal the corresponding slices of the whole."""
    from jaxr_b200 import _native as nat
    free, _ = torch.cuda.mem_get_info()
    size = 1 << 34
    if free < size * 4 + (4 << 30):
        pytest.skip("needs 68 GiB of free device memory")
    k = jr.random_key(123)
    out = jr.random_bits(k, (size,))
    idx = _sample_idx(size, 8192)
    got = take(out, idx)
    assert np.array_equal(got, oracle.bits_at(oracle.seed(123), 32, size, True, idx))
    for r in range(8):  # the 8-way shard layout
        lo = r * (size // 8)
        part = torch.empty(1 << 20, dtype=torch.uint32, device="cuda")
        nat.call("jxr_random_bits", k.data.data_ptr(), 1, size, lo, 1 << 20, 1, 32,
                 part.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert torch.equal(part.view(torch.int32), out[lo:lo + (1 << 20)].view(torch.int32))
    del out
    torch.cuda.empty_cache()


def test_config5_x64_normal_bernoulli(oracle):
    size = 16384 * 16384
    with flags(True, True):
        k = jr.random_fold_in(jr.random_key(2024), 17)
        nrm, ber = jr.random_normal_bernoulli(k, 0.3, (16384, 16384))
        assert nrm.dtype == torch.float64 and ber.dtype == torch.bool
    kk = oracle.fold_in(oracle.seed(2024, x64=True), 17)
    idx = _sample_idx(size)
    got = take(nrm, idx)
    want = oracle.normal_at(kk, "float64", size, True, True, idx)
    assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want))
    gb = take(ber, idx)
    wb = oracle.uniform_at(kk, "float64", size, True, 0.0, 1.0, True, idx) < 0.3
    assert np.array_equal(gb, wb)
    frac = ber.float().mean().item()
    assert abs(frac - 0.3) < 1e-3


# ---- bits into host memory (the host-buffer entry point) -----------------------------------------

def test_random_bits_to_host(oracle):
    from jaxr_b200.shard import random_bits_to_host
    k = jr.random_key(123)
    n = (1 << 26) + 12345  # several 64 MiB chunks and a ragged tail
    h = torch.empty(n, dtype=torch.uint32, pin_memory=True)
    for _ in range(2):  # two calls in a row reuse the staging buffers
        out = random_bits_to_host(k, (n,), out=h)
        assert out.device.type == "cpu"
        idx = _sample_idx(n)
        assert np.array_equal(out.numpy()[idx], oracle.bits_at(oracle.seed(123), 32, n, True, idx))
    whole = jr.random_bits(k, (n,))
    assert torch.equal(out.view(torch.int32), whole.cpu().view(torch.int32))


@pytest.mark.parametrize("part", [True, False], ids=["partitionable", "original"])
@pytest.mark.parametrize("bw", [8, 16, 32, 64])
def test_bits_host_abi_all_widths(oracle, part, bw):
    import ctypes
    from jaxr_b200 import _native as nat
    keys = np.array([[0, 7], [3, 4], [0xFFFFFFFF, 1]], dtype=np.uint32)
    size, begin, count = 300001, 17, 299000
    npdt = {8: np.uint8, 16: np.uint16, 32: np.uint32, 64: np.uint64}[bw]
    out = np.zeros((3, count), dtype=npdt)
    nat.call("jxr_random_bits_host", keys.ctypes.data_as(ctypes.c_void_p), 3, size, begin, count,
             int(part), bw, out.ctypes.data_as(ctypes.c_void_p))
    for r in range(3):
        assert np.array_equal(out[r], oracle.random_bits(keys[r], bw, size, part, begin, count))


# ---- original layout above 2^32 - 1 words: the key is split (R/prng.R:233-245) ----------------

U32M = (1 << 32) - 1
SPLIT_CASES = {  # bit width -> (size, element ranges around the segment boundaries)
    32: ((1 << 32) + 105, [(0, 40), (U32M - 20, 40), ((1 << 32) + 105 - 30, 30)]),
    64: ((1 << 31) + 3, [(0, 40), ((1 << 31) - 12, 15), (1 << 30, 16)]),
    16: ((1 << 33) + 107, [(0, 40), (2 * U32M - 20, 40), ((1 << 33) + 107 - 25, 25)]),
    8: ((1 << 34) + 109, [(0, 64), (4 * U32M - 30, 60), ((1 << 34) + 109 - 33, 33)]),
}


@pytest.mark.parametrize("bw", [8, 16, 32, 64])
def test_original_layout_key_splitting(oracle, bw):
    from jaxr_b200 import _native as nat
    size, ranges = SPLIT_CASES[bw]
    key = np.array([0x13198A2E, 0x03707344], np.uint32)
    kd = dev_key(np.stack([key, key ^ 0x5A5A5A5A]))
    dt = {8: torch.uint8, 16: torch.uint16, 32: torch.uint32, 64: torch.uint64}[bw]
    for begin, count in ranges:
        out = torch.empty((2, count), dtype=dt, device="cuda")
        nat.call("jxr_random_bits", kd.data_ptr(), 2, size, begin, count, 0, bw, out.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
        got = to_np(out)
        for r, k in enumerate((key, key ^ 0x5A5A5A5A)):
            want = oracle.bits_at(k, bw, size, False, range(begin, begin + count))
            assert np.array_equal(got[r], want), (bw, begin, r)


def test_original_layout_key_splitting_samplers(oracle):
    from jaxr_b200 import _native as nat
    key = np.array([0, 42], np.uint32)
    kd = dev_key(key)
    st = torch.cuda.current_stream().cuda_stream
    size, begin, count = (1 << 32) + 105, U32M - 20, 40
    out = torch.empty(count, dtype=torch.float32, device="cuda")
    nat.call("jxr_uniform", kd.data_ptr(), 1, size, begin, count, 0, nat.F32, -2.0, 3.0, 0,
             out.data_ptr(), st)
    want = oracle.uniform_at(key, "float32", size, False, -2.0, 3.0, True, range(begin, begin + count))
    assert np.array_equal(to_np(out), want.astype(np.float32))
    size, begin, count = (1 << 31) + 3, (1 << 31) - 12, 15
    out = torch.empty(count, dtype=torch.float64, device="cuda")
    nat.call("jxr_normal", kd.data_ptr(), 1, size, begin, count, 0, nat.F64, out.data_ptr(), st)
    want = oracle.normal_at(key, "float64", size, False, True, range(begin, begin + count))
    assert np.all(np.abs(to_np(out) - want) <= 1e-12 * np.abs(want))


def test_bits_fuzz_ranges_and_batches(oracle):
    """300 seeded random requests through jxr_random_bits: 1-5 keys, sizes up to 2^20 (and
    a few past 2^32 words, checked by range), random [begin, begin + count), both layouts,
    all widths; every element against the oracle."""
    from jaxr_b200 import _native as nat
    rng = np.random.default_rng(2026)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(300):
        nkeys = int(rng.integers(1, 6))
        big = rng.random() < 0.05
        size = int(rng.integers(1 << 32, (1 << 33))) if big else int(rng.integers(0, 1 << 20))
        begin = int(rng.integers(0, size + 1))
        count = int(rng.integers(0, min(size - begin, 5000 if big else 1 << 18) + 1))
        part = bool(rng.integers(0, 2)) if not big else True
        bw = int(rng.choice([8, 16, 32, 64]))
        keys = rng.integers(0, 1 << 32, (nkeys, 2), dtype=np.uint64).astype(np.uint32)
        kd = torch.from_numpy(keys).cuda()
        out = torch.empty((nkeys, max(count, 1)), dtype={8: torch.uint8, 16: torch.int16,
                                                          32: torch.int32, 64: torch.int64}[bw],
                          device="cuda")
        nat.call("jxr_random_bits", kd.data_ptr(), nkeys, size, begin, count,
                 1 if part else 0, bw, out.data_ptr(), stream)
        got = out.cpu().numpy()[:, :count].view({8: np.uint8, 16: np.uint16, 32: np.uint32,
                                                 64: np.uint64}[bw])
        for r in range(nkeys):
            want = oracle.random_bits(keys[r], bw, size, part, begin, count)
            assert np.array_equal(got[r], want), (nkeys, size, begin, count, part, bw, r)


def test_vmap_batched_sampler_parameters():
    """vmap over (key, bound) and (key, p) pairs, and over p alone with one key, equals the
    loop over the lanes (the reference's vmap batches every primitive argument,
    R/batching.R:22-50)."""
    keys = jr.random_split(jr.random_key(11), 4)
    mins = torch.tensor([-2.0, 0.0, 1.5, -0.25])
    for dt in ("float32", "float16"):
        out = jr.vmap(lambda k, m: jr.random_uniform(k, (5,), dt, minval=m, maxval=3))(keys, mins)
        assert tuple(out.shape) == (4, 5)
        for i in range(4):
            want = jr.random_uniform(keys[i], (5,), dt, minval=float(mins[i]), maxval=3)
            assert np.array_equal(to_np(out)[i], to_np(want)), (dt, i)
    # array bounds per lane, broadcast along the shape
    rows = torch.tensor([[0.0, 1.0, 2.0], [5.0, 6.0, 7.0]])
    k2 = jr.random_split(jr.random_key(12), 2)
    out = jr.vmap(lambda k, m: jr.random_uniform(k, (4, 3), minval=m, maxval=10))(k2, rows)
    for i in range(2):
        want = jr.random_uniform(k2[i], (4, 3), minval=rows[i], maxval=10)
        assert np.array_equal(to_np(out)[i], to_np(want))
    # one key for every lane: every lane draws the same unit floats
    out = jr.vmap(lambda m: jr.random_uniform(jr.random_key(3), (6,), minval=m), in_axes=0)(mins)
    for i in range(4):
        want = jr.random_uniform(jr.random_key(3), (6,), minval=float(mins[i]))
        assert np.array_equal(to_np(out)[i], to_np(want))
    ps = torch.tensor([0.1, 0.5, 0.9, 0.3], dtype=torch.float32)
    for mode in ("low", "high"):
        out = jr.vmap(lambda k, p: jr.random_bernoulli(k, p, (64,), mode=mode))(keys, ps)
        for i in range(4):
            want = jr.random_bernoulli(keys[i], ps[i], (64,), mode=mode)
            assert np.array_equal(to_np(out)[i], to_np(want)), (mode, i)


def test_vmap_batched_truncated_normal_and_randint_bounds(oracle):
    """vmap over (key, bounds) for the truncated normal and randint, and over the bounds
    alone with one key, equals the loop over the lanes with each lane's bounds given as
    arrays; randint also against the oracle lane by lane."""
    keys = jr.random_split(jr.random_key(21), 3)
    lows = torch.tensor([-1.0, 0.0, -2.5])
    for dt in ("float32", "float64", "bfloat16"):
        out = jr.vmap(lambda k, lo: jr.random_truncated_normal(k, lo, 2.0, (40,), dt))(keys, lows)
        assert tuple(out.shape) == (3, 40)
        for i in range(3):
            want = jr.random_truncated_normal(keys[i], torch.full((40,), float(lows[i])), 2.0,
                                              (40,), dt)
            assert np.array_equal(to_np(out)[i], to_np(want)), (dt, i)
    out = jr.vmap(lambda lo: jr.random_truncated_normal(jr.random_key(4), lo, 1.0, (8,)))(lows)
    for i in range(3):
        want = jr.random_truncated_normal(jr.random_key(4), torch.full((8,), float(lows[i])), 1.0,
                                          (8,))
        assert np.array_equal(to_np(out)[i], to_np(want))
    mins = torch.tensor([0, -50, 7], dtype=torch.int32)
    maxs = torch.tensor([10, 50, 1000], dtype=torch.int32)
    kraw = np.stack([oracle.split(oracle.seed(21), 3, True)[i] for i in range(3)])
    out = jr.vmap(lambda k, a, b: jr.random_randint(k, (50,), a, b))(keys, mins, maxs)
    assert tuple(out.shape) == (3, 50) and out.dtype == torch.int32
    for i in range(3):
        want = jr.random_randint(keys[i], (50,), int(mins[i]), int(maxs[i]))
        assert np.array_equal(to_np(out)[i], to_np(want)), i
        assert np.array_equal(to_np(out)[i], oracle.randint(kraw[i], (50,), int(mins[i]),
                                                            int(maxs[i]), "int32")), i
    # per-lane array bounds broadcast along the shape; one key for every lane
    rows = torch.tensor([[0, 100], [5, 6]], dtype=torch.int32)
    out = jr.vmap(lambda m: jr.random_randint(jr.random_key(9), (3, 2), m, 200))(rows)
    for i in range(2):
        want = jr.random_randint(jr.random_key(9), (3, 2), rows[i], 200)
        assert np.array_equal(to_np(out)[i], to_np(want)), i
