"""rbg and unsafe_rbg keys (R/prng.R:264-426) on the GPU: the Philox4x32-10 stream of XLA's
RngBitGenerator against the oracle, exact for every width, range and counter carry, the
key operations, the samplers drawing from it, and lax_rng_bit_generator."""

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


def rbg_key(q, impl="rbg"):
    return jr.random_wrap_key_data(torch.tensor(np.asarray(q, dtype=np.uint32)).cuda(), impl=impl)


KEYS = [[0, 0, 0, 0], [0, 3, 0, 3], [0xDEADBEEF, 0x12345678, 0x9ABCDEF0, 0x0F0F0F0F],
        [0xFFFFFFF0, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF]]  # the last carries through 128 bits


@pytest.mark.parametrize("bw", [8, 16, 32, 64])
def test_rbg_bits_exact(bw):
    for q in KEYS:
        for n in (0, 1, 3, 4, 5, 7, 16, 17, 1000, 65537, 1 << 20):
            with flags(bw == 64):
                got = to_np(jr.random_bits(rbg_key(q), (n,), f"uint{bw}"))
            assert np.array_equal(got, orc.rbg_bits(q, bw, n)), (q, n)


@pytest.mark.parametrize("bw", [8, 16, 32, 64])
def test_rbg_bits_ranges(bw):
    """Element ranges (the shard entry), unaligned starts and ends included."""
    from jaxr_b200 import _native as nat
    q = KEYS[2]
    k = torch.tensor(np.asarray(q, dtype=np.uint32)).cuda()
    size = 100003
    for lo, n in ((0, size), (1, 17), (3, 1000), (5, 65536), (size - 9, 9), (77, 0)):
        out = torch.empty(n, dtype={8: torch.uint8, 16: torch.uint16, 32: torch.uint32,
                                    64: torch.uint64}[bw], device="cuda")
        nat.call("jxr_rbg_bits", k.data_ptr(), size, lo, n, bw, out.data_ptr() if n else None,
                 None, torch.cuda.current_stream().cuda_stream)
        assert np.array_equal(to_np(out), orc.rbg_bits(q, bw, size, lo, n)), (lo, n)


def test_rbg_key_operations():
    for part in (True, False):
        for impl in ("rbg", "unsafe_rbg"):
            for q in KEYS:
                k = rbg_key(q, impl)
                with flags(False, part):
                    sp = to_np(jr.random_key_data(jr.random_split(k, 5)))
                    fo = to_np(jr.random_key_data(jr.random_fold_in(k, 123456789)))
                if impl == "rbg":
                    want_sp = orc.rbg_split(q, 5, part)
                    want_fo = orc.rbg_fold_in(q, 123456789)
                else:
                    want_sp = orc.rbg_unsafe_split(q, 5)
                    want_fo = orc.rbg_unsafe_fold_in(q, 123456789)
                assert np.array_equal(sp, want_sp), (impl, q, part)
                assert np.array_equal(fo, want_fo), (impl, q)


def test_rbg_vmap_draws_from_first_key():
    keys = jr.random_split(jr.random_key(0, impl="rbg"), 3)
    data = to_np(jr.random_key_data(keys))
    out = to_np(jr.vmap(lambda k: jr.random_bits(k, (5,)))(keys))
    assert np.array_equal(out.ravel(), orc.rbg_bits(data[0], 32, 15))
    # split and fold_in under vmap act per key (threefry on each half)
    sp = to_np(jr.random_key_data(jr.vmap(lambda k: jr.random_split(k, 2))(keys)))
    for r in range(3):
        assert np.array_equal(sp[r], orc.rbg_split(data[r], 2))


def _unit_f32(bits):
    return ((bits >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1)


def test_rbg_samplers():
    q = KEYS[2]
    k = rbg_key(q)
    n = 4097
    bits = orc.rbg_bits(q, 32, n)
    u = to_np(jr.random_uniform(k, (n,)))
    assert np.array_equal(u.view(np.uint32), _unit_f32(bits).view(np.uint32))
    # normal: sqrt(2) erf_inv(max(lo, 2 f + lo)) of the same bits, lo = -1 + 2^-24
    lo = np.float32(-1 + 2.0 ** -24)
    f = _unit_f32(bits)
    uu = np.maximum(lo, (f.astype(np.float64) * 2 + lo).astype(np.float32))
    want = (np.float32(np.sqrt(2)) * orc.erfinv(uu, "float32")).astype(np.float32)
    got = to_np(jr.random_normal(k, (n,)))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    b = to_np(jr.random_bernoulli(k, 0.3, (n,)))
    assert np.array_equal(b, _unit_f32(bits) < np.float32(0.3))
    # samplers through split and bits: randint, permutation
    r = to_np(jr.random_randint(k, (n,), -7, 100))
    ks = orc.rbg_split(q, 2)
    hi = orc.rbg_bits(ks[0], 32, n).astype(np.int64)
    lo_ = orc.rbg_bits(ks[1], 32, n).astype(np.int64)
    span = 107
    mult = (1 << 32) % span
    off = ((hi % span) * mult + lo_ % span) % span
    assert np.array_equal(r, (off - 7).astype(np.int32))
    for impl in ("rbg", "unsafe_rbg"):
        kk = rbg_key(q, impl)
        perm = to_np(jr.random_permutation(kk, 3000))
        key = np.asarray(q, dtype=np.uint32)
        cur = np.arange(3000)
        for _ in range(2):  # 3000 elements: two rounds
            sp = orc.rbg_split(key, 2) if impl == "rbg" else orc.rbg_unsafe_split(key, 2)
            key = sp[0]
            sk = orc.rbg_bits(sp[1], 32, 3000)
            cur = cur[np.argsort(sk, kind="stable")]
        assert np.array_equal(perm, cur.astype(np.int32)), impl
    # the log-transform and truncated-normal samplers run their transforms on the bits
    e = to_np(jr.random_exponential(k, (n,)))
    assert np.all(np.isfinite(e)) and np.all(e >= 0)
    t = to_np(jr.random_truncated_normal(k, -1, 2, (n,)))
    assert np.all((t > -1) & (t < 2))


def test_lax_rng_bit_generator():
    key = torch.zeros(4, dtype=torch.uint32)
    new, bits = jr.lax_rng_bit_generator(key, (2, 3), dtype="uint16")
    assert new.dtype == torch.uint32 and tuple(new.shape) == (4,)
    assert bits.dtype == torch.uint16 and tuple(bits.shape) == (2, 3)
    assert np.array_equal(to_np(bits).ravel(), orc.rbg_bits([0, 0, 0, 0], 16, 6))
    # 6 16-bit values use 2 blocks: the counter advances by 2
    assert np.array_equal(to_np(new), [2, 0, 0, 0])
    _, b4 = jr.lax_rng_bit_generator(key, 4)
    assert np.array_equal(to_np(b4), [1713891541, 3781805453, 3159862348, 2600524760])
    k64 = torch.tensor([3 << 32 | 0, 3 << 32 | 0], dtype=torch.uint64)
    new64, b = jr.lax_rng_bit_generator(k64, 5, dtype="uint8")
    assert np.array_equal(to_np(b), [211, 175, 250, 104, 232])  # key (0, 3, 0, 3)
    assert new64.dtype == torch.uint64
    with pytest.raises(jr.JaxTypeError, match="rng_bit_generator: unsupported dtype int32"):
        jr.lax_rng_bit_generator(key, 3, dtype="int32")


def test_rbg_shards_cover_the_request():
    from jaxr_b200.shard import random_bits_shard
    k = rbg_key(KEYS[3])
    size = 100003
    slabs = [to_np(random_bits_shard(k, (size,), r, 3)) for r in range(3)]
    assert np.array_equal(np.concatenate(slabs), orc.rbg_bits(KEYS[3], 32, size))


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("kind", ["normal", "normal_accurate", "exponential", "gumbel",
                                  "logistic", "laplace"])
def test_from_bits_tables_match_direct(kind, dt):
    """The from-bits transforms (how rbg keys sample) read the sampler's table for 2^22 or
    more float32 draws and 2^16 or more 16-bit draws: the same draws transformed in one
    call (table) and in chunks below the threshold (evaluated directly) agree bit for bit."""
    from jaxr_b200 import _native as nat
    code = {"float32": nat.F32, "float16": nat.F16, "bfloat16": nat.BF16}[dt]
    bits_dt = {"float32": torch.int32, "float16": torch.int16, "bfloat16": torch.uint8}[dt]
    out_dt = torch.float32 if dt == "float32" else torch.int16
    n = (1 << 22) + 3 if dt == "float32" else (1 << 16) + 3
    chunk = (1 << 21) if dt == "float32" else (1 << 15)
    g = torch.Generator(device="cuda").manual_seed(5)
    bits = torch.randint(-2**31 if bits_dt != torch.uint8 else 0,
                         2**31 - 1 if bits_dt != torch.uint8 else 256, (n,),
                         generator=g, device="cuda", dtype=torch.int64).to(bits_dt)
    st = torch.cuda.current_stream().cuda_stream
    kinds = {"exponential": 0, "gumbel": 1, "logistic": 2, "laplace": 3}

    def transform(b, out):
        if kind.startswith("normal"):
            nat.call("jxr_normal_from_bits", b.data_ptr(), b.numel(), code, out.data_ptr(), st)
        else:
            nat.call("jxr_sample_from_bits", b.data_ptr(), b.numel(), kinds[kind], code,
                     out.data_ptr(), st)

    prev = nat.lib().jxr_set_accurate_erf_inv(1 if kind == "normal_accurate" else 0)
    try:
        whole = torch.empty(n, dtype=out_dt, device="cuda")
        transform(bits, whole)
        parts = torch.empty_like(whole)
        for s in range(0, n, chunk):
            transform(bits[s:s + chunk], parts[s:s + chunk])
        torch.cuda.synchronize()
    finally:
        nat.lib().jxr_set_accurate_erf_inv(prev)
    wi = whole.view(torch.int32 if dt == "float32" else torch.int16)
    pi = parts.view(torch.int32 if dt == "float32" else torch.int16)
    assert torch.equal(wi, pi)


@pytest.mark.parametrize("impl", ["rbg", "unsafe_rbg"])
def test_permutation_and_choice_under_vmap(impl):
    """random_permutation and random_choice under vmap over rbg / unsafe_rbg keys:
    rng_bit_generator's batching rule draws every lane's bits from the first lane's key,
    lane i taking row i of one batched request (R/prng.R:300-313).  Against the oracle's
    restatement of rnd_shuffle under that rule, and lane 0 against the unbatched call with
    the first key (row 0 of the batched request is the unbatched request)."""
    keys = jr.random_split(jr.random_key(5, impl=impl), 3)
    q0 = to_np(jr.random_key_data(keys))[0]
    n = 3000
    got = to_np(jr.vmap(lambda k: jr.random_permutation(k, n))(keys))
    want = orc.shuffle_rbg_lanes(q0, impl, 3, 1, n, 1)
    assert np.array_equal(got, want.astype(np.int32)), impl
    k0 = keys[0]
    assert np.array_equal(got[0], to_np(jr.random_permutation(k0, n)))
    # a shared array along axis 1: every lane takes its own index vector
    x = torch.arange(4 * 50, dtype=torch.int32).reshape(4, 50)
    got = to_np(jr.vmap(lambda k: jr.random_permutation(k, x, axis=1))(keys))
    ind = orc.shuffle_rbg_lanes(q0, impl, 3, 1, 50, 1)
    for i in range(3):
        assert np.array_equal(got[i], np.take(x.numpy(), ind[i], axis=1)), i
    # batched arrays, shuffled independently along axis 0
    xs = torch.arange(3 * 40 * 2, dtype=torch.int32).reshape(3, 40, 2)
    got = to_np(jr.vmap(lambda k, r: jr.random_permutation(k, r, independent=True))(keys, xs))
    ind = orc.shuffle_rbg_lanes(q0, impl, 3, 1, 40, 2)
    for i in range(3):
        assert np.array_equal(got[i].ravel(), xs[i].numpy().ravel()[ind[i]]), i
    # choice: without replacement the lanes' permutations' first draws; every branch's
    # lane 0 as the unbatched choice with the first key
    got = to_np(jr.vmap(lambda k: jr.random_choice(k, 100, (7,), False))(keys))
    want = orc.shuffle_rbg_lanes(q0, impl, 3, 1, 100, 1)[:, :7]
    assert np.array_equal(got, want.astype(np.int32))
    p = torch.tensor([0.1, 0.2, 0.3, 0.4])
    for replace in (True, False):
        for pp in (None, p):
            out = to_np(jr.vmap(lambda k: jr.random_choice(k, 4, (3,), replace, pp))(keys))
            assert out.shape == (3, 3)
            one = to_np(jr.random_choice(k0, 4, (3,), replace, pp))
            assert np.array_equal(out[0], one), (replace, pp is None)
