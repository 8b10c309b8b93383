"""Host-side behaviour of the public API that needs no GPU: argument checks and error
messages/classes (tests/testthat/test-prng.R:260-279, test-random.R:382-407), dtype
canonicalisation, seeds and shard ranges."""

import numpy as np
import pytest
import torch

import jaxr_b200 as jr
from jaxr_b200 import random as jrr
from jaxr_b200.shard import shard_range

U32 = torch.uint32


def raw(*shape):
    return torch.zeros(shape, dtype=U32)


def test_key_errors_follow_reference():
    # test-prng.R:263-279
    with pytest.raises(jr.JaxValueError, match=r"split accepts a single key, but was given a key "
                                               r"array of shape \(2, 2\)"):
        jr.random_split(raw(2, 2))
    with pytest.raises(jr.JaxValueError, match="uniform accepts a single key"):
        jr.random_uniform(jr.PRNGKeyArray(raw(2, 2)))
    with pytest.raises(jr.JaxTypeError, match="expected key_data.dtype = uint32; got dtype=float32"):
        jr.random_split(np.array([0.0, 0.0]))
    with pytest.raises(jr.JaxTypeError, match=r"expected key_data.shape to end with \(2,\)"):
        jr.random_split(raw(3))
    with pytest.raises(jr.JaxTypeError, match="expected key_data.ndim >= 1"):
        jr.random_split(torch.zeros((), dtype=U32))
    with pytest.raises(jr.JaxTypeError, match="unexpected PRNG key type"):
        jr.random_split("a")
    with pytest.raises(jr.JaxTypeError, match=r"key accepts a scalar seed, but was given an array "
                                              r"of shape \(2,\)"):
        jr.random_key([1, 2])
    with pytest.raises(jr.JaxTypeError, match="accepts a scalar seed, but was given a PRNG key"):
        jr.random_PRNGKey(jr.PRNGKeyArray(raw(2)))
    with pytest.raises(jr.JaxTypeError, match="PRNG key seed must be an integer"):
        jr.random_key(0.5)
    with pytest.raises(jr.JaxValueError, match="Cannot specify both"):
        jr.random_key(0, impl="rbg", dtype="rbg")
    with pytest.raises(jr.JaxTypeError, match="fold_in accepts a scalar"):
        jr.random_fold_in(raw(2), np.array([1, 2]))
    with pytest.raises(jr.JaxOverflowError, match="out of bounds for uint32"):
        jr.random_fold_in(raw(2), -1)
    with pytest.raises(jr.JaxValueError, match="must be an unsigned int dtype"):
        jr.random_bits(raw(2), 3, "int32")
    with pytest.raises(jr.JaxTypeError, match="iteration over a 0-d key array"):
        list(jr.PRNGKeyArray(raw(2)))
    with pytest.raises(jr.JaxValueError, match="unrecognized PRNG implementation"):
        jr.random_key(0, impl="philox")


def test_sampler_argument_errors():
    # test-random.R:385-390
    k = raw(2)
    with pytest.raises(jr.JaxValueError, match="dtype argument to `uniform` must be a float dtype"):
        jr.random_uniform(k, 3, dtype="int32")
    with pytest.raises(jr.JaxValueError, match="must be a float or complex dtype"):
        jr.random_normal(k, 3, dtype="int32")
    with pytest.raises(jr.JaxTypeError, match="bernoulli probability `p` must have a floating dtype"):
        jr.random_bernoulli(k, 1)
    with pytest.raises(jr.JaxValueError, match="expected 'high' or 'low'"):
        jr.random_bernoulli(k, 0.5, mode="mid")
    with pytest.raises(jr.JaxTypeError, match="Shapes must be 1D sequences"):
        jr.random_normal(k, -1)


def test_errors_are_builtin_classes_too():
    with pytest.raises(ValueError):
        jr.random_bits(raw(2), 3, "int32")
    with pytest.raises(TypeError):
        jr.random_key(0.5)
    with pytest.raises(OverflowError):
        jr.random_fold_in(raw(2), 2 ** 32)


def test_dtype_canonicalisation():
    assert jr.canonicalize_dtype("uint64") == "uint32"
    assert jr.canonicalize_dtype("float") == "float32"
    with jr.with_jax_config("jax_enable_x64", True):
        assert jr.canonicalize_dtype("uint64") == "uint64"
        assert jr.canonicalize_dtype("float") == "float64"
        assert jrr.default_uint() == "uint64"
    assert jr.random_key_dtype() == "key<fry>"
    assert jr.random_key_dtype("rbg") == "key<rbg>"


def test_seed_words_match_reference_keys():
    # test-prng.R:27-30 and :118-119
    def words(s, x64):
        with jr.with_jax_config("jax_enable_x64", x64):
            k0, k1 = jrr._seed_words(s)
        return [int(k0), int(k1)]
    assert words(0, False) == [0, 0]
    assert words(42, False) == [0, 42]
    assert words(-1, False) == [0, 4294967295]
    assert words(2 ** 40 + 5, False) == [0, 5]
    assert words(-1, True) == [4294967295, 4294967295]
    assert words(2 ** 40 + 5, True) == [256, 5]
    # integer arrays keep their width: a 32-bit seed has k0 = 0 even with x64
    with jr.with_jax_config("jax_enable_x64", True):
        k0, k1 = jrr._seed_words(torch.tensor([-1, 3], dtype=torch.int32))
    assert k0.tolist() == [0, 0] and k1.tolist() == [4294967295, 3]
    with jr.with_jax_config("jax_random_seed_offset", 10):
        assert words(0, False) == [0, 10]


def test_shard_ranges_cover_the_request():
    size = (1 << 34) + 3
    for world in (1, 2, 3, 4, 8):
        spans = [shard_range(size, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == size
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        lens = [b - a for a, b in spans]
        assert max(lens) - min(lens) <= 1


def test_config_flags():
    assert jr.jax_config("jax_threefry_partitionable") is True
    with jr.with_jax_config("jax_threefry_partitionable", False):
        assert jrr._layout() == 0
    assert jrr._layout() == 1
    old = jr.enable_x64(True)
    try:
        assert jr.jax_config("jax_enable_x64") is True
    finally:
        jr.enable_x64(old)
    with pytest.raises(jr.JaxValueError):
        jr.jax_config_update("no_such_option", 1)


def test_vmap_argument_checks():
    with pytest.raises(jr.JaxValueError, match="inconsistent sizes"):
        jr.vmap(lambda a, b: a)(raw(3, 2), raw(4, 2))
    with pytest.raises(jr.JaxValueError, match="rank should be at least 1"):
        jr.vmap(lambda a: a)(torch.tensor(1))


def test_key_array_surface():
    k = jr.PRNGKeyArray(torch.arange(12, dtype=torch.int64).to(U32).reshape(3, 2, 2))
    assert k.shape == (3, 2) and k.ndim == 2 and len(k) == 3
    assert k[1].shape == (2,) and k[1, 0].data.tolist() == [4, 5]
    assert [x.shape for x in k] == [(2,), (2,), (2,)]
    assert "dtype=key<fry>" in repr(k)
    assert jr.random_key_impl(k) == "threefry2x32"
    assert jr.random_key_data(k) is k.data
    assert jr.random_Key(k) is k


def test_derived_sampler_argument_errors():
    # test-random.R:387, :393; R/random.R:1438-1444, :46-53
    k = raw(2)
    with pytest.raises(jr.JaxTypeError, match="randint only accepts integer dtypes, got float32"):
        jr.random_randint(k, 3, 0, 5, dtype="float32")
    with pytest.raises(jr.JaxValueError, match="Must provide valid mode for gumbel got: medium"):
        jr.random_gumbel(k, 2, mode="medium")
    for fn, name in ((jr.random_exponential, "exponential"), (jr.random_laplace, "laplace"),
                     (jr.random_logistic, "logistic"), (jr.random_gumbel, "gumbel")):
        with pytest.raises(jr.JaxValueError,
                           match=f"dtype argument to `{name}` must be a float dtype, got int32"):
            fn(k, 3, dtype="int32")
    with pytest.raises(jr.JaxValueError, match="dtype argument to `truncated_normal` must be a "
                                               "float dtype, got int32"):
        jr.random_truncated_normal(k, -1, 1, 3, dtype="int32")
    with pytest.raises(jr.JaxValueError, match=r"randint parameter shapes must be "
                                               r"broadcast-compatible with shape argument.*"
                                               r"for shape argument \(2,\)"):
        jr.random_randint(k, 2, np.array([0, 1, 2], dtype=np.int32), 5)
    with pytest.raises(jr.JaxValueError, match="split accepts a single key|randint accepts a "
                                               "single key"):
        jr.random_randint(raw(2, 2), 3, 0, 5)
    with pytest.raises(jr.JaxOverflowError, match="too large to convert to int32"):
        jr.random_randint(k, 3, 0, 1 << 40)


def test_randint_bounds_follow_reference(monkeypatch):
    """The bounds that reach the combine kernel (R/random.R:313-350): dtypes narrower than
    32 bits sample in int32 with maxval clipped to max + 1; a maxval above the sampling
    dtype's maximum flags the span to grow by one; whole floats are ints, other floats
    truncate."""
    calls = []

    def fake_call(name, *args):
        calls.append((name, args))

    monkeypatch.setattr(jrr, "_flat_keys", lambda k: k.data.reshape(-1, 2))
    monkeypatch.setattr(jrr, "_k_split", lambda kd, shape, layout, impl=None: torch.zeros(
        (kd.shape[0], 2, 2), dtype=U32))
    monkeypatch.setattr(jrr, "_k_bits", lambda kd, size, bw, layout: torch.zeros(
        (kd.shape[0], size), dtype=jrr._TORCH[f"uint{bw}"]))
    monkeypatch.setattr(jrr.nat, "call", fake_call)
    monkeypatch.setattr(jrr, "_ptr", lambda t: t)
    monkeypatch.setattr(jrr, "_stream", lambda: None)

    def bounds(*args, **kw):
        calls.clear()
        jr.random_randint(raw(2), *args, **kw)
        (name, a), = calls
        if name == "jxr_randint":  # scalar bounds, one fused kernel
            return (a[6], a[7], [a[8]], [a[9]], [a[10]], a[11])
        assert name == "jxr_randint_combine"
        return (a[3], a[4], a[5].tolist(), a[7].tolist(), a[9].tolist(), a[11])

    # nbits, signed, minval, maxval, out_of_range, out_bits
    assert bounds(6, 0, 256, "uint8") == (32, 1, [0], [256], [0], 8)
    assert bounds(6, -1000, 1000, "int8") == (32, 1, [-128], [128], [0], 8)
    assert bounds(6, 0, 10) == (32, 1, [0], [10], [0], 32)
    assert bounds(6, 0.0, 7.9) == (32, 1, [0], [7], [0], 32)  # 7.9 truncates
    with jr.with_jax_config("jax_threefry_partitionable", False):  # the three-kernel path
        assert bounds(6, -1000, 1000, "int8") == (32, 1, [-128], [128], [0], 8)
    with jr.with_jax_config("jax_enable_x64", True):
        assert bounds(6, 0, 1 << 40, "int32") == (32, 1, [0], [2**31 - 1], [1], 32)
        assert bounds(6, -5, 1 << 33, "uint32") == (32, 0, [0], [2**32 - 1], [1], 32)
        assert bounds(6, 0, 10, "uint64") == (64, 0, [0], [10], [0], 64)


def test_accurate_erf_inv_option_selects_the_library_variant(monkeypatch):
    """jax_accurate_erf_inv reaches the library as its per-thread erf_inv setting for the
    duration of each sampler call, and the previous setting comes back afterwards (no GPU
    call here: the sampler body is a stub that records the setting it sees)."""
    from jaxr_b200 import _native as nat
    lib = nat.lib()
    seen = []
    f = jrr._uses_erf_inv(lambda: seen.append(lib.jxr_get_accurate_erf_inv()))
    with jr.with_jax_config("jax_accurate_erf_inv", True):
        f()
    f()
    assert seen == [1, 0] and lib.jxr_get_accurate_erf_inv() == 0
    lib.jxr_set_accurate_erf_inv(1)
    f()
    assert seen[-1] == 0 and lib.jxr_get_accurate_erf_inv() == 1
    assert lib.jxr_set_accurate_erf_inv(7) == 1 and lib.jxr_set_accurate_erf_inv(0) == 1
    for fn in (jr.random_normal, jr.random_normal_bernoulli, jr.random_truncated_normal,
               jr.lax_erf_inv):
        assert getattr(fn, "__wrapped__", None) is not None, fn.__name__
    assert jr.jax_config("jax_accurate_erf_inv") is False
