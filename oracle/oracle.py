"""ctypes binding of the CPU oracle (oracle/jxr_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the CPU
baseline leg of bench.py, as the checker.  The product package (jaxr_b200) never
imports it.  Build with `make -C oracle`.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F64, F16, BF16 = 0, 1, 2, 3
DTYPE_CODE = {"float32": F32, "float64": F64, "float16": F16, "bfloat16": BF16}
NP_FLOAT = {F32: np.float32, F64: np.float64, F16: np.uint16, BF16: np.uint16}
NP_BITS = {8: np.uint8, 16: np.uint16, 32: np.uint32, 64: np.uint64}

_lib = None


def build():
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        vp = ctypes.c_void_p
        u64, i64, i32, dbl = ctypes.c_uint64, ctypes.c_int64, ctypes.c_int, ctypes.c_double
        L.orc_threefry2x32.argtypes = [ctypes.c_uint32] * 4 + [u32p]
        L.orc_threefry_2x32.argtypes = [u32p, u32p, i64, u32p]
        L.orc_seed.argtypes = [i64, i32, u32p]
        L.orc_split.argtypes = [u32p, i64, i32, u32p]
        L.orc_fold_in.argtypes = [u32p, ctypes.c_uint32, u32p]
        L.orc_bits_at.argtypes = [u32p, i32, u64, i32, u64]
        L.orc_bits_at.restype = u64
        L.orc_random_bits.argtypes = [u32p, i32, u64, i32, u64, u64, vp]
        L.orc_erfinv_f32.argtypes = [ctypes.c_float, i32]
        L.orc_erfinv_f32.restype = ctypes.c_float
        L.orc_erfinv_f64.argtypes = [dbl, i32]
        L.orc_erfinv_f64.restype = dbl
        L.orc_erfinv_arr.argtypes = [vp, i64, i32, i32, vp]
        L.orc_log1p_neg.argtypes = [dbl]
        L.orc_log1p_neg.restype = dbl
        L.orc_uniform.argtypes = [u32p, i32, u64, i32, dbl, dbl, i32, u64, u64, vp]
        L.orc_normal.argtypes = [u32p, i32, u64, i32, i32, u64, u64, vp]
        L.orc_bernoulli.argtypes = [u32p, i32, dbl, u64, i32, u64, u64, vp]
        L.orc_uniform_at.argtypes = [u32p, i32, u64, i32, dbl, dbl, i32, u64]
        L.orc_uniform_at.restype = dbl
        L.orc_normal_at.argtypes = [u32p, i32, u64, i32, i32, u64]
        L.orc_normal_at.restype = dbl
        L.orc_log_pos.argtypes = [dbl]
        L.orc_log_pos.restype = dbl
        L.orc_sample_f32_from_bits.argtypes = [vp, i64, i32, vp]
        L.orc_sample.argtypes = [u32p, i32, i32, u64, i32, u64, u64, vp]
        L.orc_sample_at.argtypes = [u32p, i32, i32, u64, i32, u64]
        L.orc_sample_at.restype = dbl
        L.orc_gumbel_mode.argtypes = [u32p, i32, i32, u64, i32, vp]
        L.orc_truncated_normal.argtypes = [u32p, i32, u64, i32, dbl, dbl, i32, u64, u64, vp]
        L.orc_philox4x32.argtypes = [u32p, u32p, u32p]
        L.orc_rbg_bits.argtypes = [u32p, i32, u64, u64, u64, vp]
        L.orc_rbg_unsafe_split.argtypes = [u32p, i64, u32p]
        L.orc_rbg_unsafe_fold_in.argtypes = [u32p, ctypes.c_uint32, u32p]
        L.orc_set_threads.argtypes = [i32]
        L.orc_get_threads.restype = i32
        _lib = L
    return _lib


def _key(key):
    k = (ctypes.c_uint32 * 2)(int(key[0]) & 0xFFFFFFFF, int(key[1]) & 0xFFFFFFFF)
    return k


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def threefry2x32(k0, k1, c0, c1):
    out = (ctypes.c_uint32 * 2)()
    lib().orc_threefry2x32(k0, k1, c0, c1, out)
    return int(out[0]), int(out[1])


def threefry_2x32(key, count):
    count = np.ascontiguousarray(count, dtype=np.uint32)
    out = np.empty_like(count)
    lib().orc_threefry_2x32(_key(key), count.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                            count.size, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return out


def seed(s, x64=False):
    out = (ctypes.c_uint32 * 2)()
    lib().orc_seed(int(s), int(bool(x64)), out)
    return np.array([out[0], out[1]], dtype=np.uint32)


def split(key, num, partitionable=True):
    out = np.empty((int(num), 2), dtype=np.uint32)
    lib().orc_split(_key(key), int(num), int(bool(partitionable)),
                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return out


def fold_in(key, data):
    out = (ctypes.c_uint32 * 2)()
    lib().orc_fold_in(_key(key), int(data) & 0xFFFFFFFF, out)
    return np.array([out[0], out[1]], dtype=np.uint32)


def random_bits(key, bit_width, size, partitionable=True, begin=0, count=None):
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=NP_BITS[bit_width])
    rc = lib().orc_random_bits(_key(key), bit_width, int(size), int(bool(partitionable)),
                               int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_random_bits failed ({rc})")
    return out


def bits_at(key, bit_width, size, partitionable, idx):
    L = lib()
    k = _key(key)
    return np.array([L.orc_bits_at(k, bit_width, int(size), int(bool(partitionable)), int(i))
                     for i in idx], dtype=NP_BITS[bit_width])


ERFINV_ACCURATE = 2  # ORC_ERFINV_ACCURATE: jax_accurate_erf_inv's erf_inv


def _erfinv_mode(fma, accurate):
    return int(bool(fma)) | (ERFINV_ACCURATE if accurate else 0)


def erfinv(x, dtype="float32", fma=True, accurate=False):
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32 if dtype == "float32" else np.float64))
    out = np.empty_like(a)
    lib().orc_erfinv_arr(_ptr(a), a.size, F32 if dtype == "float32" else F64,
                         _erfinv_mode(fma, accurate), _ptr(out))
    return out.ravel()


def uniform(key, dtype, size, partitionable=True, minval=0.0, maxval=1.0, fma=True, begin=0,
            count=None):
    code = DTYPE_CODE[dtype]
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=NP_FLOAT[code])
    rc = lib().orc_uniform(_key(key), code, int(size), int(bool(partitionable)), float(minval),
                           float(maxval), int(fma), int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_uniform failed ({rc})")
    return out


def normal(key, dtype, size, partitionable=True, fma=True, begin=0, count=None, accurate=False):
    code = DTYPE_CODE[dtype]
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=NP_FLOAT[code])
    rc = lib().orc_normal(_key(key), code, int(size), int(bool(partitionable)),
                          _erfinv_mode(fma, accurate), int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_normal failed ({rc})")
    return out


def complex_normal(key, dtype, size, partitionable=True, accurate=False):
    """Complex normals (R/random.R:489-499): the key split in two, a real normal of the
    component dtype from each half (real part from the first), each divided by sqrt(2)
    rounded to the component dtype.  XLA divides (re + i im) by (sqrt2 + 0i) with Smith's
    method, whose ratio 0 / sqrt2 = 0 leaves re / sqrt2 and im / sqrt2."""
    real = {"complex64": "float32", "complex128": "float64"}[dtype]
    rdt = np.float32 if real == "float32" else np.float64
    ks = split(key, 2, partitionable)
    s2 = rdt(np.sqrt(2.0))
    re = (normal(ks[0], real, size, partitionable, accurate=accurate) / s2).astype(rdt)
    im = (normal(ks[1], real, size, partitionable, accurate=accurate) / s2).astype(rdt)
    out = np.empty(int(size), dtype=np.complex64 if real == "float32" else np.complex128)
    out.real = re
    out.imag = im
    return out


def bernoulli(key, p_dtype, p, size, partitionable=True, begin=0, count=None):
    code = DTYPE_CODE[p_dtype]
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=np.uint8)
    rc = lib().orc_bernoulli(_key(key), code, float(p), int(size), int(bool(partitionable)),
                             int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_bernoulli failed ({rc})")
    return out


def uniform_at(key, dtype, size, partitionable, minval, maxval, fma, idx):
    L = lib()
    k = _key(key)
    code = DTYPE_CODE[dtype]
    return np.array([L.orc_uniform_at(k, code, int(size), int(bool(partitionable)),
                                      float(minval), float(maxval), int(fma), int(i))
                     for i in idx])


def normal_at(key, dtype, size, partitionable, fma, idx):
    L = lib()
    k = _key(key)
    code = DTYPE_CODE[dtype]
    return np.array([L.orc_normal_at(k, code, int(size), int(bool(partitionable)), int(fma),
                                     int(i)) for i in idx])


SAMPLE_KIND = {"exponential": 0, "gumbel": 1, "logistic": 2, "laplace": 3}


def sample_f32_from_bits(bits, kind):
    """float32 samples of given uint32 draws: kind "exponential" / "gumbel" / "logistic" /
    "laplace" (mode "low" gumbel), or "normal" (fused Horner steps)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint32)
    out = np.empty(bits.shape[0], dtype=np.float32)
    code = 4 if kind == "normal" else SAMPLE_KIND[kind]
    lib().orc_sample_f32_from_bits(_ptr(bits), bits.shape[0], code, _ptr(out))
    return out


def sample(key, kind, dtype, size, partitionable=True, begin=0, count=None):
    """exponential / gumbel (mode "low") / logistic / laplace samples (R/random.R:1422-1516);
    16-bit dtypes as raw uint16 bits."""
    code = DTYPE_CODE[dtype]
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=NP_FLOAT[code])
    rc = lib().orc_sample(_key(key), SAMPLE_KIND[kind], code, int(size),
                          int(bool(partitionable)), int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_sample failed ({rc})")
    return out


def sample_at(key, kind, dtype, size, partitionable, idx):
    L = lib()
    k = _key(key)
    return np.array([L.orc_sample_at(k, SAMPLE_KIND[kind], DTYPE_CODE[dtype], int(size),
                                     int(bool(partitionable)), int(i)) for i in idx])


def gumbel_mode(key, mode, dtype, size, partitionable=True):
    """random_gumbel(key, (size), dtype, mode) for mode "high" or "highest"."""
    code = DTYPE_CODE[dtype]
    out = np.empty(int(size), dtype=NP_FLOAT[code])
    rc = lib().orc_gumbel_mode(_key(key), {"high": 0, "highest": 1}[mode], code, int(size),
                               int(bool(partitionable)), _ptr(out))
    if rc:
        raise ValueError(f"orc_gumbel_mode failed ({rc})")
    return out


def truncated_normal(key, dtype, size, lower, upper, partitionable=True, begin=0, count=None,
                     accurate=False):
    code = DTYPE_CODE[dtype]
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=NP_FLOAT[code])
    rc = lib().orc_truncated_normal(_key(key), code, int(size), int(bool(partitionable)),
                                    float(lower), float(upper), _erfinv_mode(True, accurate),
                                    int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_truncated_normal failed ({rc})")
    return out


INT_INFO = {"int8": (8, True), "int16": (16, True), "int32": (32, True), "int64": (64, True),
            "uint8": (8, False), "uint16": (16, False), "uint32": (32, False),
            "uint64": (64, False)}


def _int_range(bits, signed):
    return (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if signed else (0, (1 << bits) - 1)


def _wrap(v, bits, signed):
    v &= (1 << bits) - 1
    return v - (1 << bits) if signed and v >> (bits - 1) else v


def randint(key, shape, minval, maxval, dtype, partitionable=True):
    """random_randint (R/random.R:308-359) for integer bounds, restated with exact Python
    integers: minval/maxval are ints or integer arrays broadcastable to `shape`, already
    in the bounds' dtype (values as given).  Returns a flat numpy array of `dtype`.

    dtypes narrower than 32 bits sample in int32 with the bounds wrapped to int32 and
    clipped to [min, max] and [min, max + 1] (:320-325); the sampling dtype's bounds are
    clipped to its range, maxval beyond its maximum widens the span by one (:338-350); the
    offset is ((hi % span) * (2^nbits % span) + lo % span) % span in nbits-bit unsigned
    arithmetic with XLA's x % 0 = x (:351-358), hi and lo the nbits-bit draws of the two
    halves of split(key)."""
    dbits, dsigned = INT_INFO[dtype]
    size = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    mn = [int(v) for v in np.broadcast_to(np.asarray(minval, dtype=object), shape).ravel()]
    mx = [int(v) for v in np.broadcast_to(np.asarray(maxval, dtype=object), shape).ravel()]
    if dbits < 32:
        lo_d, hi_d = _int_range(dbits, dsigned)
        mn = [min(max(_wrap(v, 32, True), lo_d), hi_d) for v in mn]
        mx = [min(max(_wrap(v, 32, True), lo_d), hi_d + 1) for v in mx]
        sbits, ssigned = 32, True
    else:
        sbits, ssigned = dbits, dsigned
    smin, smax = _int_range(sbits, ssigned)
    oor = [v > smax for v in mx]
    mn = [min(max(v, smin), smax) for v in mn]
    mx = [min(max(v, smin), smax) for v in mx]
    M = 1 << sbits
    ks = split(key, 2, partitionable)
    hi = random_bits(ks[0], sbits, size, partitionable)
    lo = random_bits(ks[1], sbits, size, partitionable)

    def xrem(a, b):
        return a if b == 0 else a % b

    out = []
    for i in range(size):
        span = (mx[i] - mn[i]) % M
        if mx[i] <= mn[i]:
            span = 1
        elif oor[i]:
            span = (span + 1) % M
        mult = xrem((1 << (sbits // 2)) % M, span)
        mult = xrem(mult * mult % M, span)
        off = xrem((xrem(int(hi[i]), span) * mult % M + xrem(int(lo[i]), span)) % M, span)
        r = _wrap(mn[i] + off, sbits, ssigned)
        out.append(_wrap(r, dbits, dsigned))
    return np.array(out, dtype=np.dtype(dtype))


def shuffle(key, outer, n, inner, partitionable=True):
    """rnd_shuffle (R/random.R:402-413) over an (outer, n, inner) array, shuffling each 1-D
    slice along the middle axis: returns cur with cur[f] = the flat source index of the
    element at flat position f.  Each of ceil(3 log(max(1, size)) / log(2^32 - 1)) rounds
    splits the key (ks[0] carries on), draws 32-bit keys from ks[1] over the whole array and
    sorts every slice stably by them (lax_sort_key_val is stable)."""
    import math
    total = outer * n * inner
    rounds = int(math.ceil(3 * math.log(max(1, total)) / math.log(2 ** 32 - 1)))
    cur = np.arange(total, dtype=np.int64)
    for _ in range(rounds):
        ks = split(key, 2, partitionable)
        key = ks[0]
        sk = random_bits(ks[1], 32, total, partitionable).reshape(outer, n, inner)
        order = np.argsort(sk, axis=1, kind="stable")
        cur = np.take_along_axis(cur.reshape(outer, n, inner), order, axis=1).ravel()
    return cur


def shuffle_rbg_lanes(key, impl, nlanes, outer, n, inner, partitionable=True):
    """rnd_shuffle (R/random.R:402-413) under vmap over nlanes rbg or unsafe_rbg keys, key
    being the first lane's u32[4] key.  rng_bit_generator's batching rule (R/prng.R:300-313)
    draws every lane's bits from the first lane's key, lane i taking row i of one
    (nlanes, shape) request; the first lane's split is its own (an rbg key splits its halves
    per lane; lane 0's rows of a batched unsafe_rbg split are rows 0 and 10 of its own
    request).  Returns cur of shape (nlanes, total): per lane, the flat source index of the
    element at each flat position, as shuffle() gives for one key."""
    import math
    total = outer * n * inner
    rounds = int(math.ceil(3 * math.log(max(1, total)) / math.log(2 ** 32 - 1)))
    cur = np.tile(np.arange(total, dtype=np.int64), (nlanes, 1))
    key = np.asarray(key, dtype=np.uint32)
    for _ in range(rounds):
        ks = rbg_split(key, 2, partitionable) if impl == "rbg" else rbg_unsafe_split(key, 2)
        key = ks[0]
        sk = rbg_bits(ks[1], 32, nlanes * total).reshape(nlanes, outer, n, inner)
        for i in range(nlanes):
            order = np.argsort(sk[i], axis=1, kind="stable")
            cur[i] = np.take_along_axis(cur[i].reshape(outer, n, inner), order, axis=1).ravel()
    return cur


def permutation(key, x, axis=0, independent=False, partitionable=True):
    """random_permutation (R/random.R:378-400): an integer x permutes arange(x) (int32); an
    array is shuffled along `axis`, slices independently or (the default) all by one
    shuffled index vector."""
    if np.ndim(x) == 0:
        n = int(x)
        return np.arange(max(n, 0), dtype=np.int32)[shuffle(key, 1, max(n, 0), 1, partitionable)]
    x = np.asarray(x)
    axis = axis + x.ndim if axis < 0 else axis
    outer = int(np.prod(x.shape[:axis], dtype=np.int64))
    n = x.shape[axis]
    inner = int(np.prod(x.shape[axis + 1:], dtype=np.int64))
    if independent or x.ndim == 1:
        return x.ravel()[shuffle(key, outer, n, inner, partitionable)].reshape(x.shape)
    ind = shuffle(key, 1, n, 1, partitionable)
    return np.take(x, ind, axis=axis)


def choice(key, a, shape=(), replace=True, p=None, axis=0, partitionable=True, x64=False):
    """random_choice (R/random.R:417-464) for p = None, and for p with replace = True
    (cumulative sum, r = total * (1 - u), searchsorted left)."""
    shape = tuple(shape)
    scalar = np.ndim(a) == 0
    arr = None if scalar else np.asarray(a)
    n_inputs = int(a) if scalar else arr.shape[axis]
    n_draws = int(np.prod(shape, dtype=np.int64)) if shape else 1
    dint = "int64" if x64 else "int32"
    if p is None:
        if replace:
            ind = randint(key, shape, 0, n_inputs, dint, partitionable).reshape(shape)
            return ind if scalar else np.take(arr, ind, axis=axis)
        perm = permutation(key, n_inputs if scalar else arr, axis, False, partitionable)
        ind_axis = 0 if scalar else axis
        return np.take(perm, np.arange(n_draws), axis=ind_axis).reshape(
            shape if scalar else arr.shape[:axis] + shape + arr.shape[axis + 1:])
    fdt = "float64" if x64 else "float32"
    pa = np.asarray(p, dtype=fdt)
    cuml = np.cumsum(pa, dtype=fdt)
    u = uniform(key, fdt, n_draws, partitionable).astype(fdt)
    r = (cuml[-1] * (np.asarray(1, dtype=fdt) - u).astype(fdt)).astype(fdt)
    ind = np.searchsorted(cuml, r, side="left").astype(dint).reshape(shape)
    return ind if scalar else np.take(arr, ind, axis=axis)


def _key4(q):
    return (ctypes.c_uint32 * 4)(*[int(v) & 0xFFFFFFFF for v in q])


def philox4x32(counter, key):
    out = (ctypes.c_uint32 * 4)()
    lib().orc_philox4x32((ctypes.c_uint32 * 4)(*counter), (ctypes.c_uint32 * 2)(*key), out)
    return [int(v) for v in out]


def rbg_seed(seed, x64=False):
    """rbg / unsafe_rbg seed (R/prng.R:385-388): the threefry seed twice."""
    return np.concatenate([seed_key := globals()["seed"](seed, x64), seed_key])


def rbg_bits(q, bit_width, size, begin=0, count=None):
    """lax_rng_bit_generator(q, (size), uint<bit_width>)[[2]] elements [begin, +count)."""
    count = size - begin if count is None else count
    out = np.empty(int(count), dtype=NP_BITS[bit_width])
    rc = lib().orc_rbg_bits(_key4(q), bit_width, int(size), int(begin), int(count), _ptr(out))
    if rc:
        raise ValueError(f"orc_rbg_bits failed ({rc})")
    return out


def rbg_split(q, num, partitionable=True):
    """rbg split (R/prng.R:391-397): each half of the key split as a threefry key; key j is
    (half 0's key j, half 1's key j)."""
    h0 = split(q[:2], num, partitionable)
    h1 = split(q[2:], num, partitionable)
    return np.concatenate([h0, h1], axis=1)


def rbg_fold_in(q, data):
    return np.concatenate([fold_in(q[:2], data), fold_in(q[2:], data)])


def rbg_unsafe_split(q, num):
    out = np.empty((int(num), 4), dtype=np.uint32)
    lib().orc_rbg_unsafe_split(_key4(q), int(num), out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return out


def rbg_unsafe_fold_in(q, data):
    out = (ctypes.c_uint32 * 4)()
    lib().orc_rbg_unsafe_fold_in(_key4(q), int(data) & 0xFFFFFFFF, out)
    return np.array(list(out), dtype=np.uint32)


def set_threads(n):
    lib().orc_set_threads(int(n))


def get_threads():
    return int(lib().orc_get_threads())
