"""Golden-vector cases of the reference (tests/golden/threefry_golden.json) and the
comparison rules its tests use.

Each case names a call of the reference's API (seed, fold_in, split, bits, uniform,
normal, bernoulli, vmap over keys, erf_inv) with the expected values the reference
recorded.  `evaluate(case, backend)` replays the call through a backend: the CPU
oracle (oracle/oracle.py) or the product's host API (jaxr_b200).
"""

from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "threefry_golden.json")


def load_cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def _f(v):
    if isinstance(v, str):
        low = v.lower()
        if low in ("nan", "inf", "-inf"):
            return float(low)
        if low == "-0.0":
            return -0.0
        return float.fromhex(v)
    return float(v)


def expected(case):
    dt = case["dtype"]
    vals = case["values"]
    shape = tuple(case["shape"])
    if dt.startswith("complex"):
        # values interleaved re, im
        real = "float32" if dt == "complex64" else "float64"
        a = np.array([_f(v) for v in vals], dtype=np.float64).astype(real).view(dt)
    elif dt.startswith("float"):
        a = np.array([_f(v) for v in vals], dtype=np.float64).astype(dt)
    elif dt == "bool":
        a = np.array(vals, dtype=bool)
    elif dt.startswith("int"):
        a = np.array([int(v) for v in vals], dtype=np.int64).astype(dt)
    else:
        a = np.array([int(v) for v in vals], dtype=np.uint64).astype(dt)
    return a.reshape(shape)


def _ordered(a):
    """Float bit patterns mapped to integers that are monotone in the float value."""
    if a.dtype == np.float32:
        i = a.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)
    i = a.view(np.int64)
    return np.where(i < 0, -(i & np.int64(0x7FFFFFFFFFFFFFFF)), i)


def ulp_distance(a, b):
    """Units in the last place between two float arrays of one dtype (NaN == NaN, values of
    opposite sign count as far apart)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b, dtype=a.dtype)
    oa, ob = _ordered(a), _ordered(b)
    same = (oa >= 0) == (ob >= 0)
    with np.errstate(over="ignore"):
        d = np.where(same, np.abs(oa - ob), np.iinfo(np.int64).max)
    return np.where(np.isnan(a) & np.isnan(b), 0, d)


def max_ulp(got, want):
    d = ulp_distance(np.asarray(got, dtype=want.dtype), want)
    return int(np.max(d)) if d.size else 0


def check(case, got):
    """(ok, detail) for a computed array against the case's expected values."""
    want = expected(case)
    got = np.asarray(got)
    if tuple(got.shape) != tuple(want.shape):
        return False, f"shape {got.shape} != {want.shape}"
    cmp = case["compare"]
    if want.dtype.kind == "c":
        # compared component by component
        got = np.ascontiguousarray(got.astype(want.dtype)).view(want.real.dtype)
        want = np.ascontiguousarray(want).view(want.real.dtype)
    if want.dtype.kind in "uib":
        ok = np.array_equal(got.astype(want.dtype), want)
        return ok, "exact" if ok else f"got {got.ravel().tolist()} want {want.ravel().tolist()}"
    got = got.astype(want.dtype)
    u = max_ulp(got, want)
    if cmp == "exact":
        ok = np.array_equal(got.view(f"u{want.itemsize}"), want.view(f"u{want.itemsize}"))
        return ok, f"max ulp {u}"
    if cmp == "ulp16":
        return u <= 16, f"max ulp {u}"
    tol = float(cmp.split(":")[1])
    fin = np.isfinite(want)
    same_special = np.array_equal(np.isnan(got[~fin]), np.isnan(want[~fin])) and np.array_equal(
        got[~fin & ~np.isnan(want)], want[~fin & ~np.isnan(want)])
    err = np.abs(got[fin].astype(np.float64) - want[fin].astype(np.float64))
    ok = bool(np.all(err <= tol * np.abs(want[fin].astype(np.float64)) + tol * 1e-3)) and same_special
    return ok, f"max ulp {u}"


# ---- replaying a case ------------------------------------------------------------------

def shape_size(shape):
    return int(np.prod(shape)) if len(shape) else 1


def float_dtype(args):
    if "dtype" in args:
        return args["dtype"]
    return "float64" if args.get("x64") else "float32"


def bits_to_float32(bits, dtype):
    """16-bit float bit patterns -> float32 values."""
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == "bfloat16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def _fma(a, b, c, npdt):
    """a * b + c rounded once to npdt (float32 or float64), from exact rationals."""
    from fractions import Fraction
    exact = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    if npdt == np.float32:
        # float(Fraction) rounds to double correctly; double -> float32 can double-round,
        # so round to float32 from the exact value directly.
        return _round_f32(exact)
    return float(exact)


def _round_f32(q):
    """Nearest float32 (ties to even) of an exact rational."""
    d = np.float32(float(q))
    lo = np.nextafter(d, np.float32(-np.inf))
    hi = np.nextafter(d, np.float32(np.inf))
    from fractions import Fraction
    best = min((lo, d, hi), key=lambda v: (abs(Fraction(float(v)) - q),
                                            int(np.array(v).view(np.uint32)) & 1))
    return best


def evaluate(case, be):
    """Replay `case` through backend `be` (see OracleBackend for the interface)."""
    a = case["args"]
    op = case["op"]
    x64 = bool(a.get("x64", False))
    part = bool(a.get("partitionable", True))

    def key_of(seed):
        if a.get("impl", "threefry2x32") != "threefry2x32":
            return be.rbg_seed(seed, x64, a["impl"])
        k = be.seed(seed, x64)
        if "fold" in a:
            k = be.fold_in(k, a["fold"])
        return k

    if op == "rbg_bits":
        n = shape_size(a["shape"])
        return np.asarray(be.rbg_bits(key_of(a["seed"]), a["bits"], n)).reshape(tuple(a["shape"]))
    if op == "rbg_split":
        return np.asarray(be.rbg_split(key_of(a["seed"]), a["num"], a["impl"], part))
    if op == "rbg_fold_in":
        return np.asarray(be.rbg_fold_in(key_of(a["seed"]), a["data"], a["impl"]))
    if op == "rbg_vmap_bits":
        keys = be.rbg_split(key_of(a["seed"]), a["nkeys"], a["impl"], part)
        return np.asarray(be.rbg_vmap_bits(keys, tuple(a["shape"])))

    if op == "threefry_2x32":
        return be.threefry_2x32(a["key"], a["count"])
    if op == "seed":
        return be.seed(a["seed"], x64)
    if op == "fold_in":
        return be.fold_in(be.seed(a["seed"], x64), a["data"])
    if op == "split":
        n = shape_size(a["shape"])
        return be.split(key_of(a["seed"]), n, part).reshape(tuple(a["shape"]) + (2,))
    if op == "vmap_split":
        keys = be.split(be.seed(a["seed"], x64), a["nkeys"], part)
        return np.stack([be.split(k, shape_size(a["shape"]), part) for k in keys]).reshape(
            (a["nkeys"],) + tuple(a["shape"]) + (2,))
    if op == "vmap_fold_in":
        k = be.seed(a["seed"], x64)
        return np.stack([be.fold_in(k, d) for d in a["data"]])
    if op == "vmap_seed":
        return np.stack([be.seed(s, x64) for s in a["seeds"]])
    if op == "bits":
        bw = {"uint8": 8, "uint16": 16, "uint32": 32, "uint64": 64}[case["dtype"]]
        n = shape_size(a["shape"])
        return be.bits(key_of(a["seed"]), bw, n, part).reshape(tuple(a["shape"]))
    if op in ("uniform", "vmap_uniform"):
        dt = float_dtype(a)
        shape = tuple(a["shape"])
        n = shape_size(shape)
        mn, mx = a.get("minval", 0.0), a.get("maxval", 1.0)
        keys = [key_of(a["seed"])] if op == "uniform" else list(
            be.split(be.seed(a["seed"], x64), a["nkeys"], part))
        outs = []
        for k in keys:
            if np.ndim(mn) == 0 and np.ndim(mx) == 0:
                u = be.uniform(k, dt, n, part, float(mn), float(mx))
            else:
                u = be.uniform_array_bounds(k, dt, shape, part, mn, mx)
            outs.append(np.asarray(u).reshape(shape))
        out = outs[0] if op == "uniform" else np.stack(outs)
        if dt in ("float16", "bfloat16"):
            out = bits_to_float32(out, dt)
        return out
    if op == "normal" and float_dtype(a).startswith("complex"):
        dt = float_dtype(a)
        shape = tuple(a["shape"])
        return np.asarray(be.complex_normal(key_of(a["seed"]), dt, shape_size(shape),
                                            part)).reshape(shape)
    if op in ("normal", "vmap_normal"):
        dt = float_dtype(a)
        shape = tuple(a["shape"])
        n = shape_size(shape)
        keys = [key_of(a["seed"])] if op == "normal" else list(
            be.split(be.seed(a["seed"], x64), a["nkeys"], part))
        outs = [np.asarray(be.normal(k, dt, n, part)).reshape(shape) for k in keys]
        out = outs[0] if op == "normal" else np.stack(outs)
        if "loc" in a or "scale" in a:
            npdt = np.dtype(dt)
            loc = np.asarray(a.get("loc", 0.0), dtype=npdt)
            scale = np.asarray(a.get("scale", 1.0), dtype=npdt)
            out = (loc + scale * out.astype(npdt)).astype(npdt)
        return out
    if op == "bernoulli":
        dt = "float64" if x64 else "float32"
        npdt = np.dtype(dt)
        p = a["p"]
        shape = tuple(a["shape"])
        k = key_of(a["seed"])
        if a.get("mode", "low") == "high":
            u = np.asarray(be.uniform(k, dt, 2 * shape_size(shape), part, 0.0, 1.0)).reshape(
                (2,) + shape)
            nmant = 23 if dt == "float32" else 52
            u1 = u[0]
            u2 = (u[1] * npdt.type(2.0 ** -nmant)).astype(npdt)
            return u2 < (npdt.type(p) - u1).astype(npdt)
        if np.ndim(p) == 0:
            return np.asarray(be.bernoulli(k, dt, float(p), shape_size(shape), part)).astype(
                bool).reshape(shape)
        u = np.asarray(be.uniform(k, dt, shape_size(shape), part, 0.0, 1.0)).reshape(shape)
        return u < np.asarray(p, dtype=npdt)
    if op == "randint":
        dt = a.get("dtype", "int64" if x64 else "int32")
        shape = tuple(a["shape"])
        return np.asarray(be.randint(key_of(a["seed"]), shape, a["minval"], a["maxval"], dt,
                                     part)).reshape(shape)
    if op in ("exponential", "gumbel", "laplace", "logistic", "truncated_normal"):
        dt = float_dtype(a)
        shape = tuple(a["shape"])
        k = key_of(a["seed"])
        n = shape_size(shape)
        if op == "truncated_normal":
            out = be.truncated_normal(k, dt, n, part, float(a["lower"]), float(a["upper"]))
        else:
            out = be.sample(k, op, dt, n, part, a.get("mode", "low"))
        out = np.asarray(out).reshape(shape)
        return bits_to_float32(out, dt) if dt in ("float16", "bfloat16") else out
    if op == "permutation":
        x = a["x"]
        if x == "arange12_f32_4x3":
            x = np.arange(12, dtype=np.float32).reshape(4, 3)
        return np.asarray(be.permutation(key_of(a["seed"]), x, part))
    if op == "choice":
        a_ = a["a"]
        if isinstance(a_, list):
            a_ = np.asarray(a_, dtype=np.int32)
        return np.asarray(be.choice(key_of(a["seed"]), a_, tuple(a["shape"]),
                                    a.get("replace", True), a.get("p"), part, x64))
    if op == "erf_inv":
        dt = a["dtype"]
        xs = np.array([_f(v) for v in a["x"]], dtype=np.float64).astype(dt)
        return be.erfinv(xs, dt, bool(a.get("accurate", False)))
    raise ValueError(f"unknown op {op}")


class OracleBackend:
    """Replays cases through the CPU oracle."""

    def __init__(self, mul_add_fma=True, erfinv_fma=True):
        from oracle import oracle as orc
        self.o = orc
        self.mul_add_fma = mul_add_fma
        self.erfinv_fma = erfinv_fma

    def threefry_2x32(self, key, count):
        return self.o.threefry_2x32(key, count)

    def seed(self, s, x64):
        return self.o.seed(s, x64)

    def fold_in(self, key, data):
        return self.o.fold_in(key, data)

    def split(self, key, n, part):
        return self.o.split(key, n, part)

    def bits(self, key, bw, n, part):
        return self.o.random_bits(key, bw, n, part)

    def uniform(self, key, dt, n, part, mn, mx):
        if len(key) == 4:  # an rbg key: the same transform of the Philox bits
            assert dt == "float32" and (mn, mx) == (0.0, 1.0)
            b = self.o.rbg_bits(key, 32, n)
            return ((b >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1)
        return self.o.uniform(key, dt, n, part, mn, mx, fma=self.mul_add_fma)

    def uniform_array_bounds(self, key, dt, shape, part, mn, mx):
        npdt = np.dtype(dt)
        f = self.o.uniform(key, dt, shape_size(shape), part, 0.0, 1.0).reshape(shape)
        mn = np.broadcast_to(np.asarray(mn, dtype=np.float64).astype(npdt), shape)
        mx = np.broadcast_to(np.asarray(mx, dtype=np.float64).astype(npdt), shape)
        d = (mx - mn).astype(npdt)
        if self.mul_add_fma:  # one rounding of the exact f * d + mn
            r = np.array([_fma(a, b, c, npdt) for a, b, c in zip(f.ravel(), d.ravel(), mn.ravel())],
                         dtype=npdt).reshape(shape)
        else:
            r = (f * d).astype(npdt) + mn
        return np.maximum(mn, r.astype(npdt))

    def normal(self, key, dt, n, part):
        return self.o.normal(key, dt, n, part, fma=self.erfinv_fma)

    def complex_normal(self, key, dt, n, part):
        return self.o.complex_normal(key, dt, n, part)

    def bernoulli(self, key, dt, p, n, part):
        return self.o.bernoulli(key, dt, p, n, part)

    def erfinv(self, xs, dt, accurate=False):
        return self.o.erfinv(xs, dt, fma=self.erfinv_fma, accurate=accurate)

    def randint(self, key, shape, mn, mx, dt, part):
        return self.o.randint(key, shape, mn, mx, dt, part)

    def rbg_seed(self, s, x64, impl):
        return self.o.rbg_seed(s, x64)

    def rbg_bits(self, key, bw, n):
        return self.o.rbg_bits(key, bw, n)

    def rbg_split(self, key, num, impl, part):
        if impl == "rbg":
            return self.o.rbg_split(key, num, part)
        return self.o.rbg_unsafe_split(key, num)

    def rbg_fold_in(self, key, data, impl):
        if impl == "rbg":
            return self.o.rbg_fold_in(key, data)
        return self.o.rbg_unsafe_fold_in(key, data)

    def rbg_vmap_bits(self, keys, shape):
        # the batching rule of rng_bit_generator: every lane draws from the first key
        n = shape_size(shape)
        return self.o.rbg_bits(keys[0], 32, len(keys) * n).reshape((len(keys),) + shape)

    def sample(self, key, kind, dt, n, part, mode="low"):
        if kind == "gumbel" and mode != "low":
            return self.o.gumbel_mode(key, mode, dt, n, part)
        return self.o.sample(key, kind, dt, n, part)

    def truncated_normal(self, key, dt, n, part, lower, upper):
        return self.o.truncated_normal(key, dt, n, lower, upper, part)

    def permutation(self, key, x, part):
        return self.o.permutation(key, x, 0, False, part)

    def choice(self, key, a, shape, replace, p, part, x64):
        return self.o.choice(key, a, shape, replace, p, 0, part, x64)
