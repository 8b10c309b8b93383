"""Extract the reference's golden vectors for the threefry path into a JSON fixture.

Run where the jaxR sources are available (the fixture this writes is committed, so the
tests do not need them):

    python tests/golden/make_golden.py JAXR_SOURCE_DIR   # or $JAXR_REFERENCE_DIR

The expected values are read from the reference's own tests as text (they were
produced there by jax 0.12.0.1 on CPU): tests/testthat/test-prng.R,
tests/testthat/test-random.R, tests/testthat/test-scipy-special.R and the JSON
fixtures tests/testthat/fixtures/{stateful_rng,lax_x32,lax_x64}.json.  The call
each vector pins (seed, operation, shape, flags) is transcribed below from the
test line that makes it, and every case records that line as its "source".
"""

from __future__ import annotations

import json
import math
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "threefry_golden.json")


# ---- a small reader for R literals -------------------------------------------------------

_TOKEN = re.compile(
    r"\s*(?:(?P<num>-?Inf\b|NaN\b|-?0x[0-9a-fA-F]+(?:\.[0-9a-fA-F]*)?(?:p[-+]?\d+)?|-?\d+\.?\d*(?:e[-+]?\d+)?L?)"
    r"|(?P<str>\"[^\"]*\")|(?P<id>[A-Za-z_.][A-Za-z0-9_.]*)|(?P<op>[(),=]))"
)


def _tokens(text):
    pos = 0
    out = []
    while pos < len(text):
        if text[pos].isspace():
            pos += 1
            continue
        m = _TOKEN.match(text, pos)
        if not m or m.end() == pos:
            raise ValueError(f"cannot read R literal at {text[pos:pos + 40]!r}")
        for kind in ("num", "str", "id", "op"):
            if m.group(kind) is not None:
                out.append((kind, m.group(kind)))
                break
        pos = m.end()
    return out


def _num(s):
    if s in ("NaN", "Inf", "-Inf"):
        return float(s.replace("NaN", "nan").replace("Inf", "inf"))
    neg = s.startswith("-")
    t = (s[1:] if neg else s).rstrip("L")
    if t.lower().startswith("0x"):
        v = float.fromhex(t) if ("." in t or "p" in t.lower()) else int(t, 16)
    elif any(ch in t for ch in ".e"):
        v = float(t)
    else:
        v = int(t)
    return -v if neg else v


class _Reader:
    def __init__(self, toks):
        self.t = toks
        self.i = 0

    def peek(self):
        return self.t[self.i] if self.i < len(self.t) else (None, None)

    def take(self, want=None):
        tok = self.t[self.i]
        if want is not None and tok[1] != want:
            raise ValueError(f"expected {want!r}, got {tok!r}")
        self.i += 1
        return tok

    def value(self):
        kind, v = self.take()
        if kind == "num":
            return _num(v)
        if kind == "str":
            return v[1:-1]
        if kind == "id":
            if v in ("TRUE", "FALSE"):
                return v == "TRUE"
            if v in ("c", "list", "integer"):
                self.take("(")
                items, names = [], []
                while self.peek()[1] != ")":
                    name = None
                    if self.peek()[0] == "id" and self.t[self.i + 1][1] == "=":
                        name = self.take()[1]
                        self.take("=")
                    items.append(self.value())
                    names.append(name)
                    if self.peek()[1] == ",":
                        self.take(",")
                self.take(")")
                if v == "integer":
                    return []
                if any(names):
                    return dict(zip(names, items))
                if v == "c":
                    flat = []
                    for it in items:
                        flat.extend(it if isinstance(it, list) else [it])
                    return flat
                return items
        raise ValueError(f"unexpected token {v!r}")


def read_r(text):
    return _Reader(_tokens(text)).value()


def _balanced(text, start):
    depth = 0
    for j in range(start, len(text)):
        if text[j] == "(":
            depth += 1
        elif text[j] == ")":
            depth -= 1
            if depth == 0:
                return j + 1
    raise ValueError("unbalanced parentheses")


def named_list(path, var, indent=""):
    """The `var <- list(...)` assignment of an R file: {name: (value, line)}."""
    text = open(path).read()
    m = re.search(rf"^{indent}{re.escape(var)} <- list\(", text, re.M)
    body_start = m.end() - 1
    end = _balanced(text, body_start)
    out = {}
    for em in re.finditer(r"^\s+([A-Za-z0-9_]+) = list\(", text[body_start:end], re.M):
        s = body_start + em.end() - len("list(")
        e = _balanced(text, s)
        line = text.count("\n", 0, s) + 1
        out[em.group(1)] = (read_r(text[s:e]), line)
    return out


def literal_at(path, pattern, which=0):
    """The `which`-th `list(...)` literal from the first match of `pattern` on, possibly
    continued over the following lines, and the line number of the match."""
    text = open(path).read()
    m = re.search(pattern, text, re.M)
    if not m:
        raise ValueError(f"pattern {pattern!r} not found in {path}")
    starts = [k.start() + m.start() for k in re.finditer(r"list\(", text[m.start():])]
    s = starts[which]
    return read_r(text[s:_balanced(text, s)]), text.count("\n", 0, m.start()) + 1


def c_vector_at(path, pattern):
    """The first `c(...)` vector starting after the first match of `pattern`."""
    text = open(path).read()
    m = re.search(pattern, text)
    s = text.index("c(", m.end())
    line = text.count("\n", 0, s) + 1
    return read_r(text[s:_balanced(text, s)]), line


# ---- value encoding ----------------------------------------------------------------------

def _enc(v, dtype):
    if dtype.startswith("float"):
        if isinstance(v, str):
            return v
        f = float(v)
        if math.isnan(f):
            return "nan"
        if math.isinf(f):
            return "inf" if f > 0 else "-inf"
        return f.hex()
    if dtype == "bool":
        return bool(v)
    return int(v)


def case(name, source, op, args, dtype, shape, values, compare, **extra):
    if isinstance(shape, int):
        shape = [shape]
    if dtype.startswith("complex"):
        # list(re = c(...), im = c(...)) -> re0, im0, re1, im1, ... as component floats
        real = "float32" if dtype == "complex64" else "float64"
        values = [_enc(v, real) for pair in zip(values["re"], values["im"]) for v in pair]
        d = {"name": name, "source": source, "op": op, "args": args, "dtype": dtype,
             "shape": list(shape), "values": values, "compare": compare}
        d.update(extra)
        return d
    d = {"name": name, "source": source, "op": op, "args": args, "dtype": dtype,
         "shape": list(shape), "values": [_enc(v, dtype) for v in values], "compare": compare}
    d.update(extra)
    return d


# ---- the cases ---------------------------------------------------------------------------

def _log_allowance(name):
    """Ulp allowance of the log-transform samplers against the recorded values.  Their
    logarithms are evaluated here to within an ulp of the correctly rounded result; the
    reference's float32 values come from XLA's own float32 log/log1p, which is up to an ulp
    from correctly rounded (its float64 values are correctly rounded; ours are within 3
    ulp).  gumbel "high" takes log(-a) of a = log1p(-x) near -1, which multiplies a
    one-ulp difference in a by 16 (test-random.R:10-27 allows 16 ulp for all samplers)."""
    if name in ("exponential", "gumbel", "gumbel_highest", "laplace", "logistic"):
        return {"max_ulp": 3}
    if name == "gumbel_high":
        return {"max_ulp": 16}
    return {}


def build(ref):
    tt = os.path.join(ref, "tests", "testthat")
    prng = os.path.join(tt, "test-prng.R")
    rand = os.path.join(tt, "test-random.R")
    spec = os.path.join(tt, "test-scipy-special.R")
    cases = []
    src = lambda path, line: f"tests/testthat/{os.path.basename(path)}:{line}"

    # Known-answer vectors of threefry_2x32 (test-prng.R:61-66).
    kat_keys = {
        r"tf\(u\(0, 0\), u\(0, 0\)\)": ([0, 0], [0, 0]),
        r"tf\(u\(2\^32 - 1, 2\^32 - 1\)": ([2**32 - 1] * 2, [2**32 - 1] * 2),
        r"tf\(u\(0x13198a2e, 0x03707344\), u\(0x243f6a88": ([0x13198a2E, 0x03707344],
                                                            [0x243F6A88, 0x85A308D3]),
        r"rp_expect\(tf\(u\(0x13198a2e, 0x03707344\), jnp_arange\(5L": ([0x13198a2E, 0x03707344],
                                                                       list(range(5))),
    }
    for k, (pat, (key, count)) in enumerate(kat_keys.items()):
        (shape, vals, dt), line = literal_at(prng, pat)
        cases.append(case(f"kat_{k}", src(prng, line), "threefry_2x32",
                          {"key": key, "count": count}, dt, [shape] if isinstance(shape, int) else shape,
                          vals, "exact"))

    # rp_ref (test-prng.R:26-55).  Call of each name, from test-prng.R:75-111 and :179-201.
    rp = named_list(prng, "rp_ref")
    rp_calls = {
        "PRNGKey_0": ("seed", {"seed": 0}),
        "PRNGKey_42": ("seed", {"seed": 42}),
        "PRNGKey_m1": ("seed", {"seed": -1}),
        "PRNGKey_big": ("seed", {"seed": 2**40 + 5}),
        "split_0": ("split", {"seed": 0, "shape": [2]}),
        "split_42_3": ("split", {"seed": 42, "shape": [3]}),
        "split_0_23": ("split", {"seed": 0, "shape": [2, 3]}),
        "fold_in_0_7": ("fold_in", {"seed": 0, "data": 7}),
        "fold_in_42_max": ("fold_in", {"seed": 42, "data": 2**32 - 1}),
        "bits_0_5": ("bits", {"seed": 0, "shape": [5]}),
        "bits_42_23": ("bits", {"seed": 42, "shape": [2, 3]}),
        "bits_0_u8": ("bits", {"seed": 0, "shape": [7]}),
        "bits_0_u16": ("bits", {"seed": 0, "shape": [5]}),
        "np_split_0": ("split", {"seed": 0, "shape": [2], "partitionable": False}),
        "np_split_42_3": ("split", {"seed": 42, "shape": [3], "partitionable": False}),
        "np_bits_0_5": ("bits", {"seed": 0, "shape": [5], "partitionable": False}),
        "np_bits_0_u8": ("bits", {"seed": 0, "shape": [7], "partitionable": False}),
        "np_bits_0_u16": ("bits", {"seed": 0, "shape": [5], "partitionable": False}),
        # vmap(function(k) random_split(k))(random_split(k0, 3))
        "vmap_split": ("vmap_split", {"seed": 0, "nkeys": 3, "shape": [2]}),
        # vmap(function(d) random_fold_in(k0, d))(jnp_arange(3L))
        "vmap_fold_in": ("vmap_fold_in", {"seed": 0, "data": [0, 1, 2]}),
        # vmap(function(s) random_key_data(random_key(s)))(jnp_arange(3L))
        "vmap_key": ("vmap_seed", {"seeds": [0, 1, 2]}),
        # rbg / unsafe_rbg (test-prng.R:216-236, :249)
        "rbg_bits": ("rbg_bits", {"seed": 0, "impl": "rbg", "shape": [4], "bits": 32}),
        "rbg_bits_u8": ("rbg_bits", {"seed": 3, "impl": "rbg", "shape": [5], "bits": 8}),
        "rbg_split": ("rbg_split", {"seed": 0, "impl": "rbg", "num": 3}),
        "rbg_fold_in": ("rbg_fold_in", {"seed": 0, "impl": "rbg", "data": 5}),
        "unsafe_rbg_split": ("rbg_split", {"seed": 0, "impl": "unsafe_rbg", "num": 3}),
        "unsafe_rbg_fold_in": ("rbg_fold_in", {"seed": 0, "impl": "unsafe_rbg", "data": 5}),
        # vmap(function(k) random_bits(k, 3))(random_split(random_key(0, impl = "rbg"), 2))
        "rbg_vmap_bits": ("rbg_vmap_bits", {"seed": 0, "impl": "rbg", "nkeys": 2, "shape": [3]}),
    }
    for name, (op, args) in rp_calls.items():
        (shape, vals, dt), line = rp[name]
        shape = [shape] if isinstance(shape, int) else shape
        cases.append(case(name, src(prng, line), op, args, dt, shape, vals, "exact"))

    # x64 seeds and uint64 bits (test-prng.R:118-127), compared through (hi, lo) halves.
    for seed, pat in ((-1, r"random_PRNGKey\(-1\), list\(2, c\(4294967295"),
                      (2**40 + 5, r"random_PRNGKey\(2\^40 \+ 5\), list\(2, c\(256")):
        (shape, vals, dt), line = literal_at(prng, pat)
        cases.append(case(f"x64_PRNGKey_{seed}", src(prng, line), "seed",
                          {"seed": seed, "x64": True}, dt, shape, vals, "exact"))
    for seed, shape, pat in ((0, [5], r"rp_expect_u64\(random_bits\(k0, 5\)"),
                             (42, [2, 3], r"rp_expect_u64\(random_bits\(random_PRNGKey\(42\)")):
        hi, line = c_vector_at(prng, pat + r"[\s\S]*?hi = ")
        lo, _ = c_vector_at(prng, pat + r"[\s\S]*?lo = ")
        vals = [(h << 32) | l for h, l in zip(hi, lo)]
        cases.append(case(f"x64_bits_{seed}", src(prng, line), "bits",
                          {"seed": seed, "shape": shape, "x64": True}, "uint64", shape, vals,
                          "exact"))

    # rr_ref (test-random.R:41-114), the threefry uniform/normal/bernoulli entries.
    rr = named_list(rand, "rr_ref")
    rr_calls = {
        "uniform_0_5": ("uniform", {"seed": 0, "shape": [5]}),
        "uniform_42_23_m": ("uniform", {"seed": 42, "shape": [2, 3], "minval": -2, "maxval": 3}),
        "uniform_0_minvec": ("uniform", {"seed": 0, "shape": [2, 3], "minval": [0, 1, 2],
                                         "maxval": 5}),
        "normal_0_5": ("normal", {"seed": 0, "shape": [5]}),
        "normal_42_23": ("normal", {"seed": 42, "shape": [2, 3]}),
        "normal_0_c64": ("normal", {"seed": 0, "shape": [3], "dtype": "complex64"}),
        "unif_bf16": ("uniform", {"seed": 0, "shape": [4], "dtype": "bfloat16"}),
        "unif_f16": ("uniform", {"seed": 0, "shape": [4], "dtype": "float16"}),
        # vmap(function(k) random_uniform(k, 3))(random_split(rr_k0(), 4))
        "vmap_uniform": ("vmap_uniform", {"seed": 0, "nkeys": 4, "shape": [3]}),
        "np_uniform_0_5": ("uniform", {"seed": 0, "shape": [5], "partitionable": False}),
        "np_normal_42": ("normal", {"seed": 42, "shape": [2, 3], "partitionable": False}),
        "bernoulli": ("bernoulli", {"seed": 7, "shape": [8], "p": 0.3}),
        "bernoulli_high": ("bernoulli", {"seed": 7, "shape": [8], "p": 0.3, "mode": "high"}),
        "bernoulli_vec": ("bernoulli", {"seed": 7, "shape": [3], "p": [0.1, 0.5, 0.9]}),
        # randint (test-random.R:133-139)
        "randint_0_6": ("randint", {"seed": 0, "shape": [6], "minval": 0, "maxval": 10}),
        "randint_42_neg": ("randint", {"seed": 42, "shape": [5], "minval": -5, "maxval": 5}),
        "randint_u8": ("randint", {"seed": 0, "shape": [6], "minval": 0, "maxval": 256,
                                   "dtype": "uint8"}),
        "randint_i8": ("randint", {"seed": 42, "shape": [6], "minval": -128, "maxval": 127,
                                   "dtype": "int8"}),
        "randint_vec": ("randint", {"seed": 0, "shape": [2, 3], "minval": [0, 10, 100],
                                    "maxval": [5, 20, 1000]}),
        "randint_empty": ("randint", {"seed": 0, "shape": [4], "minval": 5, "maxval": 5}),
        # log-transform samplers and truncated normal (test-random.R:213-226)
        "exponential": ("exponential", {"seed": 7, "shape": [4]}),
        "gumbel": ("gumbel", {"seed": 7, "shape": [4]}),
        "gumbel_high": ("gumbel", {"seed": 7, "shape": [4], "mode": "high"}),
        "gumbel_highest": ("gumbel", {"seed": 7, "shape": [4], "mode": "highest"}),
        "laplace": ("laplace", {"seed": 7, "shape": [4]}),
        "logistic": ("logistic", {"seed": 7, "shape": [4]}),
        "truncnorm": ("truncated_normal", {"seed": 7, "shape": [4], "lower": -1, "upper": 2}),
        # permutation and choice (test-random.R:338-344, :251)
        "permutation": ("permutation", {"seed": 7, "x": 10}),
        "perm_arr": ("permutation", {"seed": 7, "x": "arange12_f32_4x3"}),
        "choice": ("choice", {"seed": 7, "a": 10, "shape": [4]}),
        "choice_norep": ("choice", {"seed": 7, "a": 10, "shape": [4], "replace": False}),
        "choice_p": ("choice", {"seed": 7, "a": 5, "shape": [6], "p": [0.1, 0.2, 0.3, 0.2, 0.2]}),
        # random_uniform(random_key(0, impl = "rbg"), 4) (test-random.R:140)
        "rbg_uniform": ("uniform", {"seed": 0, "impl": "rbg", "shape": [4]}),
    }
    for name, (op, args) in rr_calls.items():
        (shape, vals, dt), line = rr[name]
        shape = [shape] if isinstance(shape, int) else shape
        cmp = "ulp16" if dt.startswith("float") else "exact"
        if dt.startswith("complex"):
            cmp = "rel:1e-6"  # test-random.R:131-132 compares complex normals to 1e-6
        if name.startswith("unif_"):
            args["result_as"] = "float32"  # the test compares jnp_astype(..., "float32")
        cases.append(case(name, src(rand, line), op, args, dt, shape, vals, cmp,
                          **_log_allowance(name)))

    # choice from an array (test-random.R:342, values inline in the call)
    ln = next(k + 1 for k, l in enumerate(open(rand).read().split("\n"))
              if "random_choice(kd, jnp_arange(5L) * 10L, c(2, 2))" in l)
    cases.append(case("choice_arr", src(rand, ln), "choice",
                      {"seed": 7, "a": [0, 10, 20, 30, 40], "shape": [2, 2]}, "int32", [2, 2],
                      [40, 20, 0, 20], "exact"))

    # x64 samplers (test-random.R:158-206).
    x64ref = named_list(rand, "ref", indent="  ")
    text = open(rand).read().split("\n")
    x64_calls = {
        "uniform_0_5": ("uniform", {"seed": 0, "shape": [5]}),
        "uniform_42_23_m": ("uniform", {"seed": 42, "shape": [2, 3], "minval": -2, "maxval": 3}),
        "normal_0_5": ("normal", {"seed": 0, "shape": [5]}),
        "normal_0_c128": ("normal", {"seed": 0, "shape": [3], "dtype": "complex128"}),
        "np_uniform_0_5": ("uniform", {"seed": 0, "shape": [5], "partitionable": False}),
        "randint_0_6": ("randint", {"seed": 0, "shape": [6], "minval": 0, "maxval": 10}),
        "randint_42_neg": ("randint", {"seed": 42, "shape": [5], "minval": -5, "maxval": 5}),
        "exponential": ("exponential", {"seed": 7, "shape": [4]}),
        "gumbel": ("gumbel", {"seed": 7, "shape": [4]}),
        "truncnorm": ("truncated_normal", {"seed": 7, "shape": [4], "lower": -1, "upper": 2}),
    }
    for name, (op, args) in x64_calls.items():
        (shape, vals, dt), line = x64ref[name]
        shape = [shape] if isinstance(shape, int) else shape
        args = dict(args, x64=True)
        # the reference holds its float64 truncated normal to 1e-14 relative (test-random.R:193)
        # complex128 normals are compared exactly (test-random.R:185, tol = 0)
        cmp = ("exact" if not dt.startswith("float") else
               "rel:1e-14" if name == "truncnorm" else "ulp16")
        cases.append(case(f"x64_{name}", src(rand, line), op, args, dt, shape, vals, cmp,
                          **_log_allowance(name)))
    (shape, vals, dt), line = rr["uniform_0_5"]
    ln206 = next(k + 1 for k, l in enumerate(text) if 'random_uniform(k0, 5, "float32")' in l)
    cases.append(case("x64_uniform_0_5_f32", src(rand, ln206), "uniform",
                      {"seed": 0, "shape": [5], "dtype": "float32", "x64": True}, dt, shape,
                      vals, "ulp16"))

    # Exact f32 normals under vmap (test-random.R:293-297).
    vals, line = c_vector_at(rand, r"expected <- (?=c\(0x1\.1d3)")
    cases.append(case("vmap_normal_exact", src(rand, line), "vmap_normal",
                      {"seed": 7, "nkeys": 3, "shape": [2], "typed_key": True}, "float32",
                      [3, 2], vals, "exact"))

    # Stateful generator (fixtures/stateful_rng.json; calls in
    # test-experimental-random.R:28-63): draw c of a generator seeded s uses
    # fold_in(key(s), c).
    sj = json.load(open(os.path.join(tt, "fixtures", "stateful_rng.json")))
    srcf = "tests/testthat/fixtures/stateful_rng.json"
    st = {
        "u1": ("uniform", {"seed": 42, "fold": 0, "shape": []}),
        "u2": ("uniform", {"seed": 42, "fold": 1, "shape": []}),
        "ju1": ("uniform", {"seed": 42, "fold": 2, "shape": []}),
        "ju2": ("uniform", {"seed": 42, "fold": 3, "shape": []}),
        "k1": ("fold_in", {"seed": 42, "data": 4}),
        "k2": ("fold_in", {"seed": 42, "data": 5}),
        "k3": ("split", {"seed": 42, "fold": 6, "shape": [3]}),
        "k23": ("split", {"seed": 42, "fold": 7, "shape": [2, 3]}),
        "key0a": ("fold_in", {"seed": 0, "data": 0}),
        "key0b": ("fold_in", {"seed": 0, "data": 1}),
        "random": ("uniform", {"seed": 7, "fold": 0, "shape": []}),
        "random3": ("uniform", {"seed": 7, "fold": 1, "shape": [3]}),
        "random23": ("uniform", {"seed": 7, "fold": 2, "shape": [2, 3]}),
        "unif_lh": ("uniform", {"seed": 7, "fold": 3, "shape": [3], "minval": -1,
                                "maxval": [1, 2, 3]}),
        "unif_size": ("uniform", {"seed": 7, "fold": 4, "shape": [4], "minval": 2, "maxval": 5}),
        "normal": ("normal", {"seed": 7, "fold": 5, "shape": []}),
        "normal_ls": ("normal", {"seed": 7, "fold": 6, "shape": [2], "loc": [0, 10], "scale": 2}),
        "normal_size": ("normal", {"seed": 7, "fold": 7, "shape": [2, 2], "loc": 1, "scale": 3}),
        "x64_u": ("uniform", {"seed": 42, "fold": 0, "shape": [], "x64": True}),
        "x64_n": ("normal", {"seed": 42, "fold": 2, "shape": [2], "x64": True}),
    }
    for name, (op, args) in st.items():
        e = sj[name]
        dt = e["dtype"]
        cmp = "exact" if dt == "uint32" else ("rel:2e-6" if dt == "float32" else "rel:1e-12")
        vals = [float(v) if dt.startswith("float") else int(v) for v in e["value"]]
        cases.append(case(f"stateful_{name}", f"{srcf}:{name}", op, args, dt, e["shape"], vals,
                          cmp))

    # erf_inv (fixtures/lax_x32.json and lax_x64.json "lax.erf_inv/*";
    # test-scipy-special.R:253-259).
    for fx in ("lax_x32.json", "lax_x64.json"):
        d = json.load(open(os.path.join(tt, "fixtures", fx)))
        for c in d["cases"]:
            if c.get("fn") != "lax_erf_inv" or c["args"][0].get("t") != "array":
                continue
            a = c["args"][0]
            if a["dtype"] not in ("float32", "float64"):
                continue
            o = c["out"]
            cases.append(case(f"erf_inv_{fx[:-5]}_{c['id'].split('/')[-1]}",
                              f"tests/testthat/fixtures/{fx}:{c['id']}", "erf_inv",
                              {"x": [v if v in ("NaN", "Inf", "-Inf", "-0.0") else v
                                     for v in a["data"]], "dtype": a["dtype"]},
                              o["dtype"], o["shape"],
                              [v for v in o["data"]], "ulp16"))
    for dt, pat in (("float32", r"scipy_special_erfinv\(as_jax\(array\((?=c\(0, 0.5, -0.8999)"),
                    ("float64", r"jit\(function\(x\) scipy_special_erfinv")):
        xs, line = c_vector_at(spec, pat)
        lst, _ = literal_at(spec, pat, which=0)
        cases.append(case(f"scipy_erfinv_{dt}", src(spec, line), "erf_inv",
                          {"x": [float(v) if not isinstance(v, str) else v for v in xs],
                           "dtype": dt}, dt, lst[1] if isinstance(lst[1], list) else [lst[1]],
                          lst[2], "rel:1e-12" if dt == "float64" else "rel:1e-5"))
    # the accurate erf_inv of jax_accurate_erf_inv (test-lax-special.R:204-212); the oracle
    # reproduces every recorded value bit for bit, so the comparison is exact
    lsp = os.path.join(tt, "test-lax-special.R")
    for dt, pat in (("float32", r"sp_erf_inv_impl\(as_jax\(array\((?=c\(0, 0.300000012)"),
                    ("float64", r"sp_erf_inv_impl\(as_jax\(array\((?=c\(0, 0x1.3333333333333p-2)")):
        xs, line = c_vector_at(lsp, pat)
        lst, _ = literal_at(lsp, pat, which=0)
        cases.append(case(f"erf_inv_accurate_{dt}", src(lsp, line), "erf_inv",
                          {"x": [float(v) if not isinstance(v, str) else v for v in xs],
                           "dtype": dt, "accurate": True}, dt,
                          lst[1] if isinstance(lst[1], list) else [lst[1]], lst[2], "exact"))
    return cases


def _normalise_specials(cases):
    for c in cases:
        if c["op"] != "erf_inv":
            continue
        xs = []
        for v in c["args"]["x"]:
            if isinstance(v, str):
                low = v.lower()
                xs.append({"nan": "nan", "inf": "inf", "-inf": "-inf"}.get(low, v))
            else:
                xs.append(float(v).hex())
        c["args"]["x"] = xs
        c["values"] = [{"NaN": "nan", "Inf": "inf", "-Inf": "-inf"}.get(v, v) for v in c["values"]]
    return cases


def main(argv):
    ref = argv[1] if len(argv) > 1 else os.environ.get("JAXR_REFERENCE_DIR")
    if not ref:
        sys.exit(f"usage: {argv[0]} JAXR_SOURCE_DIR (or set $JAXR_REFERENCE_DIR): the root "
                 "of the jaxR source tree to read")
    cases = _normalise_specials(build(ref))
    meta = {"generated_by": "tests/golden/make_golden.py",
            "reference": "jaxR (adamrsophie/jaxR); values produced there by jax 0.12.0.1 on CPU",
            "ncases": len(cases)}
    with open(OUT, "w") as f:
        json.dump({"meta": meta, "cases": cases}, f, indent=1)
        f.write("\n")
    print(f"wrote {len(cases)} cases to {OUT}")


if __name__ == "__main__":
    main(sys.argv)
