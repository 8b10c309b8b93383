"""The R .Call shim (jaxr_b200/r): its core's argument checks on the CPU, its R glue
compile-checked against declarations of R's C API (no R in this image), and -- on a GPU --
a plain C driver making the shim's call sequence through the core, whose results must
equal the oracle's."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RDIR = os.path.join(ROOT, "jaxr_b200", "r")
LIBDIR = os.path.join(ROOT, "jaxr_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _cc():
    cc = shutil.which("gcc")
    if cc is None or not os.path.exists(os.path.join(LIBDIR, "libjxrng.so")):
        pytest.skip("needs gcc and the built libjxrng.so")
    return cc


def _link_args():
    return ["-L" + LIBDIR, "-ljxrng", "-L" + os.path.join(CUDA, "lib64"), "-lcudart",
            "-Wl,-rpath," + LIBDIR, "-Wl,-rpath," + os.path.join(CUDA, "lib64")]


def _includes():
    return ["-I" + os.path.join(ROOT, "include"), "-I" + RDIR, "-I" + os.path.join(CUDA, "include")]


@pytest.fixture(scope="module")
def core(tmp_path_factory):
    cc = _cc()
    out = str(tmp_path_factory.mktemp("shim") / "libjxrng_shim.so")
    subprocess.run([cc, "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror", "-fPIC", "-shared",
                    *_includes(), os.path.join(RDIR, "jxrng_shim.c"), "-o", out, *_link_args()],
                   check=True)
    lib = ctypes.CDLL(out)
    lib.jxs_error.restype = ctypes.c_char_p
    lib.jxs_count.argtypes = [ctypes.c_double, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]
    lib.jxs_key_words.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.jxs_bytes.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_size_t)]
    return lib


def test_counts_are_whole_numbers_up_to_2p53(core):
    v = ctypes.c_uint64(0)
    for x in (0.0, 1.0, 2.0 ** 34, 2.0 ** 53):
        assert core.jxs_count(x, b"size", ctypes.byref(v)) == 0 and v.value == int(x)
    for x in (-1.0, 0.5, 2.0 ** 53 + 2, float("nan"), float("inf")):
        assert core.jxs_count(x, b"size", ctypes.byref(v)) == 1
        assert b"size must be a whole number in [0, 2^53]" in core.jxs_error()


def test_key_words_are_uint32_pairs(core):
    out = (ctypes.c_uint32 * 4)()
    ok = (ctypes.c_double * 4)(0, 42, 4294967295.0, 7)
    assert core.jxs_key_words(ok, 4, out) == 0 and list(out) == [0, 42, 4294967295, 7]
    assert core.jxs_key_words(ok, 3, out) == 1 and b"two words per key" in core.jxs_error()
    for bad in (4294967296.0, -1.0, 1.5, float("nan")):
        w = (ctypes.c_double * 2)(0, bad)
        assert core.jxs_key_words(w, 2, out) == 1 and b"not a uint32" in core.jxs_error()


def test_byte_counts_do_not_overflow(core):
    b = ctypes.c_size_t(0)
    assert core.jxs_bytes(1 << 40, 8, ctypes.byref(b)) == 0 and b.value == 8 << 40
    assert core.jxs_bytes(1 << 62, 8, ctypes.byref(b)) == 1 and b"overflow" in core.jxs_error()


def test_r_glue_compiles_against_r_api_declarations():
    """jxrng_r.c against tests/r_api (the R API functions it calls, declared as R declares
    them); R's own headers are not in this image."""
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-fsyntax-only",
                        "-I" + os.path.join(ROOT, "tests", "r_api"), *_includes(),
                        os.path.join(RDIR, "jxrng_r.c")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    src = open(os.path.join(RDIR, "jxrng_r.c")).read()
    registered = {ln.split('"')[1] for ln in src.splitlines() if ln.strip().startswith('{"jxr_r_')}
    assert registered == {"jxr_r_random_bits", "jxr_r_uniform", "jxr_r_normal", "jxr_r_bernoulli",
                          "jxr_r_split", "jxr_r_fold_in", "jxr_r_prepare"}
    rsrc = open(os.path.join(RDIR, "jxrng.R")).read()
    for name in registered:  # every routine the R side looks up exists, and vice versa
        assert f'"{name}"' in rsrc, name
    # the key-reuse sinks of prng_bits_jit / prng_split_jit (R/prng.R:524, :533) are kept
    code = "\n".join(ln for ln in rsrc.splitlines() if not ln.lstrip().startswith("#"))
    assert code.count('kr_sink(key, "random_bits")') == 4  # bits, uniform, normal, bernoulli
    assert code.count('kr_sink(key, "random_split")') == 1


@pytest.mark.gpu
def test_c_driver_matches_the_oracle(tmp_path):
    import torch

    from oracle import oracle as orc
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    cc = _cc()
    exe = str(tmp_path / "r_shim_driver")
    subprocess.run([cc, "-std=c99", "-O2", "-Wall", "-Werror", *_includes(),
                    os.path.join(ROOT, "tests", "r_shim_driver.c"), os.path.join(RDIR, "jxrng_shim.c"),
                    "-o", exe, *_link_args()], check=True)
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "R_SHIM_DRIVER_OK" in r.stdout, r.stderr[-2000:]

    def load(name, dt):
        return np.fromfile(tmp_path / f"{name}.bin", dtype=dt).reshape(2, -1)

    keys = [orc.seed(0), orc.seed(42)]
    n = 1001
    for i, k in enumerate(keys):
        assert np.array_equal(load("bits_p32", np.uint32)[i], orc.random_bits(k, 32, n, True))
        assert np.array_equal(load("bits_o8", np.uint8)[i], orc.random_bits(k, 8, n, False))
        assert np.array_equal(load("bits_p64", np.uint64)[i], orc.random_bits(k, 64, n, True))
        assert np.array_equal(load("unif_f32", np.uint32)[i],
                              orc.uniform(k, "float32", n, True, -2.0, 3.0).view(np.uint32))
        assert np.array_equal(load("unif_o64", np.uint64)[i],
                              orc.uniform(k, "float64", n, False, 0.0, 1.0).view(np.uint64))
        assert np.array_equal(load("unif_bf16", np.uint16)[i],
                              orc.uniform(k, "bfloat16", n, True, -1.0, 1.0).view(np.uint16))
        wz = orc.normal(k, "float32", n, True).view(np.int32).astype(np.int64)
        assert np.abs(load("norm_f32", np.int32)[i].astype(np.int64) - wz).max() <= 2
        w64 = orc.normal(k, "float64", n, True)
        assert np.all(np.abs(load("norm_f64", np.float64)[i] - w64) <= 1e-12 * np.abs(w64))
        wa = orc.normal(k, "float32", n, True, accurate=True)
        assert np.array_equal(load("norm_f32_acc", np.uint32)[i], wa.view(np.uint32))
        assert np.array_equal(load("bern_f32", np.uint8)[i],
                              orc.bernoulli(k, "float32", 0.3, n, True).astype(np.uint8))
        assert np.array_equal(load("split_p5", np.uint32)[i].reshape(5, 2), orc.split(k, 5, True))
        assert np.array_equal(load("split_o3", np.uint32)[i].reshape(3, 2), orc.split(k, 3, False))
        assert np.array_equal(load("fold_17", np.uint32)[i], orc.fold_in(k, 17))
