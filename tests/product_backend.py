"""Replays golden cases through the product's public API (jaxr_b200), on the GPU."""

from __future__ import annotations

import contextlib

import numpy as np
import torch

import jaxr_b200 as jr
from jaxr_b200 import random as jrr


def to_np(t):
    if isinstance(t, jr.PRNGKeyArray):
        t = t.data
    t = t.detach().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.float().numpy()
    return t.numpy()


@contextlib.contextmanager
def flags(x64=False, partitionable=True):
    with jr.with_jax_config("jax_enable_x64", x64), \
            jr.with_jax_config("jax_threefry_partitionable", partitionable):
        yield


class ProductBackend:
    """The interface of golden_cases.OracleBackend on jaxr_b200 (raw uint32 keys)."""

    def __init__(self, x64=False, partitionable=True):
        self.x64 = x64
        self.part = partitionable

    def _ctx(self, part=None):
        return flags(self.x64, self.part if part is None else part)

    def threefry_2x32(self, key, count):
        k = torch.tensor(np.asarray(key, dtype=np.uint32))
        c = torch.tensor(np.asarray(count, dtype=np.uint32))
        return to_np(jr.threefry_2x32(k, c))

    def seed(self, s, x64):
        with flags(x64, self.part):
            return to_np(jr.random_PRNGKey(s))

    def rbg_seed(self, s, x64, impl):
        with flags(x64, self.part):
            return jr.random_key(s, impl=impl)

    def rbg_bits(self, key, bw, n):
        with self._ctx():
            return to_np(jr.random_bits(key, (n,), f"uint{bw}"))

    def rbg_split(self, key, num, impl, part):
        with self._ctx(part):
            return to_np(jr.random_key_data(jr.random_split(key, num)))

    def rbg_fold_in(self, key, data, impl):
        with self._ctx():
            return to_np(jr.random_key_data(jr.random_fold_in(key, data)))

    def rbg_vmap_bits(self, keys, shape):
        with self._ctx():
            typed = jr.random_wrap_key_data(torch.tensor(np.asarray(keys, np.uint32)), impl="rbg")
            return to_np(jr.vmap(lambda k: jr.random_bits(k, shape))(typed))

    def fold_in(self, key, data):
        with self._ctx():
            return to_np(jr.random_fold_in(torch.tensor(np.asarray(key, np.uint32)), int(data)))

    def split(self, key, n, part):
        with self._ctx(part):
            return to_np(jr.random_split(torch.tensor(np.asarray(key, np.uint32)), n))

    def bits(self, key, bw, n, part):
        with flags(bw == 64 or self.x64, part):
            return to_np(jr.random_bits(torch.tensor(np.asarray(key, np.uint32)), (n,), f"uint{bw}"))

    def uniform(self, key, dt, n, part, mn, mx):
        if isinstance(key, jr.PRNGKeyArray):
            with flags(dt == "float64" or self.x64, part):
                return _raw(jr.random_uniform(key, (n,), dt, mn, mx), dt)
        with flags(dt == "float64" or self.x64, part):
            out = jr.random_uniform(torch.tensor(np.asarray(key, np.uint32)), (n,), dt, mn, mx)
        return _raw(out, dt)

    def uniform_array_bounds(self, key, dt, shape, part, mn, mx):
        with flags(dt == "float64" or self.x64, part):
            out = jr.random_uniform(torch.tensor(np.asarray(key, np.uint32)), shape, dt,
                                    np.asarray(mn, dtype=np.float64), np.asarray(mx, dtype=np.float64))
        return _raw(out, dt)

    def normal(self, key, dt, n, part):
        with flags(dt == "float64" or self.x64, part):
            out = jr.random_normal(torch.tensor(np.asarray(key, np.uint32)), (n,), dt)
        return _raw(out, dt)

    def complex_normal(self, key, dt, n, part):
        with flags(dt == "complex128" or self.x64, part):
            return to_np(jr.random_normal(torch.tensor(np.asarray(key, np.uint32)), (n,), dt))

    def bernoulli(self, key, dt, p, n, part):
        with flags(dt == "float64" or self.x64, part):
            pt = torch.tensor(p, dtype=jrr._TORCH[dt])
            return to_np(jr.random_bernoulli(torch.tensor(np.asarray(key, np.uint32)), pt, (n,)))

    def erfinv(self, xs, dt, accurate=False):
        with flags(dt == "float64", self.part), \
                jr.with_jax_config("jax_accurate_erf_inv", accurate):
            return to_np(jr.lax_erf_inv(torch.tensor(np.asarray(xs))))


    def randint(self, key, shape, mn, mx, dt, part):
        with flags(dt.endswith("64") or self.x64, part):
            mn = torch.tensor(mn, dtype=torch.int32) if isinstance(mn, list) else mn
            mx = torch.tensor(mx, dtype=torch.int32) if isinstance(mx, list) else mx
            return to_np(jr.random_randint(torch.tensor(np.asarray(key, np.uint32)), shape, mn,
                                           mx, dt))

    def sample(self, key, kind, dt, n, part, mode="low"):
        fn = {"exponential": jr.random_exponential, "gumbel": jr.random_gumbel,
              "laplace": jr.random_laplace, "logistic": jr.random_logistic}[kind]
        kw = {"mode": mode} if kind == "gumbel" else {}
        with flags(dt == "float64" or self.x64, part):
            out = fn(torch.tensor(np.asarray(key, np.uint32)), (n,), dt, **kw)
        return _raw(out, dt)

    def truncated_normal(self, key, dt, n, part, lower, upper):
        with flags(dt == "float64" or self.x64, part):
            out = jr.random_truncated_normal(torch.tensor(np.asarray(key, np.uint32)), lower,
                                             upper, (n,), dt)
        return _raw(out, dt)


    def permutation(self, key, x, part):
        with flags(self.x64, part):
            return to_np(jr.random_permutation(torch.tensor(np.asarray(key, np.uint32)), x))

    def choice(self, key, a, shape, replace, p, part, x64):
        with flags(x64, part):
            a = torch.from_numpy(a) if isinstance(a, np.ndarray) else a
            return to_np(jr.random_choice(torch.tensor(np.asarray(key, np.uint32)), a, shape,
                                          replace, p))


def _raw(out, dt):
    """16-bit floats as their raw bits (as the oracle returns them)."""
    if dt in ("float16", "bfloat16"):
        return out.detach().cpu().view(torch.uint16).numpy()
    return to_np(out)
