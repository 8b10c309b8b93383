"""Configuration flags read by the random-bits path (R/config.R:3-39, :75-114).

Only the options this path reads are kept: jax_enable_x64 (default dtypes and seed
width), jax_threefry_partitionable (counter layout), jax_default_prng_impl and
jax_random_seed_offset; jax_legacy_prng_key governs raw uint32 keys;
jax_use_high_dynamic_range_gumbel picks random_gumbel's default mode;
jax_accurate_erf_inv (R/lax_special.R:1324-1331) selects JAX's erf_inv_core for the normal
and truncated-normal samplers and lax_erf_inv.
"""

from __future__ import annotations

import contextlib
import os
import warnings

from .errors import JaxValueError

_DEFAULTS = {
    "jax_enable_x64": False,
    "jax_threefry_partitionable": True,
    "jax_default_prng_impl": "threefry2x32",
    "jax_random_seed_offset": 0,
    "jax_legacy_prng_key": "allow",
    "jax_use_high_dynamic_range_gumbel": False,
    "jax_accurate_erf_inv": False,
}

_config = dict(_DEFAULTS)


def _env_bool(name):
    v = os.environ.get(name)
    if v is None:
        return None
    return v.strip().lower() in ("1", "true", "yes", "on")


if _env_bool("JAX_ENABLE_X64") is not None:  # R/config.R:109-114
    _config["jax_enable_x64"] = _env_bool("JAX_ENABLE_X64")


def jax_config(name=None):
    """Value of option `name`, or a copy of all options."""
    if name is None:
        return dict(_config)
    if name not in _config:
        raise JaxValueError(f"Unrecognized config option: {name}")
    return _config[name]


def jax_config_update(name, value):
    """Set option `name`; returns the previous value."""
    if name not in _config:
        raise JaxValueError(f"Unrecognized config option: {name}")
    old = _config[name]
    if name in ("jax_enable_x64", "jax_threefry_partitionable",
                "jax_use_high_dynamic_range_gumbel", "jax_accurate_erf_inv"):
        value = bool(value)
    if name == "jax_legacy_prng_key" and value not in ("allow", "warn", "error"):
        raise JaxValueError("jax_legacy_prng_key must be one of 'allow', 'warn', 'error'")
    _config[name] = value
    return old


@contextlib.contextmanager
def with_jax_config(name, value):
    """Run a block with option `name` set to `value`."""
    old = jax_config_update(name, value)
    try:
        yield
    finally:
        _config[name] = old


def enable_x64(flag=True):
    """Turn 64-bit mode on or off; returns the previous setting."""
    return jax_config_update("jax_enable_x64", flag)


def x64_enabled():
    return bool(_config["jax_enable_x64"])


def partitionable():
    return bool(_config["jax_threefry_partitionable"])


def legacy_key_mode():
    return _config["jax_legacy_prng_key"]


def warn_legacy(msg):
    warnings.warn(msg, stacklevel=3)
