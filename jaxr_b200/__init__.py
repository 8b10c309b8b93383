"""jaxr_b200: jaxR's threefry2x32 random-bits path on B200 (sm_100a).

The public functions mirror the reference's R API (R/random.R, R/prng.R); see
jaxr_b200.random.  The kernels live in libjxrng.so behind the C ABI of
include/jxrng.h; jaxr_b200.build compiles it.
"""

from . import config
from .config import enable_x64, jax_config, jax_config_update, with_jax_config
from .errors import (JaxError, JaxNotImplementedError, JaxOverflowError, JaxTypeError,
                     JaxValueError)
from .random import (PRNGKeyArray, canonicalize_dtype, dtype, free_caches, lax_erf_inv, lax_RandomAlgorithm,
                     lax_rng_bit_generator, random_bernoulli,
                     random_bits, random_choice, random_clone, random_exponential,
                     random_fold_in, random_gumbel, random_Key, random_key, random_key_data,
                     random_key_dtype, random_key_impl, random_laplace, random_logistic,
                     random_normal, random_normal_bernoulli, random_permutation,
                     random_PRNGKey, random_randint, random_split, random_truncated_normal,
                     random_uniform, random_wrap_key_data, threefry2x32, threefry_2x32, vmap)

__all__ = [
    "config", "enable_x64", "jax_config", "jax_config_update", "with_jax_config", "JaxError",
    "JaxNotImplementedError", "JaxOverflowError", "JaxTypeError", "JaxValueError",
    "PRNGKeyArray", "canonicalize_dtype", "dtype", "free_caches", "lax_erf_inv", "lax_RandomAlgorithm",
    "lax_rng_bit_generator", "random_bernoulli",
    "random_bits", "random_choice", "random_clone", "random_exponential", "random_fold_in",
    "random_gumbel", "random_Key", "random_key", "random_key_data", "random_key_dtype",
    "random_key_impl", "random_laplace", "random_logistic", "random_normal",
    "random_normal_bernoulli", "random_permutation", "random_PRNGKey", "random_randint",
    "random_split", "random_truncated_normal", "random_uniform", "random_wrap_key_data",
    "threefry2x32", "threefry_2x32", "vmap",
]
