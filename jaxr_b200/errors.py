"""Error classes of the reference (jax_error(..., class = ...), R/aaa_state.R:19-22).

Each is also the matching Python builtin, so `except TypeError` catches a
jax_type_error as R code catches the condition class.
"""


class JaxError(Exception):
    """jax_error"""


class JaxTypeError(JaxError, TypeError):
    """jax_type_error"""


class JaxValueError(JaxError, ValueError):
    """jax_value_error"""


class JaxOverflowError(JaxError, OverflowError):
    """jax_overflow_error"""


class JaxNotImplementedError(JaxError, NotImplementedError):
    """jax_not_implemented_error"""
