# jxrng for jaxR: the eager threefry2x32 path of random_bits, random_split,
# random_fold_in, random_uniform, random_normal and random_bernoulli computed on a B200
# by libjxrng, through the .Call shim in jxrng_r.c.
#
# Install: add this file to jaxR's R/ collated after prng.R and random.R (e.g. as
# R/zz_jxrng.R), build jxrngR.so (see jxrng_r.c) and call jxrng_attach() from .onLoad
# when $JXRNG_DIR names this directory's parent.  The public API does not change.
#
# Each replaced function keeps jaxR's own as `jaxr_<name>` and takes the shim only for a
# concrete (not traced) threefry2x32 key and the arguments the shim covers; everything
# else -- values traced by jit, vmap or grad, rbg keys, complex normals, array bounds,
# bernoulli mode "high" -- runs jaxR's own code, unchanged.  The key-reuse checker sees
# the same consumption as in jaxR: kr_sink(key, "random_bits") before every draw and
# kr_sink(key, "random_split") before a split, as prng_bits_jit and prng_split_jit do
# (R/prng.R:524, :533); new keys go through prng_key_array (kr_init).

.jxrng <- new.env(parent = emptyenv())

jxrng_dtype_codes <- c(float32 = 0L, float64 = 1L, float16 = 2L, bfloat16 = 3L)

# Loads jxrngR.so (linked to libjxrng.so), looks its routines up, and builds the samplers'
# lookup tables on the current GPU (jxr_prepare_device; 63 = every table).
jxrng_attach <- function(dir = Sys.getenv("JXRNG_DIR")) {
  so <- file.path(dir, "r", paste0("jxrngR", .Platform$dynlib.ext))
  if (!nzchar(dir) || !file.exists(so)) return(invisible(FALSE))
  dll <- dyn.load(so)
  for (nm in c("jxr_r_random_bits", "jxr_r_uniform", "jxr_r_normal", "jxr_r_bernoulli",
               "jxr_r_split", "jxr_r_fold_in", "jxr_r_prepare"))
    .jxrng[[nm]] <- getNativeSymbolInfo(nm, dll)
  .Call(.jxrng$jxr_r_prepare, 63L)
  .jxrng$on <- TRUE
  invisible(TRUE)
}

jxrng_on <- function() isTRUE(.jxrng$on) && !isFALSE(.jx$config$jax_jxrng)

jxrng_layout <- function() as.integer(isTRUE(.jx$config$jax_threefry_partitionable))

# A concrete, unbatched jax array (not a tracer).
jxrng_concrete <- function(x) inherits(x, "jax_array") && !is_tracer(x)

# The two key words of a concrete threefry2x32 key as doubles, or NULL when the shim does
# not apply (traced or batched key, other implementation, shim not attached).
jxrng_key_words <- function(key) {
  if (!jxrng_on() || !is_prng_key(key) ||
      !identical(attr(key, "impl", exact = TRUE), "threefry2x32"))
    return(NULL)
  d <- key$data
  if (!jxrng_concrete(d) || !identical(aval_of(d)$shape, 2L)) return(NULL)
  as.numeric(array_host(d))
}

# A scalar parameter as a double: an R number or a concrete 0-d jax array, else NULL.
jxrng_scalar <- function(x) {
  if (is.numeric(x) && !is_jax_value(x) && length(x) == 1L && !is.na(x)) return(as.numeric(x))
  if (jxrng_concrete(x) && length(aval_of(x)$shape) == 0L) return(as.numeric(array_host(x)))
  NULL
}

jxrng_u32_array <- function(v, shape) new_array(new_aval(shape, "uint32"), host = c_unravel(v, shape))

# doubles from the shim -> a jax array of dtype dt (16-bit floats arrive as bit patterns)
jxrng_float_array <- function(v, shape, dt) {
  if (dt %in% c("float16", "bfloat16"))
    return(lax_bitcast_convert_type(new_array(new_aval(shape, "uint16"), host = c_unravel(v, shape)), dt))
  new_array(new_aval(shape, dt), host = c_unravel(v, shape))
}

# ---- R/prng.R:537-541 ----------------------------------------------------------------------

jaxr_prng_random_bits <- prng_random_bits
prng_random_bits <- function(key, bit_width, shape) {
  w <- jxrng_key_words(key)
  if (is.null(w)) return(jaxr_prng_random_bits(key, bit_width, shape))
  kr_sink(key, "random_bits")
  bit_width <- as.integer(bit_width)
  prng_check_bit_width(bit_width)
  shape <- as.integer(shape)
  size <- prod(as.numeric(shape))
  if (size > 2^64)
    jax_error("random bits array of size exceeding 2 ** 64", class = "jax_not_implemented_error")
  dt <- prng_uint_dtypes[[as.character(bit_width)]]
  v <- .Call(.jxrng$jxr_r_random_bits, w, size, jxrng_layout(), bit_width)
  if (bit_width == 64L) {  # join the 32-bit halves as R/prng.R:220-224 does
    hi <- lax_convert_element_type(jxrng_u32_array(v[[1L]], shape), dt)
    lo <- lax_convert_element_type(jxrng_u32_array(v[[2L]], shape), dt)
    return(lax_bitwise_or(lax_shift_left(hi, prng_const(hi, 32)), lo))
  }
  new_array(new_aval(shape, dt), host = c_unravel(v, shape))
}

jaxr_prng_random_split <- prng_random_split
prng_random_split <- function(key, shape) {
  w <- jxrng_key_words(key)
  if (is.null(w)) return(jaxr_prng_random_split(key, shape))
  kr_sink(key, "random_split")
  shape <- as.integer(shape)
  v <- .Call(.jxrng$jxr_r_split, w, prod(as.numeric(shape)), jxrng_layout())
  prng_key_array(jxrng_u32_array(v, c(shape, 2L)), "threefry2x32")
}

jaxr_prng_random_fold_in <- prng_random_fold_in
prng_random_fold_in <- function(key, data) {
  w <- jxrng_key_words(key)
  d <- if (is.null(w)) NULL else jxrng_scalar(data)
  if (is.null(d)) return(jaxr_prng_random_fold_in(key, data))
  v <- .Call(.jxrng$jxr_r_fold_in, w, d)
  prng_key_array(jxrng_u32_array(v, 2L), "threefry2x32")
}

# ---- R/random.R:288-304, :502-508, :656-666 ------------------------------------------------

jaxr_rnd_uniform <- rnd_uniform
rnd_uniform <- function(key, minval, maxval, shape, dtype) {
  w <- jxrng_key_words(key)
  lo <- jxrng_scalar(minval)
  hi <- jxrng_scalar(maxval)
  if (is.null(w) || is.null(lo) || is.null(hi) || !dtype %in% names(jxrng_dtype_codes))
    return(jaxr_rnd_uniform(key, minval, maxval, shape, dtype))
  kr_sink(key, "random_bits")
  shape <- as.integer(shape)
  v <- .Call(.jxrng$jxr_r_uniform, w, prod(as.numeric(shape)), jxrng_layout(),
             jxrng_dtype_codes[[dtype]], lo, hi)
  jxrng_float_array(v, shape, dtype)
}

jaxr_rnd_normal_real <- rnd_normal_real
rnd_normal_real <- function(key, shape, dtype) {
  w <- jxrng_key_words(key)
  if (is.null(w) || !dtype %in% names(jxrng_dtype_codes))
    return(jaxr_rnd_normal_real(key, shape, dtype))
  kr_sink(key, "random_bits")
  shape <- as.integer(shape)
  v <- .Call(.jxrng$jxr_r_normal, w, prod(as.numeric(shape)), jxrng_layout(),
             jxrng_dtype_codes[[dtype]], isTRUE(.jx$config$jax_accurate_erf_inv))
  jxrng_float_array(v, shape, dtype)
}

jaxr_rnd_bernoulli <- rnd_bernoulli
rnd_bernoulli <- function(key, p, shape, mode) {
  w <- jxrng_key_words(key)
  pv <- if (is.null(w) || mode != "low") NULL else jxrng_scalar(p)
  dt <- if (is.null(pv)) NULL else aval_of(p)$dtype
  if (is.null(pv) || !dt %in% names(jxrng_dtype_codes))
    return(jaxr_rnd_bernoulli(key, p, shape, mode))
  if (is.null(shape)) shape <- integer(0) else rnd_check_shape("bernoulli", shape, integer(0))
  kr_sink(key, "random_bits")
  shape <- as.integer(shape)
  v <- .Call(.jxrng$jxr_r_bernoulli, w, prod(as.numeric(shape)), jxrng_layout(),
             jxrng_dtype_codes[[dt]], pv)
  new_array(new_aval(shape, "bool"), host = c_unravel(v, shape))
}
