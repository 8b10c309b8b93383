"""jax.random's threefry path with jaxR's interface, on sm_100a kernels.

Host-side mirror of the reference's R API (R/random.R, R/prng.R): same function
names, argument meanings, defaults, dtype rules and error messages/classes.  Arrays
are torch tensors on the current CUDA device (torch is plumbing here: device memory
and streams); every value is computed by libjxrng (include/jxrng.h).  There is no
CPU path.

Shapes are C order, as in the reference; uint32/uint64 results are torch.uint32 /
torch.uint64 tensors, bool results torch.bool.
"""

from __future__ import annotations

import functools
import math
import numbers
import warnings

import numpy as np
import torch

from . import _native as nat
from . import config as cfg
from .errors import (JaxNotImplementedError, JaxOverflowError, JaxTypeError, JaxValueError)

# ---- dtypes -------------------------------------------------------------------------------

_TORCH = {
    "bool": torch.bool, "uint8": torch.uint8, "uint16": torch.uint16, "uint32": torch.uint32,
    "uint64": torch.uint64, "int8": torch.int8, "int16": torch.int16, "int32": torch.int32,
    "int64": torch.int64, "float16": torch.float16, "bfloat16": torch.bfloat16,
    "float32": torch.float32, "float64": torch.float64, "complex64": torch.complex64,
    "complex128": torch.complex128,
}
_NAME = {v: k for k, v in _TORCH.items()}
_BITS = {"uint8": 8, "uint16": 16, "uint32": 32, "uint64": 64, "int8": 8, "int16": 16,
         "int32": 32, "int64": 64, "float16": 16, "bfloat16": 16, "float32": 32, "float64": 64,
         "bool": 8, "complex64": 64, "complex128": 128}
_FLOAT_CODE = {"float32": nat.F32, "float64": nat.F64, "float16": nat.F16, "bfloat16": nat.BF16}
_NMANT = {"float32": 23, "float64": 52, "float16": 10, "bfloat16": 7}


def default_uint():
    return "uint64" if cfg.x64_enabled() else "uint32"


def default_float():
    return "float64" if cfg.x64_enabled() else "float32"


def default_int():
    return "int64" if cfg.x64_enabled() else "int32"


def canonicalize_dtype(dt):
    """A dtype name (or torch/numpy dtype, or 'float'/'int'/'uint'), canonicalised for the
    x64 setting as the reference's dtype() does (64-bit types become 32-bit with x64 off)."""
    if isinstance(dt, torch.dtype):
        name = _NAME[dt]
    elif isinstance(dt, np.dtype) or (isinstance(dt, type) and issubclass(dt, np.generic)):
        name = np.dtype(dt).name
    else:
        name = str(dt)
    alias = {"float": default_float(), "float_": default_float(), "double": default_float(),
             "numeric": default_float(), "int": default_int(), "integer": default_int(),
             "uint": default_uint(), "complex": "complex128" if cfg.x64_enabled() else "complex64",
             "logical": "bool", "bool_": "bool"}
    name = alias.get(name, name)
    if name not in _TORCH:
        raise JaxTypeError(f"Unsupported dtype {dt}")
    if not cfg.x64_enabled():
        name = {"uint64": "uint32", "int64": "int32", "float64": "float32",
                "complex128": "complex64"}.get(name, name)
    return name


def dtype(x):
    """dtype name of an array, key array or scalar (the reference's jaxR::dtype)."""
    if isinstance(x, PRNGKeyArray):
        return x.dtype
    if isinstance(x, torch.Tensor):
        return _NAME[x.dtype]
    if isinstance(x, np.ndarray):
        return canonicalize_dtype(x.dtype)
    if isinstance(x, bool):
        return "bool"
    if isinstance(x, numbers.Integral):
        return default_int()
    if isinstance(x, numbers.Real):
        return default_float()
    raise JaxTypeError(f"no dtype for {type(x).__name__}")


def _is_unsigned(dt):
    return dt.startswith("uint")


def _is_float(dt):
    return dt in _FLOAT_CODE


_cuda_ready = False


def _device():
    global _cuda_ready
    if not _cuda_ready:
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device: the threefry kernels run on an sm_100 GPU and "
                               "there is no CPU path")
        _cuda_ready = True
    return torch.device("cuda", torch.cuda.current_device())


# the current stream's handle without building a torch.cuda.Stream object per call
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream():
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return ctypes_stream(torch.cuda.current_stream())


def ctypes_stream(s):
    return s.cuda_stream


def _ptr(t):
    return t.data_ptr()


# Lookup tables that jxr_prepare_device has built in this process, per device index (bit
# masks of JXR_PREPARE_TABLE_*).  The library's sampling entry points only read tables; this
# host layer builds a sampler's tables the first time a request large enough to read them
# comes, outside CUDA graph capture (building allocates and waits for the stream).
_PREPARED = {}
_TABLE_MIN = {"float32": 1 << 22, "float16": 1 << 16, "bfloat16": 1 << 16}
_TABLE_BIT = {"normal": 1, "normal_accurate": 2, "exponential": 4, "gumbel": 8,
              "logistic": 16, "laplace": 32}


def _prepare_table(device, sampler, dt, n):
    if n < _TABLE_MIN.get(dt, 1 << 63):
        return
    if sampler == "normal" and cfg.jax_config("jax_accurate_erf_inv"):
        sampler = "normal_accurate"
    bit = _TABLE_BIT[sampler]
    done = _PREPARED.get(device.index, 0)
    if done & bit or torch.cuda.is_current_stream_capturing():
        return
    nat.call("jxr_prepare_device", bit, _stream())
    _PREPARED[device.index] = done | bit


def shape_str(s):
    """The reference's prng_shape_str: (5,), (2, 3), ()."""
    s = tuple(int(v) for v in s)
    if len(s) == 1:
        return f"({s[0]},)"
    return "(" + ", ".join(str(v) for v in s) + ")"


def canon_shape(shape):
    """Shape argument to a tuple of non-negative ints (R/lax_shape.R:16-28)."""
    if type(shape) is tuple and all(type(v) is int and v >= 0 for v in shape):
        return shape
    if shape is None:
        return ()
    if isinstance(shape, torch.Tensor):
        shape = shape.tolist()
    if isinstance(shape, numbers.Integral):
        shape = (shape,)
    try:
        out = tuple(shape)
    except TypeError:
        raise JaxTypeError(f"Shapes must be 1D sequences of concrete values of integer type, "
                           f"got {shape!r}.")
    for v in out:
        if not isinstance(v, numbers.Integral) and not (isinstance(v, float) and v == int(v)):
            raise JaxTypeError(f"Shapes must be 1D sequences of concrete values of integer type, "
                               f"got {shape_str(out)}.")
        if v < 0:
            raise JaxTypeError(f"Shapes must be 1D sequences of concrete values of integer type, "
                               f"got {shape_str(out)}.")
    return tuple(int(v) for v in out)


def _size(shape):
    return math.prod(shape) if shape else 1


# ---- vmap batching --------------------------------------------------------------------------

class _Batched:
    """A value inside vmap: `value` carries `nb` leading batch axes that the function body
    does not see (R/batching.R:4-50 for the reference's batch trace)."""

    __slots__ = ("value", "nb")

    def __init__(self, value, nb):
        self.value = value
        self.nb = nb

    @property
    def batch_shape(self):
        v = self.value
        s = v.shape if isinstance(v, PRNGKeyArray) else tuple(v.shape)
        return tuple(s[:self.nb])

    @property
    def shape(self):
        v = self.value
        s = v.shape if isinstance(v, PRNGKeyArray) else tuple(v.shape)
        return tuple(s[self.nb:])

    def __repr__(self):
        return f"Batched({self.value!r}, batch axes={self.nb})"


def _unbatch(x):
    if isinstance(x, _Batched):
        return x.value, x.nb
    return x, 0


def _rebatch(x, nb):
    return _Batched(x, nb) if nb else x


def vmap(fun, in_axes=0, out_axes=0):
    """Vectorise `fun` over the leading axis of its arguments (R/batching.R).

    Inside `fun`, key arrays, raw keys, seeds and fold_in data carry the batch; the
    random functions run one key-batched kernel launch for the whole batch, which is
    what the reference's batching rule for threefry2x32 (lax_broadcast_batcher,
    R/prng.R:99) amounts to.  in_axes is 0 (batch every argument), None, or a
    sequence of 0/None per argument; out_axes must be 0.
    """
    if out_axes != 0:
        raise JaxValueError("vmap: only out_axes = 0 is supported")

    def wrapped(*args):
        axes = in_axes if isinstance(in_axes, (list, tuple)) else [in_axes] * len(args)
        if len(axes) != len(args):
            raise JaxValueError("vmap in_axes must have one entry per argument")
        level = 1 + max([a.nb for a in args if isinstance(a, _Batched)], default=0)
        sizes = set()
        bargs = []
        for a, ax in zip(args, axes):
            if ax is None:
                bargs.append(a)
                continue
            if ax != 0:
                raise JaxValueError("vmap: in_axes must be 0 or None")
            v, nb = _unbatch(a)
            if isinstance(v, (numbers.Number, np.generic)) or (
                    not isinstance(v, PRNGKeyArray) and not isinstance(v, torch.Tensor)):
                v = torch.as_tensor(np.asarray(v))
            vs = v.shape if isinstance(v, PRNGKeyArray) else tuple(v.shape)
            if len(vs) <= nb:
                raise JaxValueError("vmap was requested to map its argument along axis 0, "
                                    "which implies that its rank should be at least 1, but is only 0")
            sizes.add(vs[nb])
            bargs.append(_Batched(v, nb + 1))
        if len(sizes) > 1:
            raise JaxValueError(f"vmap got inconsistent sizes for the mapped axis: {sorted(sizes)}")
        out = fun(*bargs)
        size = sizes.pop() if sizes else None
        return _vmap_out(out, level, size)

    return wrapped


def _vmap_out(out, level, size):
    if isinstance(out, (list, tuple)):
        return type(out)(_vmap_out(o, level, size) for o in out)
    if isinstance(out, _Batched):
        if out.nb != level:
            raise JaxValueError("vmap: output batched at an unexpected level")
        return _rebatch(out.value, level - 1)
    # an output that does not depend on the mapped arguments is broadcast
    if size is None:
        return out
    if isinstance(out, PRNGKeyArray):
        return PRNGKeyArray(out.data.unsqueeze(0).expand((size,) + tuple(out.data.shape)).contiguous(),
                            out.impl)
    t = torch.as_tensor(out)
    return t.unsqueeze(0).expand((size,) + tuple(t.shape)).contiguous()


# ---- key arrays (R/prng.R:455-584) ----------------------------------------------------------

_IMPLS = {"threefry2x32": "fry", "rbg": "rbg", "unsafe_rbg": "urbg"}
_KEY_WORDS = {"threefry2x32": 2, "rbg": 4, "unsafe_rbg": 4}  # key_shape (R/prng.R:430-440)
_IMPL_CODE = {"threefry2x32": 0, "rbg": 1, "unsafe_rbg": 2}


class PRNGKeyArray:
    """A typed key array: uint32 key data of shape (*shape, 2) for threefry2x32 and
    (*shape, 4) for rbg and unsafe_rbg."""

    __slots__ = ("data", "impl")

    def __init__(self, data, impl="threefry2x32"):
        self.data = data
        self.impl = impl

    @property
    def shape(self):
        return tuple(self.data.shape[:-1])

    @property
    def ndim(self):
        return len(self.shape)

    @property
    def dtype(self):
        return f"key<{_IMPLS[self.impl]}>"

    def __len__(self):
        if not self.shape:
            raise JaxTypeError("len() of unsized object")
        return self.shape[0]

    def __getitem__(self, idx):
        if not isinstance(idx, tuple):
            idx = (idx,)
        if len(idx) > self.ndim:
            raise IndexError("too many indices for key array")
        return PRNGKeyArray(self.data[idx], self.impl)

    def __iter__(self):
        if not self.shape:
            raise JaxTypeError("iteration over a 0-d key array")
        return iter([PRNGKeyArray(self.data[i], self.impl) for i in range(self.shape[0])])

    def as_list(self):
        return list(iter(self))

    def __repr__(self):
        return f"Array({shape_str(self.shape)}, dtype={self.dtype}) overlaying:\n{self.data!r}"


def _resolve_impl(spec):
    """R/prng.R:444-453."""
    if spec is None:
        spec = cfg.jax_config("jax_default_prng_impl")
    if not isinstance(spec, str):
        raise JaxTypeError(f"unrecognized type {type(spec).__name__} for specifying PRNG "
                           "implementation.")
    name = spec
    for impl, tag in _IMPLS.items():
        if spec == f"key<{tag}>":
            name = impl
    if name not in _IMPLS:
        names = ", ".join(f'"{n}"' for n in _IMPLS)
        raise JaxValueError(f'unrecognized PRNG implementation "{spec}". Did you mean one of: '
                            f"{names}?")
    return name


def _as_uint32_data(x, impl="threefry2x32"):
    """Raw key data to a uint32 device tensor, checked as _check_prng_key_data
    (R/prng.R:478-492) for implementation `impl`."""
    if isinstance(x, torch.Tensor):
        t = x
        dt = _NAME[t.dtype]
    else:
        arr = np.asarray(x)
        if arr.dtype.kind == "f":
            dt = default_float()
        elif arr.dtype.kind in "iu":
            dt = canonicalize_dtype(arr.dtype) if arr.dtype != np.uint32 else "uint32"
            if arr.dtype.kind == "i" and arr.dtype != np.int64:
                dt = canonicalize_dtype(arr.dtype)
        elif arr.dtype.kind == "b":
            dt = "bool"
        else:
            raise JaxTypeError(f"unexpected PRNG key type {type(x).__name__}")
        t = None
    shape = tuple(t.shape) if t is not None else np.asarray(x).shape
    if len(shape) < 1:
        raise JaxTypeError("JAX encountered invalid PRNG key data: expected key_data.ndim >= 1; "
                           f"got ndim={len(shape)}")
    kw = _KEY_WORDS[impl]
    if shape[-1] != kw:
        raise JaxTypeError("JAX encountered invalid PRNG key data: expected key_data.shape to end "
                           f"with ({kw},); got shape={shape_str(shape)} for impl={impl}")
    if dt != "uint32":
        raise JaxTypeError("JAX encountered invalid PRNG key data: expected key_data.dtype = "
                           f"uint32; got dtype={dt}")
    if t is None:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(x), dtype=np.uint32))
    return t


def _legacy_check():
    msg = ("Legacy uint32 key array passed as key to jax.random function. Please create keys "
           "using jax.random.key(). If use of a raw key array was intended, set "
           'jax_legacy_prng_key="allow".')
    mode = cfg.legacy_key_mode()
    if mode == "error":
        raise JaxValueError(msg)
    if mode == "warn":
        warnings.warn(msg, stacklevel=4)


def _check_key(name, key, allow_batched=False):
    """R/random.R:55-77: (typed key, wrapped, batch axes)."""
    key, nb = _unbatch(key)
    if isinstance(key, PRNGKeyArray):
        k, wrapped = key, False
    elif isinstance(key, (torch.Tensor, np.ndarray, list, tuple, numbers.Number)) and not isinstance(key, str):
        _legacy_check()
        impl = _resolve_impl(None)  # raw keys use the default implementation
        k, wrapped = PRNGKeyArray(_as_uint32_data(key, impl), impl), True
    else:
        raise JaxTypeError(f"unexpected PRNG key type {type(key).__name__}")
    per_shape = k.shape[nb:]
    if not allow_batched and per_shape:
        raw = tuple(k.data.shape[nb:]) if wrapped else per_shape
        raise JaxValueError(f"{name} accepts a single key, but was given a key array of shape "
                            f"{shape_str(raw)} != (). Use jax.vmap for batching.")
    return k, wrapped, nb


def _return_keys(wrapped, key):
    return key.data if wrapped else key


def _layout():
    return nat.LAYOUT_PARTITIONABLE if cfg.partitionable() else nat.LAYOUT_ORIGINAL


# ---- seeds (R/prng.R:159-170, :501-519) --------------------------------------------------------

def _seed_words(seed):
    """(k0, k1) uint32 numpy arrays of the keys of integer seeds (R/prng.R:159-170).

    An R number (here a Python/numpy number) is an int64 that wraps to int32 with x64
    off (R/prng.R:505-514); an integer array keeps its width, canonicalised for x64.
    jax_random_seed_offset is added first (R/prng.R:516-517).  k0 is the seed shifted
    right by 32, which is 0 for 32-bit seeds; k1 is its low word.
    """
    x64 = cfg.x64_enabled()
    off = int(cfg.jax_config("jax_random_seed_offset") or 0)
    if isinstance(seed, torch.Tensor):
        dt = _NAME[seed.dtype]
        if not dt.startswith(("int", "uint")):
            raise JaxTypeError(f"PRNG key seed must be an integer; got {seed.tolist()}")
        wide = _BITS[dt] == 64 and x64
        vals = [int(v) + off for v in np.asarray(seed.detach().cpu().reshape(-1).tolist(),
                                                 dtype=object)]
        shape = tuple(seed.shape)
    else:
        arr = np.asarray(seed)
        if arr.dtype.kind == "f":
            if not np.all(arr == np.round(arr)):
                raise JaxTypeError(f"PRNG key seed must be an integer; got {seed}")
        elif arr.dtype.kind not in "iu":
            raise JaxTypeError(f"PRNG key seed must be an integer; got {seed}")
        wide = x64
        vals = [int(v) + off for v in arr.reshape(-1).tolist()]
        shape = arr.shape
    mod = 1 << (64 if wide else 32)
    v = np.array([x % mod for x in vals], dtype=np.uint64).reshape(shape)
    k0 = (v >> np.uint64(32)).astype(np.uint32)
    k1 = (v & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    return k0, k1


def _keys_from_seeds(seed):
    k0, k1 = _seed_words(seed)
    data = np.stack([k0, k1], axis=-1).astype(np.uint32)
    return torch.from_numpy(np.ascontiguousarray(data)).to(_device())


def _key_ctor(ctor, seed, impl_spec):
    impl = _resolve_impl(impl_spec)
    s, nb = _unbatch(seed)
    if isinstance(s, PRNGKeyArray):
        raise JaxTypeError(f"{ctor} accepts a scalar seed, but was given a PRNG key.")
    sshape = tuple(s.shape) if isinstance(s, (torch.Tensor, np.ndarray)) else np.shape(s)
    if len(sshape) > nb:
        raise JaxTypeError(f"{ctor} accepts a scalar seed, but was given an array of shape "
                           f"{shape_str(sshape[nb:])} != (). Use jax.vmap for batching")
    if not isinstance(s, (torch.Tensor, np.ndarray, numbers.Number)):
        raise JaxTypeError(f"PRNG key seed must be an integer; got {s!r}")
    data = _keys_from_seeds(s)
    if _KEY_WORDS[impl] == 4:  # rbg seed: the threefry seed twice (R/prng.R:385-388)
        data = torch.cat([data, data], dim=-1)
    return _rebatch(PRNGKeyArray(data, impl), nb)


def random_key(seed, impl=None, dtype=None):
    """A typed key from an integer seed (R/random.R:169-189)."""
    if dtype is not None:
        if impl is not None:
            raise JaxValueError("Cannot specify both `impl` and `dtype` arguments to "
                                "jax.random.key")
        impl = dtype
    return _key_ctor("key", seed, impl)


def random_PRNGKey(seed, impl=None):
    """A legacy raw key: uint32 data of shape (2,) (R/random.R:191-193)."""
    k = _key_ctor("PRNGKey", seed, impl)
    kv, nb = _unbatch(k)
    return _rebatch(kv.data, nb)


def random_key_data(keys):
    k, _, nb = _check_key("key_data", keys, allow_batched=True)
    return _rebatch(k.data, nb)


def random_key_impl(keys):
    k, _, _ = _check_key("key_impl", keys, allow_batched=True)
    return k.impl


def random_key_dtype(impl_spec=None):
    if impl_spec is not None and impl_spec not in _IMPLS and not str(impl_spec).startswith("key<"):
        _resolve_impl(impl_spec)
    name = impl_spec if impl_spec in _IMPLS else (impl_spec and next(
        (n for n, t in _IMPLS.items() if impl_spec == f"key<{t}>"), None))
    if name is None:
        name = cfg.jax_config("jax_default_prng_impl")
    return f"key<{_IMPLS[name]}>"


def random_wrap_key_data(key_bits_array, impl=None, dtype=None):
    if dtype is not None:
        if impl is not None:
            raise JaxValueError("Cannot specify both `impl` and `dtype` arguments to "
                                "jax.random.wrap_key_data")
        impl = dtype
    name = _resolve_impl(impl)
    kb, nb = _unbatch(key_bits_array)
    return _rebatch(PRNGKeyArray(_as_uint32_data(kb, name), name), nb)


def random_clone(key):
    if not isinstance(key, PRNGKeyArray):
        return key
    return PRNGKeyArray(key.data.clone(), key.impl)


def random_Key(x):
    return x


# ---- kernels on flat key batches -------------------------------------------------------------

def _flat_keys(k):
    """Key data as a contiguous (nkeys, 2) (threefry2x32) or (nkeys, 4) (rbg, unsafe_rbg)
    uint32 tensor on the current device."""
    d = k.data
    if d.is_cuda and d.is_contiguous() and d.get_device() == torch.cuda.current_device():
        return d.view(-1, _KEY_WORDS[k.impl])
    return d.to(_device()).reshape(-1, _KEY_WORDS[k.impl]).contiguous()


def _is_rbg(kd):
    return kd.shape[-1] == 4


def _k_split(kd, shape, layout, impl="threefry2x32"):
    """split of every key of kd into _size(shape) keys: (nkeys, num, key words)."""
    n = kd.shape[0]
    num = _size(shape)
    if impl == "threefry2x32":
        out = torch.empty((n, num, 2), dtype=torch.uint32, device=kd.device)
        nat.call("jxr_split", _ptr(kd), n, num, layout, _ptr(out), _stream())
        return out
    out = torch.empty((n, num, 4), dtype=torch.uint32, device=kd.device)
    if not n * num:
        return out
    if impl == "rbg":
        # each half split as a threefry key (R/prng.R:391-397); key j = (half 0's key j,
        # half 1's key j): the (2, num) halves of each key transposed to (num, 2)
        tmp = torch.empty((2 * n, num, 2), dtype=torch.uint32, device=kd.device)
        nat.call("jxr_split", _ptr(kd), 2 * n, num, layout, _ptr(tmp), _stream())
        m = np.arange(2 * num, dtype=np.int64)
        idx = torch.from_numpy(((m % 2) * num + m // 2).astype(np.uint32)).to(kd.device)
        nat.call("jxr_take", _ptr(tmp), n, 2 * num, _ptr(idx), 2 * num, 8, _ptr(out), None,
                 _stream())
        return out
    # unsafe_rbg (R/prng.R:415-420): rows 0, 10, 20, ... of rng_bit_generator(key, (10 num, 4));
    # batched keys all draw from the first key (the primitive's batching rule)
    nat.call("jxr_rbg_blocks", _ptr(kd[0]), 0, 10, n * num, _ptr(out), _stream())
    return out


def _k_fold_in(kd, data, impl="threefry2x32"):
    n = max(kd.shape[0], data.shape[0])
    if impl == "threefry2x32":
        out = torch.empty((n, 2), dtype=torch.uint32, device=kd.device)
        nat.call("jxr_fold_in", _ptr(kd), kd.shape[0], _ptr(data), data.shape[0], _ptr(out),
                 _stream())
        return out
    out = torch.empty((n, 4), dtype=torch.uint32, device=kd.device)
    if impl == "rbg":  # each half folded as a threefry key (R/prng.R:400-403)
        keys = kd.expand(n, 4).contiguous().reshape(2 * n, 2)
        d2 = data.expand(n).contiguous().repeat_interleave(2)
        nat.call("jxr_fold_in", _ptr(keys), 2 * n, _ptr(d2), 2 * n, _ptr(out), _stream())
        return out
    # unsafe_rbg (R/prng.R:423-426)
    nat.call("jxr_rbg_unsafe_fold_in", _ptr(kd), kd.shape[0], _ptr(data), data.shape[0],
             int(data.shape[0] > 1), _ptr(out), _stream())
    return out


def _check_size(size, layout):
    if size >= 1 << 64:
        raise JaxNotImplementedError("random bits array of size exceeding 2 ** 64")


def _k_bits(kd, size, bit_width, layout, shape=None):
    """(nkeys, size) random bits (allocated as `shape`, of as many elements, when given).
    rbg / unsafe_rbg keys draw from XLA's RngBitGenerator; batched keys of those all draw
    from the first key, (nkeys, size) of its stream (the primitive's batching rule,
    R/prng.R:309-320)."""
    _check_size(size, layout)
    out = torch.empty(shape if shape is not None else (kd.shape[0], size),
                      dtype=_TORCH[f"uint{bit_width}"], device=kd.device)
    if _is_rbg(kd):
        total = kd.shape[0] * size
        nat.call("jxr_rbg_bits", _ptr(kd[0]), total, 0, total, bit_width, _ptr(out), None,
                 _stream())
        return out
    nat.call("jxr_random_bits", _ptr(kd), kd.shape[0], size, 0, size, layout, bit_width,
             _ptr(out), _stream())
    return out


# bits per draw of the float samplers (R/random.R:288-299: bfloat16 uses 8 random bits)
_DRAW_BITS = {"float32": 32, "float64": 64, "float16": 16, "bfloat16": 8}


def _float_storage(dt):
    return torch.uint16 if dt in ("float16", "bfloat16") else _TORCH[dt]


def _as_float_view(t, dt):
    return t.view(_TORCH[dt]) if dt in ("float16", "bfloat16") else t


def _k_uniform(kd, size, dt, mn, mx, layout, flags=0, shape=None):
    _check_size(size, layout)
    out = torch.empty(shape if shape is not None else (kd.shape[0], size),
                      dtype=_float_storage(dt), device=kd.device)
    if _is_rbg(kd):
        bits = _k_bits(kd, size, _DRAW_BITS[dt], layout)
        nat.call("jxr_uniform_from_bits", _ptr(bits), bits.numel(), _FLOAT_CODE[dt], float(mn),
                 float(mx), flags, _ptr(out), _stream())
        return _as_float_view(out, dt)
    nat.call("jxr_uniform", _ptr(kd), kd.shape[0], size, 0, size, layout, _FLOAT_CODE[dt],
             float(mn), float(mx), flags, _ptr(out), _stream())
    return _as_float_view(out, dt)


def _k_normal(kd, size, dt, layout, shape=None):
    _check_size(size, layout)
    out = torch.empty(shape if shape is not None else (kd.shape[0], size),
                      dtype=_float_storage(dt), device=kd.device)
    _prepare_table(kd.device, "normal", dt, kd.shape[0] * size)
    if _is_rbg(kd):
        bits = _k_bits(kd, size, _DRAW_BITS[dt], layout)
        nat.call("jxr_normal_from_bits", _ptr(bits), bits.numel(), _FLOAT_CODE[dt], _ptr(out),
                 _stream())
        return _as_float_view(out, dt)
    nat.call("jxr_normal", _ptr(kd), kd.shape[0], size, 0, size, layout, _FLOAT_CODE[dt],
             _ptr(out), _stream())
    return _as_float_view(out, dt)


def _k_bernoulli(kd, size, dt, p, layout):
    _check_size(size, layout)
    out = torch.empty((kd.shape[0], size), dtype=torch.uint8, device=kd.device)
    if _is_rbg(kd):
        u = _k_uniform(kd, size, dt, 0.0, 1.0, layout)
        pt = _broadcast_param(torch.tensor(float(p), dtype=torch.float64), (size,), dt, "bernoulli")
        pt = pt.expand(kd.shape[0], size).contiguous()  # every key row in one launch
        nat.call("jxr_bernoulli_from_uniform", _ptr(_raw16(u.contiguous(), dt)), None,
                 _ptr(_raw16(pt, dt)), kd.shape[0] * size, _FLOAT_CODE[dt], _ptr(out), _stream())
        return out.view(torch.bool)
    nat.call("jxr_bernoulli", _ptr(kd), kd.shape[0], size, 0, size, layout, _FLOAT_CODE[dt],
             float(p), _ptr(out), _stream())
    return out.view(torch.bool)


# ---- threefry primitives (R/prng.R:88-120) ----------------------------------------------------

def _u32_tensor(x, what):
    if isinstance(x, torch.Tensor):
        return x
    return torch.as_tensor(np.asarray(x))


def threefry2x32(key1, key2, x1, x2):
    """The threefry2x32 primitive: uint32 arrays broadcast to one shape -> (x0, x1)
    (R/prng.R:88-99)."""
    args = [_u32_tensor(a, "arg") for a in (key1, key2, x1, x2)]
    if any(a.dtype != torch.uint32 for a in args):
        raise JaxTypeError("Arguments to threefry2x32 must have uint32 type, got "
                           + ", ".join(f"{_NAME[a.dtype]}{list(a.shape)}" for a in args))
    shape = torch.broadcast_shapes(*[a.shape for a in args])
    dev = _device()
    flat = [a.to(dev).broadcast_to(shape).contiguous().reshape(-1) for a in args]
    n = flat[0].numel()
    o0 = torch.empty(n, dtype=torch.uint32, device=dev)
    o1 = torch.empty(n, dtype=torch.uint32, device=dev)
    nat.call("jxr_threefry2x32", *[_ptr(f) for f in flat], _ptr(o0), _ptr(o1), n, _stream())
    return o0.reshape(shape), o1.reshape(shape)


def threefry_2x32(keypair, count):
    """prng_threefry_2x32: the Threefry-2x32 hash of a uint32 `count` array
    (R/prng.R:101-120)."""
    if isinstance(keypair, (list, tuple)) and len(keypair) == 2:
        k = [_u32_tensor(v, "key") for v in keypair]
    else:
        kt = _u32_tensor(keypair, "key")
        k = [kt[0], kt[1]]
    c = _u32_tensor(count, "count")
    dts = [_NAME[t.dtype] for t in (k[0], k[1], c)]
    if any(d != "uint32" for d in dts):
        raise JaxTypeError(f"threefry_2x32 requires uint32 arguments, got [{', '.join(dts)}]")
    dev = _device()
    kd = torch.stack([k[0].reshape(()), k[1].reshape(())]).to(dev).reshape(1, 2).contiguous()
    flat = c.to(dev).contiguous().reshape(-1)
    out = torch.empty_like(flat)
    nat.call("jxr_threefry_2x32", _ptr(kd), 1, _ptr(flat), flat.numel(), _ptr(out), _stream())
    return out.reshape(c.shape)


# ---- split / fold_in / bits (R/random.R:195-276) ---------------------------------------------

def random_split(key, num=2):
    """Split a key into `num` (an int or a shape) new keys (R/random.R:209-213)."""
    k, wrapped, nb = _check_key("split", key)
    shape = canon_shape(num)
    bshape = k.shape[:nb]
    out = _k_split(_flat_keys(k), shape, _layout(), k.impl).reshape(
        bshape + shape + (_KEY_WORDS[k.impl],))
    return _rebatch(_return_keys(wrapped, PRNGKeyArray(out, k.impl)), nb)


def _fold_data(data):
    d, nb = _unbatch(data)
    if isinstance(d, (torch.Tensor, np.ndarray)):
        dshape = tuple(d.shape)
        if len(dshape) > nb:
            raise JaxTypeError(f"fold_in accepts a scalar, but was given an array of shape "
                               f"{shape_str(dshape[nb:])} != (). Use jax.vmap for batching.")
        t = torch.as_tensor(d) if not isinstance(d, torch.Tensor) else d
        if t.dtype == torch.uint32:
            vals = t.reshape(-1)
        else:
            if t.dtype.is_floating_point:
                t = t.to(torch.int64)
            vals = (t.to(torch.int64).reshape(-1) & 0xFFFFFFFF).to(torch.uint32)
        return vals.to(_device()).contiguous(), dshape[:nb], nb
    if isinstance(d, (list, tuple)):
        raise JaxTypeError(f"fold_in accepts a scalar, but was given an array of shape "
                           f"{shape_str(np.shape(d))} != (). Use jax.vmap for batching.")
    if isinstance(d, numbers.Number):
        if not float(d) == int(d):
            raise JaxTypeError(f"fold_in data must be an integer; got {d}")
        v = int(d)
        if v < 0 or v >= 1 << 32:
            raise JaxOverflowError(f"Python integer {v} out of bounds for uint32")
        return torch.tensor([v], dtype=torch.uint32).to(_device()), (), 0
    raise JaxTypeError(f"fold_in data must be an integer; got {type(d).__name__}")


def random_fold_in(key, data):
    """Fold a 32-bit integer into a key (R/random.R:195-206)."""
    k, wrapped, knb = _check_key("fold_in", key)
    dvals, dbshape, dnb = _fold_data(data)
    kd = _flat_keys(k)
    kbshape = k.shape[:knb]
    nb = max(knb, dnb)
    if knb and dnb and kbshape != dbshape:
        raise JaxValueError("fold_in: key and data batch shapes differ")
    bshape = kbshape if knb >= dnb else dbshape
    out = _k_fold_in(kd, dvals, k.impl).reshape(bshape + (_KEY_WORDS[k.impl],))
    return _rebatch(_return_keys(wrapped, PRNGKeyArray(out, k.impl)), nb)


def random_bits(key, shape=(), dtype=None):
    """Uniform random bits of an unsigned dtype (R/random.R:269-276)."""
    k, _, nb = _check_key("bits", key)
    dt = default_uint() if dtype is None else canonicalize_dtype(dtype)
    if not _is_unsigned(dt):
        raise JaxValueError(f"dtype argument to `bits` must be an unsigned int dtype, got {dt}")
    shape = canon_shape(shape)
    out = _k_bits(_flat_keys(k), _size(shape), _BITS[dt], _layout(), k.shape[:nb] + shape)
    return _rebatch(out, nb)


# ---- uniform / normal / bernoulli (R/random.R:278-304, :466-508, :643-666) -------------------

def free_caches():
    """Frees the current device's library caches (the samplers' tables, 32 MiB each for
    float32, and the host-copy staging buffers); later calls rebuild what they need."""
    nat.call("jxr_free_caches")
    _PREPARED.pop(torch.cuda.current_device(), None)


def _uses_erf_inv(fn):
    """Runs `fn` with the library's erf_inv (a per-thread setting) set to the one that
    jax_accurate_erf_inv names (R/lax_special.R:1324-1331): chlo.erf_inv by default, JAX's
    erf_inv_core (R/lax_special.R:1022-1082) when the option is set.  The previous setting
    is restored on return, so other callers of the library on this thread see theirs."""
    @functools.wraps(fn)
    def wrapped(*args, **kwargs):
        lib = nat.lib()
        prev = lib.jxr_set_accurate_erf_inv(1 if cfg.jax_config("jax_accurate_erf_inv") else 0)
        try:
            return fn(*args, **kwargs)
        finally:
            lib.jxr_set_accurate_erf_inv(prev)
    return wrapped


def _float_dtype(name, dt, kind="a float"):
    d = canonicalize_dtype(dt if dt is not None else "float")
    ok = d in _FLOAT_CODE or (kind == "a float or complex" and d.startswith("complex"))
    if not ok:
        raise JaxValueError(f"dtype argument to `{name}` must be {kind} dtype, got {d}")
    return d


def _param(x, dt):
    """A bound or probability: a Python number (scalar) or an array converted to dt."""
    x, nb = _unbatch(x)
    if nb:
        raise JaxNotImplementedError("batched sampler parameters are not supported")
    if isinstance(x, numbers.Number) and not isinstance(x, bool):
        return float(x), None
    t = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x, dtype=np.float64))
    if t.ndim == 0:
        return float(t.item()), None
    return None, t


def _batch_rows(nb, kbshape, params, shape, dt, name):
    """Sampler parameters batched under vmap (the reference's vmap batches every primitive
    argument, R/batching.R:22-50): params are (value, batch axes) pairs.  Every batched
    value must carry the key's batch axes (or, with an unbatched key, all the same ones),
    which give the batch shape B.  Returns (levels, B, rows) with rows the parameters, each
    broadcast per lane to `shape` and laid out as a contiguous (prod(B), size) tensor of
    dt."""
    levels = max([nb] + [pb for _, pb in params])
    if any(pb not in (0, levels) for _, pb in params) or (nb not in (0, levels)):
        raise JaxNotImplementedError("vmap: sampler parameters batched at other levels than the key")
    bshapes = [tuple(v.shape[:pb]) for v, pb in params if pb]
    B = tuple(kbshape) if nb else bshapes[0]
    if any(b != B for b in bshapes):
        raise JaxValueError(f"vmap got inconsistent sizes for the mapped axis: {sorted(set(bshapes))}")
    nrows, size = _size(B), _size(shape)
    rows = []
    for v, pb in params:
        t = v if isinstance(v, torch.Tensor) else torch.as_tensor(np.asarray(v, dtype=np.float64))
        lane = tuple(t.shape[pb:])
        _check_param_shape(lane, shape, name)  # the per-lane shape rule
        t = t.to(torch.float64).to(_device()).to(_TORCH[dt])
        t = t.reshape((B if pb else ()) + (1,) * (len(shape) - len(lane)) + lane)
        rows.append(t.expand(B + tuple(shape)).reshape(nrows, size).contiguous())
    return levels, B, rows


def _check_param_shape(pshape, shape, name):
    try:
        b = torch.broadcast_shapes(tuple(pshape), shape)
    except RuntimeError:
        b = None
    if b != tuple(shape):
        raise JaxValueError(
            f"{name} parameter shapes must be broadcast-compatible with shape argument, and the "
            "result of broadcasting the shapes must equal the shape argument, but got result "
            f"{shape_str(b or tuple(pshape))} for shape argument {shape_str(shape)}.")


def _broadcast_param(t, shape, dt, name):
    _check_param_shape(t.shape, shape, name)
    # convert in double then to the dtype (one rounding), as lax_convert_element_type
    t64 = t.to(torch.float64).to(_device())
    conv = t64.to(_TORCH[dt])
    return conv.broadcast_to(shape).contiguous()


def _raw16(t, dt):
    return t.view(torch.uint16) if dt in ("float16", "bfloat16") else t


def random_uniform(key, shape=(), dtype=None, minval=0.0, maxval=1.0):
    """Uniform floats in [minval, maxval) (R/random.R:278-304)."""
    k, _, nb = _check_key("uniform", key)
    dt = _float_dtype("uniform", dtype)
    shape = canon_shape(shape)
    size = _size(shape)
    kd = _flat_keys(k)
    (mnv, mnb), (mxv, mxb) = _unbatch(minval), _unbatch(maxval)
    if mnb or mxb:  # bounds batched under vmap: one row of bounds per lane
        levels, B, (mn, mx) = _batch_rows(nb, k.shape[:nb], [(mnv, mnb), (mxv, mxb)], shape, dt,
                                          "uniform")
        unit = _k_uniform(kd, size, dt, 0.0, 1.0, _layout())
        if unit.shape[0] != mn.shape[0]:  # an unbatched key: every lane draws the same
            unit = unit.expand(mn.shape[0], size).contiguous()
        out = torch.empty_like(unit)
        nat.call("jxr_uniform_affine", _ptr(_raw16(unit, dt)), _ptr(_raw16(mn, dt)),
                 _ptr(_raw16(mx, dt)), unit.numel(), _FLOAT_CODE[dt], 0, _ptr(_raw16(out, dt)),
                 _stream())
        return _rebatch(out.reshape(B + shape), levels)
    mn_s, mn_t = _param(minval, dt)
    mx_s, mx_t = _param(maxval, dt)
    if mn_t is None and mx_t is None:
        return _rebatch(_k_uniform(kd, size, dt, mn_s, mx_s, _layout(), shape=k.shape[:nb] + shape),
                        nb)
    else:
        unit = _k_uniform(kd, size, dt, 0.0, 1.0, _layout())
        mn = _broadcast_param(mn_t if mn_t is not None else torch.tensor(mn_s), shape, dt, "uniform")
        mx = _broadcast_param(mx_t if mx_t is not None else torch.tensor(mx_s), shape, dt, "uniform")
        out = torch.empty_like(unit)
        # one launch for every key row, each with the same row of bounds
        nat.call("jxr_uniform_affine_rows", _ptr(_raw16(unit, dt)), _ptr(_raw16(mn, dt)),
                 _ptr(_raw16(mx, dt)), unit.shape[0], size, _FLOAT_CODE[dt], 0,
                 _ptr(_raw16(out, dt)), _stream())
    return _rebatch(out.reshape(k.shape[:nb] + shape), nb)


@_uses_erf_inv
def random_normal(key, shape=(), dtype=None):
    """Standard normal floats: sqrt(2) * erf_inv(u), u uniform in (-1, 1)
    (R/random.R:482-508)."""
    k, _, nb = _check_key("normal", key)
    dt = _float_dtype("normal", dtype, kind="a float or complex")
    shape = canon_shape(shape)
    size = _size(shape)
    bshape = k.shape[:nb]
    if dt.startswith("complex"):
        return _rebatch(_complex_normal(k, bshape, shape, dt), nb)
    return _rebatch(_k_normal(_flat_keys(k), size, dt, _layout(), bshape + shape), nb)


def _complex_normal(k, bshape, shape, dt):
    """(re + i im) / sqrt(2) with re, im normals of the two halves of split(key)
    (R/random.R:489-499)."""
    real = "float32" if dt == "complex64" else "float64"
    kd = _flat_keys(k)
    halves = _k_split(kd, (2,), _layout(), k.impl)  # (n, 2, key words)
    size = _size(shape)
    re = _k_normal(halves[:, 0].contiguous(), size, real, _layout())
    im = _k_normal(halves[:, 1].contiguous(), size, real, _layout())
    # complex / complex(sqrt 2, 0): each part divided by sqrt(2) in the real dtype
    z = torch.empty(re.shape, dtype=_TORCH[dt], device=re.device)
    nat.call("jxr_complex_from_parts", _ptr(re), _ptr(im), re.numel(), _FLOAT_CODE[real],
             math.sqrt(2), _ptr(z), _stream())
    return z.reshape(bshape + shape)


def random_bernoulli(key, p=0.5, shape=None, mode="low"):
    """Bernoulli draws uniform(dtype(p)) < p (R/random.R:643-666)."""
    if shape is not None:
        shape = canon_shape(shape)
    if mode not in ("high", "low"):
        raise JaxValueError(f"got mode='{mode}', expected 'high' or 'low'")
    k, _, nb = _check_key("bernoulli", key)
    pv, pnb = _unbatch(p)
    if isinstance(pv, bool) or (isinstance(pv, numbers.Integral)):
        raise JaxTypeError(f"bernoulli probability `p` must have a floating dtype, got "
                           f"{default_int()}.")
    if isinstance(pv, torch.Tensor):
        dt = _NAME[pv.dtype]
    elif isinstance(pv, np.ndarray):
        dt = canonicalize_dtype(pv.dtype)
    elif isinstance(pv, (list, tuple)):
        arr = np.asarray(pv)
        dt = default_float() if arr.dtype.kind == "f" else canonicalize_dtype(arr.dtype)
    else:
        dt = default_float()  # an R number: weak float of the default width
    if not _is_float(dt):
        raise JaxTypeError(f"bernoulli probability `p` must have a floating dtype, got {dt}.")
    if pnb:  # p batched under vmap: one row of p per lane
        dt = canonicalize_dtype(dt)  # an array of R numbers is float32 unless x64 is on
        if shape is None:
            shape = tuple(pv.shape[pnb:])
        size = _size(shape)
        kd = _flat_keys(k)
        levels, B, (pr,) = _batch_rows(nb, k.shape[:nb], [(pv, pnb)], shape, dt, "bernoulli")
        nrows = pr.shape[0]
        if mode == "low":
            lo = _k_uniform(kd, size, dt, 0.0, 1.0, _layout())
            hi = None
        else:
            u = _k_uniform(kd, 2 * size, dt, 0.0, 1.0, _layout()).reshape(kd.shape[0], 2, size)
            lo, hi = u[:, 0], u[:, 1]
        if lo.shape[0] != nrows:  # an unbatched key: every lane draws the same
            lo = lo.expand(nrows, size)
            hi = hi.expand(nrows, size) if hi is not None else None
        lo = _raw16(lo.contiguous(), dt)
        hi = _raw16(hi.contiguous(), dt) if hi is not None else None
        out = torch.empty((nrows, size), dtype=torch.uint8, device=kd.device)
        nat.call("jxr_bernoulli_from_uniform", _ptr(lo), _ptr(hi) if hi is not None else None,
                 _ptr(_raw16(pr, dt)), nrows * size, _FLOAT_CODE[dt], _ptr(out), _stream())
        return _rebatch(out.view(torch.bool).reshape(B + shape), levels)
    p_s, p_t = _param(p, dt)
    if shape is None:
        shape = () if p_t is None else tuple(p_t.shape)
    size = _size(shape)
    kd = _flat_keys(k)
    bshape = k.shape[:nb]
    layout = _layout()
    if mode == "low" and p_t is None:
        out = _k_bernoulli(kd, size, dt, p_s, layout)
        return _rebatch(out.reshape(bshape + shape), nb)
    pt = _broadcast_param(p_t if p_t is not None else torch.tensor(p_s), shape, dt, "bernoulli")
    n = size
    if mode == "low":
        u = _k_uniform(kd, size, dt, 0.0, 1.0, layout)
        lo, hi = u, None
    else:
        u = _k_uniform(kd, 2 * size, dt, 0.0, 1.0, layout).reshape(kd.shape[0], 2, size)
        lo, hi = u[:, 0], u[:, 1]
    out = torch.empty((kd.shape[0], size), dtype=torch.uint8, device=kd.device)
    # every key row in one launch: p repeated per row, the draws' rows made contiguous
    pt = pt.reshape(-1).expand(kd.shape[0], n).contiguous()
    lo_c = _raw16(lo.contiguous(), dt)
    hi_c = _raw16(hi.contiguous(), dt) if hi is not None else None
    nat.call("jxr_bernoulli_from_uniform", _ptr(lo_c), _ptr(hi_c) if hi_c is not None else None,
             _ptr(_raw16(pt, dt)), kd.shape[0] * n, _FLOAT_CODE[dt], _ptr(out), _stream())
    return _rebatch(out.view(torch.bool).reshape(bshape + shape), nb)


@_uses_erf_inv
def random_normal_bernoulli(key, p=0.5, shape=(), dtype=None):
    """(random_normal(key, shape, dtype), random_bernoulli(key, p, shape)) of one key in a
    single cipher pass; p is a Python float converted to dtype."""
    k, _, nb = _check_key("normal", key)
    dt = _float_dtype("normal", dtype)
    shape = canon_shape(shape)
    size = _size(shape)
    kd = _flat_keys(k)
    layout = _layout()
    _check_size(size, layout)
    if _is_rbg(kd):  # two passes over the same bits
        return random_normal(key, shape, dt), random_bernoulli(
            key, torch.tensor(float(p), dtype=_TORCH[dt]), shape)
    nout = torch.empty((kd.shape[0], size), dtype=_float_storage(dt), device=kd.device)
    bout = torch.empty((kd.shape[0], size), dtype=torch.uint8, device=kd.device)
    _prepare_table(kd.device, "normal", dt, kd.shape[0] * size)
    nat.call("jxr_normal_bernoulli", _ptr(kd), kd.shape[0], size, 0, size, layout,
             _FLOAT_CODE[dt], float(p), _ptr(nout), _ptr(bout), _stream())
    bshape = k.shape[:nb]
    return (_rebatch(_as_float_view(nout, dt).reshape(bshape + shape), nb),
            _rebatch(bout.view(torch.bool).reshape(bshape + shape), nb))


# ---- log-transform samplers (R/random.R:1420-1516) ------------------------------------------

_SAMPLE_KIND = {"exponential": 0, "gumbel": 1, "logistic": 2, "laplace": 3}


def _k_sample(kd, size, dt, kind, layout):
    _check_size(size, layout)
    out = torch.empty((kd.shape[0], size), dtype=_float_storage(dt), device=kd.device)
    _prepare_table(kd.device, kind, dt, kd.shape[0] * size)
    if _is_rbg(kd):
        bits = _k_bits(kd, size, _DRAW_BITS[dt], layout)
        nat.call("jxr_sample_from_bits", _ptr(bits), bits.numel(), _SAMPLE_KIND[kind],
                 _FLOAT_CODE[dt], _ptr(out), _stream())
        return _as_float_view(out, dt)
    nat.call("jxr_sample", _ptr(kd), kd.shape[0], size, 0, size, layout, _SAMPLE_KIND[kind],
             _FLOAT_CODE[dt], _ptr(out), _stream())
    return _as_float_view(out, dt)


def _log_sampler(kind, key, shape, dtype):
    k, _, nb = _check_key(kind, key)
    dt = _float_dtype(kind, dtype)
    shape = canon_shape(shape)
    out = _k_sample(_flat_keys(k), _size(shape), dt, kind, _layout())
    return _rebatch(out.reshape(k.shape[:nb] + shape), nb)


def random_exponential(key, shape=(), dtype=None):
    """Exponential(1) samples -log1p(-u), u uniform in [0, 1) (R/random.R:1420-1432)."""
    return _log_sampler("exponential", key, shape, dtype)


def random_laplace(key, shape=(), dtype=None):
    """Laplace(0, 1) samples sign(u) log1p(-|u|), u uniform in (-1, 1)
    (R/random.R:1492-1503)."""
    return _log_sampler("laplace", key, shape, dtype)


def random_logistic(key, shape=(), dtype=None):
    """Logistic samples log(x) - log1p(-x), x uniform in [tiny, 1) (R/random.R:1505-1516)."""
    return _log_sampler("logistic", key, shape, dtype)


def random_gumbel(key, shape=(), dtype=None, mode=None):
    """Gumbel samples (R/random.R:1434-1489).  mode "low" (the default unless
    jax_use_high_dynamic_range_gumbel is set) is -log(-log(u)), u uniform in [tiny, 1);
    "high" and "highest" (float32; other dtypes take "high") combine two draws for more
    dynamic range near u = 0."""
    k, _, nb = _check_key("gumbel", key)
    dt = _float_dtype("gumbel", dtype)
    shape = canon_shape(shape)
    if mode is None:
        mode = "high" if cfg.jax_config("jax_use_high_dynamic_range_gumbel") else "low"
    if mode not in ("highest", "high", "low"):
        raise JaxValueError(f"Must provide valid mode for gumbel got: {mode}")
    kd = _flat_keys(k)
    size = _size(shape)
    layout = _layout()
    if mode == "low":
        out = _k_sample(kd, size, dt, "gumbel", layout)
        return _rebatch(out.reshape(k.shape[:nb] + shape), nb)
    if dt == "float32" and mode == "highest":
        rows = _k_bits(kd, 2 * size, 32, layout).reshape(kd.shape[0], 2, size)
        code = 1
    else:
        rows = _raw16(_k_uniform(kd, 2 * size, dt, 0.0, 1.0, layout), dt).reshape(
            kd.shape[0], 2, size)
        code = 0
    out = torch.empty((kd.shape[0], size), dtype=_float_storage(dt), device=kd.device)
    if kd.shape[0] == 1:
        r0, r1 = rows[0, 0], rows[0, 1]
    else:  # every key row in one launch: the two draws of each row gathered
        r0, r1 = rows[:, 0].contiguous(), rows[:, 1].contiguous()
    nat.call("jxr_gumbel_rows", _ptr(r0), _ptr(r1), kd.shape[0] * size, code, _FLOAT_CODE[dt],
             _ptr(out), _stream())
    return _rebatch(_as_float_view(out, dt).reshape(k.shape[:nb] + shape), nb)


# ---- truncated normal (R/random.R:576-603) ---------------------------------------------------

@_uses_erf_inv
def random_truncated_normal(key, lower, upper, shape=None, dtype=None):
    """Normal samples truncated to (lower, upper): sqrt(2) erf_inv(u) with u uniform in
    [erf(lower / sqrt 2), erf(upper / sqrt 2)), clipped to the open interval
    (R/random.R:576-603).  Scalar bounds run in one fused kernel; array bounds
    (broadcast to `shape`) take the unit draw and a per-element transform."""
    if shape is not None:
        shape = canon_shape(shape)
    k, _, nb = _check_key("truncated_normal", key)
    dt = _float_dtype("truncated_normal", dtype)
    (lov, lob), (hiv, hib) = _unbatch(lower), _unbatch(upper)
    if lob or hib:  # bounds batched under vmap: one row of bounds per lane
        if shape is None:
            lane = lambda v, pb: tuple(np.shape(v))[pb:]  # noqa: E731
            shape = tuple(torch.broadcast_shapes(lane(lov, lob), lane(hiv, hib)))
        levels, B, (lo, hi) = _batch_rows(nb, k.shape[:nb], [(lov, lob), (hiv, hib)], shape, dt,
                                          "truncated_normal")
        unit = _k_uniform(_flat_keys(k), _size(shape), dt, 0.0, 1.0, _layout())
        if unit.shape[0] != lo.shape[0]:  # an unbatched key: every lane draws the same
            unit = unit.expand(lo.shape[0], unit.shape[1]).contiguous()
        out = torch.empty_like(unit)
        nat.call("jxr_truncated_normal_from_unit", _ptr(_raw16(unit, dt)), _ptr(_raw16(lo, dt)), 1,
                 _ptr(_raw16(hi, dt)), 1, unit.numel(), _FLOAT_CODE[dt], _ptr(_raw16(out, dt)),
                 _stream())
        return _rebatch(out.reshape(B + shape), levels)
    lo_s, lo_t = _param(lower, dt)
    hi_s, hi_t = _param(upper, dt)
    if shape is None:
        shape = tuple(torch.broadcast_shapes(
            tuple(lo_t.shape) if lo_t is not None else (),
            tuple(hi_t.shape) if hi_t is not None else ()))
    kd = _flat_keys(k)
    size = _size(shape)
    layout = _layout()
    bshape = k.shape[:nb]
    if lo_t is None and hi_t is None:
        _check_size(size, layout)
        out = torch.empty((kd.shape[0], size), dtype=_float_storage(dt), device=kd.device)
        if _is_rbg(kd):
            bits = _k_bits(kd, size, _DRAW_BITS[dt], layout)
            nat.call("jxr_truncated_normal_from_bits", _ptr(bits), bits.numel(), _FLOAT_CODE[dt],
                     float(lo_s), float(hi_s), _ptr(out), _stream())
        else:
            # large requests build the sampler's table for these bounds in the call (float32:
            # 2^23 floats of scratch from torch's allocator; 16-bit: 2 KiB)
            total = kd.shape[0] * size
            words = (1 << 23 if dt == "float32" and total >= _TRUNC_TABLE_MIN else
                     512 if dt in ("float16", "bfloat16") and total >= 1 << 16 else 0)
            big = words > 0
            scratch = torch.empty(words, dtype=torch.float32, device=kd.device)
            nat.call("jxr_truncated_normal_scratch", _ptr(kd), kd.shape[0], size, 0, size, layout,
                     _FLOAT_CODE[dt], float(lo_s), float(hi_s),
                     _ptr(scratch) if big else None, scratch.numel() * 4, _ptr(out), _stream())
        return _rebatch(_as_float_view(out, dt).reshape(bshape + shape), nb)
    lo = _broadcast_param(lo_t if lo_t is not None else torch.tensor(lo_s), shape, dt,
                          "truncated_normal")
    hi = _broadcast_param(hi_t if hi_t is not None else torch.tensor(hi_s), shape, dt,
                          "truncated_normal")
    unit = _k_uniform(kd, size, dt, 0.0, 1.0, layout)
    out = torch.empty_like(unit)
    if kd.shape[0] > 1:  # every key row in one launch: the bounds repeated per row
        lo = lo.reshape(-1).expand(kd.shape[0], size).contiguous()
        hi = hi.reshape(-1).expand(kd.shape[0], size).contiguous()
    nat.call("jxr_truncated_normal_from_unit", _ptr(_raw16(unit, dt)), _ptr(_raw16(lo, dt)), 1,
             _ptr(_raw16(hi, dt)), 1, kd.shape[0] * size, _FLOAT_CODE[dt], _ptr(_raw16(out, dt)),
             _stream())
    return _rebatch(out.reshape(bshape + shape), nb)


# float32 truncated normals of at least this many samples read a table built in the call
# (jxr_truncated_normal_scratch's own threshold)
_TRUNC_TABLE_MIN = 1 << 25


# ---- randint (R/random.R:306-359) -------------------------------------------------------------

_INT_INFO = {"int8": (8, True), "int16": (16, True), "int32": (32, True), "int64": (64, True),
             "uint8": (8, False), "uint16": (16, False), "uint32": (32, False),
             "uint64": (64, False)}


def _int_range(bits, signed):
    return (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if signed else (0, (1 << bits) - 1)


def _wrap_int(v, bits, signed):
    v &= (1 << bits) - 1
    return v - (1 << bits) if signed and v >> (bits - 1) else v


def _int_bound(x, name):
    """A randint bound as (numpy object array of exact Python ints, dtype name): whole
    numbers become the default int dtype (R/random.R:126-130), integer arrays keep their
    (canonical) dtype, other floats are converted to the default int by truncation
    (R/random.R:333-334)."""
    x, nb = _unbatch(x)
    if nb:
        raise JaxNotImplementedError("batched sampler parameters are not supported")
    dint = default_int()
    if isinstance(x, torch.Tensor):
        a, adt = x.detach().cpu().numpy(), _NAME[x.dtype]
    else:
        a = np.asarray(x)
        adt = None if a.dtype.kind in "fb" or not isinstance(x, np.ndarray) else a.dtype.name
    if a.dtype.kind == "b":
        a = a.astype(np.int64)
    if adt is not None and adt in _INT_INFO:
        dt = canonicalize_dtype(adt)
        bits, signed = _INT_INFO[dt]
        vals = np.vectorize(lambda v: _wrap_int(int(v), bits, signed), otypes=[object])(a) \
            if a.size else a.astype(object)
        return vals, dt
    f = a.astype(np.float64)
    bits, signed = _INT_INFO[dint]
    lo, hi = _int_range(bits, signed)
    if a.dtype.kind in "iu" or (f.size and np.all(np.isfinite(f)) and np.all(f == np.round(f))):
        ints = [int(v) for v in (a.ravel() if a.dtype.kind in "iu" else f.ravel())]
        for v in ints:
            if not lo <= v <= hi:
                raise JaxOverflowError(f"Python int {v} too large to convert to {dint}")
        return np.array(ints, dtype=object).reshape(a.shape), dint

    def trunc(v):  # float -> int conversion: toward zero, saturating, NaN -> 0
        if v != v:
            return 0
        if v == float("inf"):
            return hi
        if v == float("-inf"):
            return lo
        return min(max(int(v), lo), hi)
    return np.array([trunc(float(v)) for v in f.ravel()], dtype=object).reshape(f.shape), dint


def random_randint(key, shape, minval, maxval, dtype=None):
    """Integers uniform in [minval, maxval) (R/random.R:306-359): two draws of nbits-bit
    random bits from the halves of split(key) combined modulo the span; dtypes narrower
    than 32 bits sample in int32."""
    k, _, nb = _check_key("randint", key)
    dt = canonicalize_dtype(dtype if dtype is not None else "int")
    shape = canon_shape(shape)
    if dt not in _INT_INFO:
        raise JaxTypeError(f"randint only accepts integer dtypes, got {dt}")
    (mnv, mnb), (mxv, mxb) = _unbatch(minval), _unbatch(maxval)
    levels, bshape = nb, tuple(k.shape[:nb])
    if mnb or mxb:  # bounds batched under vmap: every lane its own bounds, one launch
        levels = max(nb, mnb, mxb)
        if any(b not in (0, levels) for b in (nb, mnb, mxb)):
            raise JaxNotImplementedError("vmap: sampler parameters batched at other levels than "
                                         "the key")
        bs = [tuple(np.shape(v))[:b] for v, b in ((mnv, mnb), (mxv, mxb)) if b]
        if not nb:
            bshape = bs[0]
        if any(b != bshape for b in bs):
            raise JaxValueError(f"vmap got inconsistent sizes for the mapped axis: "
                                f"{sorted(set(bs + [bshape]))}")
    mn, mn_dt = _int_bound(mnv, "minval")
    mx, mx_dt = _int_bound(mxv, "maxval")
    nlead = len(bshape) if (mnb or mxb) else 0
    if nlead:  # per-lane bounds: B + (1,) * pad + lane shape, broadcast to B + shape
        def per_lane(vals, pb):
            lane = tuple(vals.shape[pb:])
            if len(lane) > len(shape):
                lane_b = None
            else:
                try:
                    lane_b = tuple(np.broadcast_shapes(shape, lane))
                except ValueError:
                    lane_b = None
            if lane_b != tuple(shape):
                raise JaxValueError(
                    "randint parameter shapes must be broadcast-compatible with shape argument, "
                    "and the result of broadcasting the shapes must equal the shape argument, "
                    f"but got result {shape_str(lane_b or lane)} for shape argument "
                    f"{shape_str(shape)}.")
            full = vals.reshape((bshape if pb else ()) + (1,) * (len(shape) - len(lane)) + lane)
            return np.broadcast_to(full, bshape + tuple(shape))
        mn, mx = per_lane(mn, mnb), per_lane(mx, mxb)
    dbits, dsigned = _INT_INFO[dt]
    if dbits < 32:  # sample in int32, bounds wrapped to int32 and clipped (:320-325)
        lo_d, hi_d = _int_range(dbits, dsigned)
        mn = np.vectorize(lambda v: min(max(_wrap_int(v, 32, True), lo_d), hi_d),
                          otypes=[object])(mn) if mn.size else mn
        mx = np.vectorize(lambda v: min(max(_wrap_int(v, 32, True), lo_d), hi_d + 1),
                          otypes=[object])(mx) if mx.size else mx
        sbits, ssigned = 32, True
    else:
        sbits, ssigned = dbits, dsigned
    try:
        b = tuple(np.broadcast_shapes(bshape[:nlead] + tuple(shape), mn.shape, mx.shape))[nlead:]
    except ValueError:
        b = None
    if b != tuple(shape):
        raise JaxValueError(
            "randint parameter shapes must be broadcast-compatible with shape argument, and the "
            "result of broadcasting the shapes must equal the shape argument, but got result "
            f"{shape_str(b or np.broadcast_shapes(mn.shape, mx.shape))} for shape argument "
            f"{shape_str(shape)}.")
    smin, smax = _int_range(sbits, ssigned)
    kd = _flat_keys(k)
    size = _size(shape)
    layout = _layout()
    _check_size(size, layout)
    dev = kd.device

    def as_param(vals, f):
        flat = [f(int(v)) for v in np.asarray(vals, dtype=object).ravel()]
        if len(flat) != 1 or nlead:
            flat = [f(int(v)) for v in np.broadcast_to(np.asarray(vals, dtype=object),
                                                       bshape[:nlead] + tuple(shape)).ravel()]
        t = torch.tensor([_wrap_int(v, 64, True) for v in flat], dtype=torch.int64)
        return t.to(dev), (0 if len(flat) == 1 else 1)

    clip = lambda v: min(max(v, smin), smax)  # noqa: E731 - convert_and_clip_integer
    halves = _k_split(kd, (2,), layout, k.impl)
    if nlead:  # every lane a row of draws (an unbatched key: the same draws in every lane)
        nrows = _size(bshape)
        hi = _k_bits(halves[:, 0].contiguous(), size, sbits, layout)
        lo = _k_bits(halves[:, 1].contiguous(), size, sbits, layout)
        if hi.shape[0] != nrows:
            hi = hi.expand(nrows, size).contiguous()
            lo = lo.expand(nrows, size).contiguous()
        oor_t, _ = as_param(mx, lambda v: int(v > smax))
        mn_t, _ = as_param(mn, clip)
        mx_t, _ = as_param(mx, clip)
        oor_t = oor_t.to(torch.uint8)
        out = torch.empty((nrows, size), dtype=_TORCH[dt], device=dev)
        if size:
            nat.call("jxr_randint_combine", _ptr(hi), _ptr(lo), nrows * size, sbits, int(ssigned),
                     _ptr(mn_t), 1, _ptr(mx_t), 1, _ptr(oor_t), 1, dbits, _ptr(out), _stream())
        return _rebatch(out.reshape(bshape + shape), levels)
    out = torch.empty((kd.shape[0], size), dtype=_TORCH[dt], device=dev)
    if (mn.size == 1 and mx.size == 1 and k.impl == "threefry2x32"
            and layout == nat.LAYOUT_PARTITIONABLE):
        # scalar bounds: both draws and the combine in one kernel
        mn1, mx1 = int(np.asarray(mn).ravel()[0]), int(np.asarray(mx).ravel()[0])
        kh, kl = halves[:, 0].contiguous(), halves[:, 1].contiguous()  # alive until launched
        nat.call("jxr_randint", _ptr(kh), _ptr(kl),
                 kd.shape[0], size, 0, size, sbits, int(ssigned), _wrap_int(clip(mn1), 64, True),
                 _wrap_int(clip(mx1), 64, True), int(mx1 > smax), dbits, _ptr(out), _stream())
        return _rebatch(out.reshape(k.shape[:nb] + shape), nb)
    oor_t, oor_s = as_param(mx, lambda v: int(v > smax))
    mn_t, mn_s = as_param(mn, clip)
    mx_t, mx_s = as_param(mx, clip)
    oor_t = oor_t.to(torch.uint8)
    hi = _k_bits(halves[:, 0].contiguous(), size, sbits, layout)
    lo = _k_bits(halves[:, 1].contiguous(), size, sbits, layout)
    if size:
        if mn_s == 0 and mx_s == 0:  # one call over every key's row
            nat.call("jxr_randint_combine", _ptr(hi), _ptr(lo), kd.shape[0] * size, sbits,
                     int(ssigned), _ptr(mn_t), 0, _ptr(mx_t), 0, _ptr(oor_t), 0, dbits,
                     _ptr(out), _stream())
        else:  # every key row in one launch: per-element parameters repeated per row
            nrows = kd.shape[0]
            oor_s = int(oor_t.numel() != 1)

            def rows(t, stride):
                return t.reshape(-1).expand(nrows, size).contiguous() if stride and nrows > 1 else t

            mn_r, mx_r, oor_r = rows(mn_t, mn_s), rows(mx_t, mx_s), rows(oor_t, oor_s)
            nat.call("jxr_randint_combine", _ptr(hi), _ptr(lo), nrows * size, sbits,
                     int(ssigned), _ptr(mn_r), mn_s, _ptr(mx_r), mx_s, _ptr(oor_r), oor_s, dbits,
                     _ptr(out), _stream())
    return _rebatch(out.reshape(k.shape[:nb] + shape), nb)


# ---- permutation and choice (R/random.R:361-464) ---------------------------------------------

def _norm_axis(axis, rank):
    a = int(axis)
    out = a + rank if a < 0 else a
    if (out < 0 or out >= max(rank, 1)) and not (rank == 0 and out == 0):
        raise JaxValueError(f"axis {a} is out of bounds for array of rank {rank}")
    return out


def _as_device_array(x):
    """An array argument as a contiguous device tensor of its canonical dtype (R numbers:
    default float; whole R integers: int32; logicals: bool)."""
    if isinstance(x, torch.Tensor):
        t = x
    else:
        a = np.asarray(x)
        if a.dtype.kind == "f":
            a = a.astype(default_float())
        elif a.dtype.kind in "iu":
            a = a.astype(canonicalize_dtype(a.dtype.name) if isinstance(x, np.ndarray)
                         else "int32")
        t = torch.from_numpy(np.ascontiguousarray(a))
    name = canonicalize_dtype(t.dtype)
    return t.to(device=_device(), dtype=_TORCH[name]).contiguous()


def _k_shuffle(kd_row, impl, outer, n, inner, layout):
    """Flat source index of every position after rnd_shuffle (uint32 tensor)."""
    total = outer * n * inner
    perm = torch.empty(total, dtype=torch.uint32, device=kd_row.device)
    if total:
        nbytes = nat.lib().jxr_shuffle_scratch_bytes(total)
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=kd_row.device)
        nat.call("jxr_shuffle", _ptr(kd_row), _IMPL_CODE[impl], outer, n, inner, layout,
                 _ptr(perm), _ptr(scratch), nbytes, _stream())
    return perm


def _k_shuffle_lanes(kd0, impl, nlanes, outer, n, inner, layout):
    """rnd_shuffle under one vmap level with rbg / unsafe_rbg keys: (nlanes, total) uint32,
    every lane's sort keys drawn from the first lane's key kd0 (rng_bit_generator's
    batching rule, R/prng.R:300-313)."""
    total = outer * n * inner
    perm = torch.empty((nlanes, total), dtype=torch.uint32, device=kd0.device)
    if total and nlanes:
        nbytes = nat.lib().jxr_shuffle_lanes_scratch_bytes(nlanes, total)
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=kd0.device)
        nat.call("jxr_shuffle_lanes", _ptr(kd0), _IMPL_CODE[impl], nlanes, outer, n, inner,
                 layout, _ptr(perm), _ptr(scratch), nbytes, _stream())
    return perm


def _permute_rbg_lanes(kd0, impl, rows, axis, independent, layout):
    """Each lane's array rows[i] shuffled along `axis` by the lanes' permutations of
    _k_shuffle_lanes (rnd_permutation's array branch per lane, R/random.R:388-400)."""
    nl = rows.shape[0]
    shape = tuple(rows.shape[1:])
    outer, n, inner = _size(shape[:axis]), shape[axis], _size(shape[axis + 1:])
    if independent or len(shape) == 1:
        perms = _k_shuffle_lanes(kd0, impl, nl, outer, n, inner, layout)
        return torch.stack([_take(rows[i].reshape(-1), perms[i], 0).reshape(shape)
                            for i in range(nl)])
    inds = _k_shuffle_lanes(kd0, impl, nl, 1, n, 1, layout)
    return torch.stack([_take(rows[i], inds[i], axis) for i in range(nl)])


def _take(x, idx, axis):
    """jnp_take(x, idx, axis) for a device tensor x and uint32 (or non-negative int)
    indices of any shape: result shape x.shape[:axis] + idx.shape + x.shape[axis+1:]."""
    outer = _size(tuple(x.shape[:axis]))
    n_src = x.shape[axis]
    inner = _size(tuple(x.shape[axis + 1:]))
    flat = idx.reshape(-1).contiguous()
    if flat.dtype != torch.uint32:
        flat = flat.to(torch.int64).to(torch.int32).view(torch.uint32)
    out = torch.empty(tuple(x.shape[:axis]) + tuple(idx.shape) + tuple(x.shape[axis + 1:]),
                      dtype=x.dtype, device=x.device)
    nat.call("jxr_take", _ptr(x), outer, n_src, _ptr(flat), flat.numel(),
             inner * x.element_size(), _ptr(out), None, _stream())
    return out


def random_permutation(key, x, axis=0, independent=False):
    """A shuffled copy of x along `axis`, or of arange(x) for an integer x (int32)
    (R/random.R:378-400).  Every round of rnd_shuffle (R/random.R:402-413) draws 32-bit sort
    keys with the threefry kernels and sorts (key, position) pairs with a stable radix sort
    on the device."""
    k, _, nb = _check_key("permutation", key)
    xv, xnb = _unbatch(x)
    if xnb:  # x batched under vmap: each lane shuffles its own array with its own key
        return _permutation_lanes(k, nb, xv, xnb, axis, independent)
    ndim = xv.ndim if isinstance(xv, (torch.Tensor, np.ndarray)) else np.ndim(xv)
    axis = _norm_axis(axis, max(ndim, 1))
    kd = _flat_keys(k)
    layout = _layout()
    bshape = k.shape[:nb]
    rbg_lanes = nb and k.impl != "threefry2x32"  # the lanes' bits from the first key
    if rbg_lanes and nb > 1:
        raise JaxNotImplementedError("random_permutation under nested vmap with rbg keys")
    if ndim == 0:
        if isinstance(xv, (torch.Tensor, np.ndarray)):
            t = torch.as_tensor(xv)
            if t.dtype.is_floating_point or t.dtype.is_complex or t.dtype == torch.bool:
                raise JaxTypeError("x must be an integer or at least 1-dimensional")
            n = int(t.item())
        elif isinstance(xv, bool) or not isinstance(xv, numbers.Real) or xv != int(xv):
            raise JaxTypeError("x must be an integer or at least 1-dimensional")
        else:
            n = int(xv)
        n = max(n, 0)
        if rbg_lanes:
            out = _k_shuffle_lanes(kd[0], k.impl, kd.shape[0], 1, n, 1, layout).view(torch.int32)
            return _rebatch(out.reshape(bshape + (n,)), nb)
        outs = [_k_shuffle(kd[r], k.impl, 1, n, 1, layout).view(torch.int32)
                for r in range(kd.shape[0])]
        out = torch.stack(outs) if outs else torch.empty((0, n), dtype=torch.int32)
        return _rebatch(out.reshape(bshape + (n,)), nb)
    xt = _as_device_array(xv)
    shape = tuple(xt.shape)
    if rbg_lanes:
        rows = xt.unsqueeze(0).expand((kd.shape[0],) + shape).contiguous()
        out = _permute_rbg_lanes(kd[0], k.impl, rows, axis, independent, layout)
        return _rebatch(out.reshape(bshape + shape), nb)
    outs = [_permute_array(kd[r], k.impl, xt, axis, independent, layout)
            for r in range(kd.shape[0])]
    out = torch.stack(outs) if outs else torch.empty((0,) + shape, dtype=xt.dtype)
    return _rebatch(out.reshape(bshape + shape), nb)


def _permute_array(kd_row, impl, xt, axis, independent, layout):
    """One key's shuffle of the device array xt along `axis` (rnd_permutation's array
    branch, R/random.R:388-400)."""
    shape = tuple(xt.shape)
    outer, n, inner = _size(shape[:axis]), shape[axis], _size(shape[axis + 1:])
    if independent or xt.ndim == 1:
        perm = _k_shuffle(kd_row, impl, outer, n, inner, layout)
        return _take(xt.reshape(-1), perm, 0).reshape(shape)
    ind = _k_shuffle(kd_row, impl, 1, n, 1, layout)
    return _take(xt, ind, axis)


def _permutation_lanes(k, nb, xv, xnb, axis, independent):
    """random_permutation with x batched under vmap (the reference's vmap batches every
    argument, R/batching.R:22-50): lane i shuffles x's i-th array with key i (or with the
    one key when only x is batched), as the loop over the lanes would."""
    levels = max(nb, xnb)
    if nb not in (0, levels):
        raise JaxNotImplementedError("vmap: sampler parameters batched at other levels than the key")
    if nb > 1 and k.impl != "threefry2x32":
        raise JaxNotImplementedError("random_permutation under nested vmap with rbg keys")
    xt = _as_device_array(xv)
    B = tuple(xt.shape[:xnb])
    if nb and tuple(k.shape[:nb]) != B:
        raise JaxValueError(f"vmap got inconsistent sizes for the mapped axis: "
                            f"{sorted({tuple(k.shape[:nb]), B})}")
    lane = tuple(xt.shape[xnb:])
    if not lane:  # an integer n per lane would give lanes of different lengths
        raise JaxTypeError("x must be an integer or at least 1-dimensional")
    axis = _norm_axis(axis, len(lane))
    kd = _flat_keys(k)
    rows = xt.reshape((-1,) + lane)
    if nb and k.impl != "threefry2x32":  # the lanes' bits from the first key
        out = _permute_rbg_lanes(kd[0], k.impl, rows.contiguous(), axis, independent, _layout())
        return _rebatch(out.reshape(B + lane), levels)
    outs = [_permute_array(kd[i] if kd.shape[0] > 1 else kd[0], k.impl, rows[i].contiguous(),
                           axis, independent, _layout()) for i in range(rows.shape[0])]
    out = torch.stack(outs) if outs else torch.empty((0,) + lane, dtype=xt.dtype)
    return _rebatch(out.reshape(B + lane), levels)


def random_choice(key, a, shape=(), replace=True, p=None, axis=0, mode=None):
    """Samples of a (an integer n: arange(n)) along `axis` (R/random.R:417-464): with
    replacement through randint; without, the first draws of a permutation; with p,
    searchsorted of the cumulative sums (replace) or the top draws of gumbel + log(p)."""
    k, _, nb = _check_key("choice", key)
    (av0, anb), (pv0, pnb) = _unbatch(a), _unbatch(p)
    if (anb or pnb) and k.impl != "threefry2x32" and nb:
        raise JaxNotImplementedError("random_choice under vmap over rbg keys with batched a or p")
    if anb or pnb:  # a or p batched under vmap: each lane's choice, stacked
        levels = max(nb, anb, pnb)
        if any(b not in (0, levels) for b in (nb, anb, pnb)):
            raise JaxNotImplementedError("vmap: sampler parameters batched at other levels than "
                                         "the key")
        bs = [tuple(np.shape(v))[:b] for v, b in ((av0, anb), (pv0, pnb)) if b]
        B = tuple(k.shape[:nb]) if nb else bs[0]
        if any(b != B for b in bs):
            raise JaxValueError(f"vmap got inconsistent sizes for the mapped axis: "
                                f"{sorted(set(bs + [B]))}")

        def lanes(v, b):
            if not b:
                return None
            t = v if isinstance(v, torch.Tensor) else torch.as_tensor(np.asarray(v))
            return t.reshape((-1,) + tuple(t.shape[b:]))
        arows, prows = lanes(av0, anb), lanes(pv0, pnb)
        kw = _KEY_WORDS[k.impl]
        kdata = k.data.reshape((-1, kw))
        rows = [random_choice(PRNGKeyArray(kdata[i] if nb else kdata[0], k.impl),
                              arows[i] if anb else av0, shape, replace,
                              prows[i] if pnb else pv0, axis, mode) for i in range(_size(B))]
        out = torch.stack(rows) if rows else torch.empty((0,))
        return _rebatch(out.reshape(B + tuple(out.shape[1:])), levels)
    if nb and k.impl == "threefry2x32":  # vmap over keys: each key's choice, stacked
        rows = [random_choice(PRNGKeyArray(d, k.impl), a, shape, replace, p, axis, mode)
                for d in k.data.reshape((-1, _KEY_WORDS[k.impl]))]
        out = torch.stack(rows) if rows else torch.empty((0,))
        return _rebatch(out.reshape(k.shape[:nb] + tuple(out.shape[1:])), nb)
    if nb > 1:
        raise JaxNotImplementedError("random_choice under nested vmap with rbg keys")
    # rbg / unsafe_rbg keys under vmap: the draws follow rng_bit_generator's batching rule
    # (every lane's bits from the first key, R/prng.R:300-313), lane i taking row i
    lanes = _size(k.shape[:nb]) if nb else 0
    shape = canon_shape(shape)
    av, anb = _unbatch(a)
    if anb:
        raise JaxNotImplementedError("batched choice arguments are not supported")
    if isinstance(av, (torch.Tensor, np.ndarray)) and np.ndim(av) > 0:
        arr = _as_device_array(av)
        axis = _norm_axis(axis, arr.ndim)
        n_inputs = arr.shape[axis]
        adtype = arr.dtype
    elif isinstance(av, (list, tuple)) and len(av) != 1:
        arr = _as_device_array(av)
        axis = _norm_axis(axis, arr.ndim)
        n_inputs = arr.shape[axis]
        adtype = arr.dtype
    else:
        arr = None
        v = av[0] if isinstance(av, (list, tuple)) else av
        v = v.item() if isinstance(v, (torch.Tensor, np.ndarray)) else v
        n_inputs = int(v)
        adtype = _TORCH[default_int()] if float(v) == int(v) else _TORCH[default_float()]
    n_draws = _size(shape)
    lshape = ((lanes,) if nb else ()) + tuple(shape)  # the result's shape (before a's axes)
    if n_draws == 0:
        z = torch.zeros(lshape, dtype=adtype, device=_device())
        return _rebatch(z, nb) if arr is None else _rebatch(
            torch.stack([_take(arr, z[i].to(torch.int64), axis) for i in range(lanes)])
            if nb else _take(arr, z.to(torch.int64), axis), nb)
    if n_inputs <= 0:
        raise JaxValueError("a must be greater than 0 unless no samples are taken")
    if not replace and n_draws > n_inputs:
        raise JaxValueError(f"Cannot take a larger sample (size {n_draws}) than population "
                            f"(size {n_inputs}) when 'replace=False'")
    def take_lanes(ind):  # ind: lshape indices -> arr's rows (per lane under vmap)
        if arr is None:
            return _rebatch(ind, nb)
        if not nb:
            return _take(arr, ind, axis)
        return _rebatch(torch.stack([_take(arr, ind[i], axis) for i in range(lanes)]), nb)
    if p is None:
        if replace:
            ind, _ = _unbatch(random_randint(key, shape, 0, n_inputs))
            return take_lanes(ind)
        kd = _flat_keys(k)
        if nb:
            perm = _k_shuffle_lanes(kd[0], k.impl, lanes, 1, n_inputs, 1, _layout())
            ind = perm[:, :n_draws].contiguous()
        else:
            ind = _k_shuffle(kd[0], k.impl, 1, n_inputs, 1, _layout())[:n_draws]
        if arr is None:
            return _rebatch(ind.view(torch.int32).reshape(lshape), nb)
        return take_lanes(ind.reshape(lshape))
    # promote_dtypes_inexact: float arrays keep their dtype, everything else is the
    # default float
    if isinstance(p, torch.Tensor):
        pt = p
        pdt = _NAME[p.dtype] if p.dtype.is_floating_point else default_float()
    else:
        pa = np.asarray(p)
        pdt = (canonicalize_dtype(pa.dtype.name) if isinstance(p, np.ndarray) and pa.dtype.kind == "f"
               else default_float())
        pt = torch.from_numpy(np.ascontiguousarray(pa, dtype=np.float64))
    pdt = canonicalize_dtype(pdt)
    if pdt not in ("float32", "float64"):
        raise JaxNotImplementedError(f"random_choice with p of dtype {pdt}")
    if tuple(pt.shape) != (n_inputs,):
        raise JaxValueError(f"p must be None or a 1D vector with the same size as a.shape[axis]. "
                            f"p has shape {shape_str(tuple(pt.shape))} and a.shape[axis] is "
                            f"{n_inputs}.")
    dint = default_int()
    kd = _flat_keys(k)
    layout = _layout()
    if replace:
        # cumulative sums in the dtype, left to right (jnp_cumsum)
        pd = pt.to(device=kd.device, dtype=_TORCH[pdt]).contiguous()
        cuml = torch.empty_like(pd)
        nat.call("jxr_cumsum", _ptr(pd), n_inputs, _FLOAT_CODE[pdt], _ptr(cuml), _stream())
        unit = _k_uniform(kd, n_draws, pdt, 0.0, 1.0, layout)  # (lanes or 1, n_draws)
        ind = torch.empty(unit.numel(), dtype=_TORCH[dint], device=kd.device)
        nat.call("jxr_choice_p_from_unit", _ptr(unit), unit.numel(), _FLOAT_CODE[pdt],
                 _ptr(cuml), n_inputs, _BITS[dint], _ptr(ind), _stream())
    else:
        gv, _ = _unbatch(random_gumbel(key, (n_inputs,), pdt, mode=mode))
        g = gv.reshape(-1, n_inputs).contiguous()  # (lanes or 1, n_inputs)
        pd = pt.to(device=kd.device, dtype=_TORCH[pdt]).contiguous()
        nbytes = nat.lib().jxr_argsort_scratch_bytes(n_inputs)
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=kd.device)
        inds = []
        for r in range(g.shape[0]):
            nat.call("jxr_add_log", _ptr(g[r]), _ptr(pd), n_inputs, _FLOAT_CODE[pdt], _stream())
            order = torch.empty(n_inputs, dtype=torch.uint32, device=kd.device)
            nat.call("jxr_argsort_float", _ptr(g[r]), n_inputs, _FLOAT_CODE[pdt], 1,
                     _ptr(order), _ptr(scratch), nbytes, _stream())
            inds.append(order[:n_draws].view(torch.int32).to(_TORCH[dint]))
        ind = torch.stack(inds)
    return take_lanes(ind.reshape(lshape))


# ---- rng_bit_generator (R/prng.R:264-345) ---------------------------------------------------

lax_RandomAlgorithm = {"RNG_DEFAULT": 0, "RNG_THREE_FRY": 1, "RNG_PHILOX": 2}


def lax_rng_bit_generator(key, shape, dtype="uint32", algorithm=0):
    """(new_key, bits): random bits from XLA's RngBitGenerator for a uint32[4] (or
    uint64[2]) key (R/prng.R:322-345).  The default algorithm is Philox4x32-10, as XLA's CPU
    backend runs it; new_key is the state after the request (the 128-bit counter advanced
    by the blocks used)."""
    shape = tuple(int(v) for v in np.atleast_1d(np.asarray(shape, dtype=np.int64)))
    dt = canonicalize_dtype(dtype)
    if dt not in ("uint8", "uint16", "uint32", "uint64"):
        raise JaxTypeError(f"rng_bit_generator: unsupported dtype {dt}")
    kt = key if isinstance(key, torch.Tensor) else torch.as_tensor(np.asarray(key))
    kname = _NAME[kt.dtype]
    if not ((kname == "uint32" and tuple(kt.shape) == (4,)) or
            (kname == "uint64" and tuple(kt.shape) == (2,))):
        raise JaxValueError("rng_bit_generator: key must be uint32[4] or uint64[2], got "
                            f"{kname}{list(kt.shape)}")
    if int(algorithm) == lax_RandomAlgorithm["RNG_THREE_FRY"]:
        raise JaxNotImplementedError("rng_bit_generator with RNG_THREE_FRY: only the default "
                                     "(Philox) algorithm is provided")
    k4 = kt.to(_device()).contiguous().view(torch.uint32).reshape(4)
    size = _size(shape)
    out = torch.empty(size, dtype=_TORCH[dt], device=k4.device)
    new = torch.empty(4, dtype=torch.uint32, device=k4.device)
    nat.call("jxr_rbg_bits", _ptr(k4), size, 0, size, _BITS[dt], _ptr(out), _ptr(new), _stream())
    new_key = new if kname == "uint32" else new.view(torch.uint64)
    return new_key, out.reshape(shape)


# ---- erf_inv (R/lax.R:222) ---------------------------------------------------------------------

@_uses_erf_inv
def lax_erf_inv(x):
    """Element-wise inverse error function for float32/float64 arrays."""
    t = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x, dtype=default_float()))
    dt = _NAME[t.dtype]
    if dt not in ("float32", "float64"):
        raise JaxTypeError(f"erf_inv does not accept dtype {dt}")
    src = t.to(_device()).contiguous()
    out = torch.empty_like(src)
    nat.call("jxr_erf_inv", _ptr(src), src.numel(), _FLOAT_CODE[dt], _ptr(out), _stream())
    return out
