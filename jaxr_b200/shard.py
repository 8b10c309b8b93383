"""Requests split by contiguous counter range over the GPUs of one node.

Every element of a threefry request depends only on (key, element index), so device
r of G produces elements [r*size/G, (r+1)*size/G) of the C-order result with no
communication (the partitionable layout; for the original layout the same element
range is produced from the blocks that feed it).

When a caller wants the whole array on one device there are two ways:
`random_bits_gathered` has every rank's kernel store its slab directly into the root
GPU's buffer over NVLink (a CUDA IPC peer mapping, plain stores), so generation and
transfer are one pass; `gather_to` copies slabs that already exist to the root with NCCL
point-to-point.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as nat
from .random import (_TORCH, _BITS, _KEY_WORDS, _check_key, _flat_keys, _layout, _ptr, _size,
                     _stream, canon_shape, canonicalize_dtype, default_uint)
from .errors import JaxValueError


def _bits_range(k, kd, size, lo, n, bit_width, out_ptr):
    """Elements [lo, lo + n) of random_bits(k, (size,)) written at out_ptr: threefry keys
    through the cipher kernels, rbg / unsafe_rbg keys through the Philox stream."""
    if _KEY_WORDS[k.impl] == 4:
        nat.call("jxr_rbg_bits", _ptr(kd), size, lo, n, bit_width, out_ptr, None, _stream())
    else:
        nat.call("jxr_random_bits", _ptr(kd), 1, size, lo, n, _layout(), bit_width, out_ptr,
                 _stream())


def shard_range(size, rank, world):
    """[begin, end) of `rank`'s slab of a size-element request over `world` devices."""
    if world < 1 or not 0 <= rank < world:
        raise JaxValueError(f"bad rank {rank} of world {world}")
    return size * rank // world, size * (rank + 1) // world


def random_bits_shard(key, shape, rank, world, dtype=None, out=None):
    """This device's slab of random_bits(key, shape, dtype): a 1-D tensor of the elements
    [begin, end) of the flattened C-order result (see shard_range)."""
    k, _, nb = _check_key("bits", key)
    if nb:
        raise JaxValueError("random_bits_shard takes a single key")
    dt = default_uint() if dtype is None else canonicalize_dtype(dtype)
    size = _size(canon_shape(shape))
    lo, hi = shard_range(size, rank, world)
    n = hi - lo
    if out is None:
        out = torch.empty(n, dtype=_TORCH[dt], device=k.data.device)
    elif out.numel() != n or out.dtype != _TORCH[dt] or not out.is_contiguous():
        raise JaxValueError(f"out must be a contiguous {dt} tensor of {n} elements")
    _bits_range(k, _flat_keys(k), size, lo, n, _BITS[dt], _ptr(out))
    return out


def random_bits_to_host(key, shape, dtype=None, out=None):
    """random_bits(key, shape, dtype) written into host memory (pinned `out`, allocated if
    not given): generated on the current device in chunks, each copied to the host while
    the next is generated.  Returns the host tensor of `shape`."""
    k, _, nb = _check_key("bits", key)
    if nb:
        raise JaxValueError("random_bits_to_host takes a single key")
    dt = default_uint() if dtype is None else canonicalize_dtype(dtype)
    shape = canon_shape(shape)
    size = _size(shape)
    if k.impl != "threefry2x32":
        raise JaxValueError("random_bits_to_host takes a threefry2x32 key")
    if out is None:
        out = torch.empty(size, dtype=_TORCH[dt], pin_memory=True)
    keys_host = k.data.reshape(-1, 2).cpu().contiguous()
    nat.call("jxr_random_bits_host", _ptr(keys_host), 1, size, 0, size, _layout(), _BITS[dt],
             _ptr(out))
    return out.reshape(shape)


def gather_to(local, root, group=None):
    """Assemble the slabs of all ranks (rank order) on rank `root` with NCCL; returns the
    whole flattened array on root and None elsewhere.  Every rank passes its slab; slabs
    may differ in length by one element (shard_range)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = torch.tensor([local.numel()], device=local.device, dtype=torch.int64)
    sizes = [torch.empty_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    view = local.view(torch.int32) if local.element_size() == 4 else local.view(torch.uint8)
    if rank == root:
        total = sum(sizes) * local.element_size() // view.element_size()
        whole = torch.empty(total, dtype=view.dtype, device=local.device)
        parts = list(torch.split(whole, [s * local.element_size() // view.element_size()
                                         for s in sizes]))
        ops = []
        for r in range(world):
            if r == root:
                parts[r].copy_(view)
            else:
                ops.append(dist.P2POp(dist.irecv, parts[r], r, group=group))
        for w in dist.batch_isend_irecv(ops) if ops else []:
            w.wait()
        return whole.view(local.dtype)
    for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, view, root, group=group)]):
        w.wait()
    return None


# ---- whole request on one device, written over NVLink by every rank's kernel ----------------

_peer_maps = {}  # IPC handle -> base address of the mapping in this process


def _export(t):
    handle = (ctypes.c_uint8 * 64)()
    off = ctypes.c_uint64(0)
    nat.call("jxr_ipc_export", t.data_ptr(), handle, ctypes.byref(off))
    return bytes(handle), off.value


def _open(handle):
    base = _peer_maps.get(handle)
    if base is None:
        buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
        ptr = ctypes.c_void_p(0)
        nat.call("jxr_ipc_open", buf, ctypes.byref(ptr))
        base = _peer_maps[handle] = ptr.value
    return base


def close_peer_mappings():
    """Unmap every peer buffer random_bits_gathered opened in this process."""
    for base in _peer_maps.values():
        nat.call("jxr_ipc_close", base)
    _peer_maps.clear()


def random_bits_gathered(key, shape, root=0, dtype=None, out=None, group=None):
    """random_bits(key, shape, dtype) on rank `root`, generated by all ranks: rank r's
    kernel computes elements shard_range(size, r, world) and stores them straight into the
    root's buffer through a peer mapping over NVLink.  Collective (every rank calls it
    with the same key and shape); returns the flattened result on the root and None
    elsewhere.  `out`, on the root, is reused as the destination; the mapping of a buffer
    stays open in the other processes until close_peer_mappings()."""
    import torch.distributed as dist
    k, _, nb = _check_key("bits", key)
    if nb:
        raise JaxValueError("random_bits_gathered takes a single key")
    dt = default_uint() if dtype is None else canonicalize_dtype(dtype)
    size = _size(canon_shape(shape))
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    kd = _flat_keys(k)
    whole = None
    if rank == root:
        whole = out if out is not None else torch.empty(size, dtype=_TORCH[dt], device=kd.device)
        if whole.numel() != size or whole.dtype != _TORCH[dt] or not whole.is_contiguous():
            raise JaxValueError(f"out must be a contiguous {dt} tensor of {size} elements")
        meta = [_export(whole)]
    else:
        meta = [None]
    dist.broadcast_object_list(meta, src=root, group=group)
    handle, off = meta[0]
    base = whole.data_ptr() if rank == root else _open(handle) + off
    lo, hi = shard_range(size, rank, world)
    esz = _BITS[dt] // 8
    _bits_range(k, kd, size, lo, hi - lo, _BITS[dt], base + lo * esz)
    torch.cuda.current_stream().synchronize()
    dist.barrier(group=group)
    return whole


# ---- several GPUs from one process -----------------------------------------------------------

def random_bits_multi(key, shape, devices=None, dtype=None, gather_to=None):
    """random_bits(key, shape, dtype) computed by several GPUs of this process (all visible
    ones by default): device i produces elements shard_range(size, i, len(devices)).
    Returns the list of slabs (a 1-D tensor on each device), or, with gather_to = i, the
    whole flattened request on devices[i], every device's kernel storing its slab there
    through peer access.  Threefry keys only."""
    import torch
    k, _, nb = _check_key("bits", key)
    if nb or k.impl != "threefry2x32":
        raise JaxValueError("random_bits_multi takes a single threefry2x32 key")
    dt = default_uint() if dtype is None else canonicalize_dtype(dtype)
    size = _size(canon_shape(shape))
    devices = list(range(torch.cuda.device_count())) if devices is None else list(devices)
    n = len(devices)
    keys = [k.data.reshape(2).to(torch.device("cuda", d)).contiguous() for d in devices]
    streams = [torch.cuda.current_stream(d).cuda_stream for d in devices]
    dev_arr = (ctypes.c_int * n)(*devices)
    key_arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in keys])
    st_arr = (ctypes.c_void_p * n)(*streams)
    if gather_to is None:
        slabs = [torch.empty(shard_range(size, i, n)[1] - shard_range(size, i, n)[0],
                             dtype=_TORCH[dt], device=torch.device("cuda", d))
                 for i, d in enumerate(devices)]
        out_arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in slabs])
        nat.call("jxr_random_bits_multi", dev_arr, n, key_arr, size, _layout(), _BITS[dt],
                 out_arr, -1, None, st_arr)
        for d in devices:
            torch.cuda.current_stream(d).synchronize()
        return slabs
    whole = torch.empty(size, dtype=_TORCH[dt], device=torch.device("cuda", devices[gather_to]))
    nat.call("jxr_random_bits_multi", dev_arr, n, key_arr, size, _layout(), _BITS[dt], None,
             int(gather_to), whole.data_ptr(), st_arr)
    for d in devices:
        torch.cuda.current_stream(d).synchronize()
    return whole
