"""One rank of the multi-GPU check (launched by tests/test_multi_gpu.py through
torch.distributed.run): each rank produces its slab of a request on its own GPU, the
slabs are gathered on rank 0 over NCCL, and rank 0 compares the result with the whole
request generated on its own device and with the oracle at sampled positions."""

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import jaxr_b200 as jr  # noqa: E402
from jaxr_b200.shard import (close_peer_mappings, gather_to, random_bits_gathered,  # noqa: E402
                             random_bits_shard)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    ok = True
    size = (1 << 27) + 3
    for part in (True, False):
        with jr.with_jax_config("jax_threefry_partitionable", part):
            key = jr.random_key(123)
            slab = random_bits_shard(key, (size,), rank, world)
            whole = gather_to(slab, root=0)
            if rank == 0:
                mine = jr.random_bits(key, (size,))
                ok &= bool(torch.equal(whole.view(torch.int32), mine.view(torch.int32)))
                from oracle import oracle as orc
                idx = np.unique(np.random.default_rng(0).integers(0, size, 2048))
                got = whole.view(torch.int32)[torch.from_numpy(idx).to(dev)].cpu().numpy().view(np.uint32)
                ok &= bool(np.array_equal(got, orc.bits_at(orc.seed(123), 32, size, part, idx)))
            # every rank stores its slab straight into rank 0's buffer over NVLink
            for _ in range(2):  # the second call reuses the peer mapping
                g = random_bits_gathered(key, (size,), root=0)
                if rank == 0:
                    ok &= bool(torch.equal(g.view(torch.int32), mine.view(torch.int32)))
        torch.cuda.synchronize()
    close_peer_mappings()
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print("MULTI_GPU_OK" if flag.item() == 1 else "MULTI_GPU_MISMATCH", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
