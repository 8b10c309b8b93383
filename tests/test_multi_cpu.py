"""The multi-device host logic on CPU with gloo, world size 2: every rank's slab of a
request (shard_range) assembled on one rank (shard.gather_to) equals the whole request,
and a rank that fails before the gather makes the other rank's gather end with an error
instead of waiting for ever.  The slabs are computed by the oracle (no GPU here)."""

import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, size, fail_rank, results):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist

    from jaxr_b200.shard import gather_to, shard_range
    from oracle import oracle as orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        lo, hi = shard_range(size, rank, world)
        key = orc.seed(123)
        slab = torch.from_numpy(orc.random_bits(key, 32, size, True, lo, hi - lo).view(np.int32))
        if rank == fail_rank:
            raise RuntimeError("simulated rank failure before the gather")
        whole = gather_to(slab, root=0)
        if rank == 0:
            want = orc.random_bits(key, 32, size, True).view(np.int32)
            results[rank] = bool(np.array_equal(whole.numpy(), want))
        else:
            results[rank] = whole is None
    except Exception as e:  # noqa: BLE001 - report any failure to the parent
        results[rank] = f"error: {type(e).__name__}: {e}"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, size, fail_rank=-1):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, size, fail_rank, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
                p.join()
        return dict(results)


def test_slabs_gathered_on_one_rank_equal_the_request():
    res = _run(2, 100003)  # an odd size: slabs of different lengths
    assert res == {0: True, 1: True}, res


def test_a_failed_rank_ends_the_gather_with_an_error():
    res = _run(2, 4096, fail_rank=1)
    assert str(res.get(1, "")).startswith("error: RuntimeError: simulated rank failure"), res
    assert str(res.get(0, "")).startswith("error:"), res  # timed out or connection closed
