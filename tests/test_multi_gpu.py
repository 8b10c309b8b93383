"""Counter-range shards on two GPUs of one node, gathered on one of them, equal the
whole request (both layouts).  Needs at least two GPUs; runs tests/multi_gpu_worker.py
under torch.distributed.run, and drives every GPU from one process through
jxr_random_bits_multi."""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_gpu_shards_gather_to_the_whole_request():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(port), os.path.join(ROOT, "tests", "multi_gpu_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "MULTI_GPU_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.gpu
def test_random_bits_multi_one_process(oracle):
    """jxr_random_bits_multi: every visible GPU driven from this process, slabs per device
    and the whole request gathered on device 0 through peer stores."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs in one process")
    import jaxr_b200 as jr
    from jaxr_b200.shard import random_bits_multi
    size = (1 << 24) + 5
    want = oracle.random_bits(oracle.seed(31), 32, size, True)
    key = jr.random_key(31)
    slabs = random_bits_multi(key, (size,))
    got = np.concatenate([s.cpu().numpy() for s in slabs])
    assert np.array_equal(got, want)
    whole = random_bits_multi(key, (size,), gather_to=0)
    assert whole.device.index == 0
    assert np.array_equal(whole.cpu().numpy(), want)
    with jr.with_jax_config("jax_threefry_partitionable", False):
        whole = random_bits_multi(key, (size,), gather_to=1, dtype="uint8")
        assert np.array_equal(whole.cpu().numpy(), oracle.random_bits(oracle.seed(31), 8, size,
                                                                       False))
