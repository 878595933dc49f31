"""Host logic of the N-sharded path on CPU ranks (gloo, world size 2): each
rank computes its column shard with the oracle's restatement, the all-gather
reassembles y, which must equal the unsharded result bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import w4a16_inputs


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _local_gemm(x, q, s, z, group):
    from oracle import w4a16 as o
    return torch.from_numpy(o.forward_fp32(x.numpy(), q.numpy(), s.numpy(), z.numpy(), group))


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kernelbench_harbor_b200 import parallel
        x, q, s, z = w4a16_inputs(8, 256, 512, 128, "fp16", seed=3)
        qs, ss, zs = parallel.shard_weights(q, s, z, world, rank)
        y = parallel.ColumnShardedW4A16(128, local_gemm=_local_gemm)(x, qs, ss, zs)
        if rank == 0:
            out.put(y.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_gather_matches_unsharded():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    y = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, q, s, z = w4a16_inputs(8, 256, 512, 128, "fp16", seed=3)
    ref = _local_gemm(x, q, s, z, 128).numpy()
    assert np.array_equal(y, ref)


def test_shard_bounds_errors():
    from kernelbench_harbor_b200 import parallel
    with pytest.raises(ValueError):
        parallel.shard_bounds(4096, 3, 0)
    with pytest.raises(ValueError):
        parallel.shard_bounds(48 * 3, 3, 0)
    assert parallel.shard_bounds(4096, 8, 7) == (3584, 4096)
