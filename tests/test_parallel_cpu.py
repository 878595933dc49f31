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


def _ep_worker(rank, world, port, out, padded=True):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kernelbench_harbor_b200 import parallel
        from oracle import moe as om
        E, T, D = 4, 12, 8
        g = torch.Generator().manual_seed(11)
        xs = torch.randn(world * T, D, generator=g)
        logits = torch.randn(world * T, E, generator=g)
        mats = torch.randn(E, D, D, generator=g)

        def route(lg):
            ti, ga = om.route(lg.numpy())
            return torch.from_numpy(ti), torch.from_numpy(ga)

        def expert(el, rows, w):
            return rows @ w[el]

        def combine(ye, ts, ga):
            return ye[ts[:, 0].long()] * ga[:, :1] + ye[ts[:, 1].long()] * ga[:, 1:]

        epr = E // world
        local_w = mats[rank * epr:(rank + 1) * epr]
        mod = parallel.ExpertParallelMoE(E, route=route, expert=expert, combine=combine, padded=padded)
        y = mod(xs[rank * T:(rank + 1) * T], logits[rank * T:(rank + 1) * T], local_w)
        out.put((rank, y.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("padded", [True, False])
def test_expert_parallel_matches_dense(padded):
    from oracle import moe as om
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q_out, padded)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q_out.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    E, T, D = 4, 12, 8
    g = torch.Generator().manual_seed(11)
    xs = torch.randn(2 * T, D, generator=g)
    logits = torch.randn(2 * T, E, generator=g)
    mats = torch.randn(E, D, D, generator=g)
    ti, ga = om.route(logits.numpy())
    ref = np.zeros((2 * T, D), dtype=np.float32)
    for t in range(2 * T):
        for k in range(2):
            ref[t] += ga[t, k] * (xs[t].numpy() @ mats[ti[t, k]].numpy())
    y = np.concatenate([res[0], res[1]])
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)
