"""Column-sharded W4A16 with the all-gather fused into the GEMM epilogue
(NVLink peer stores between device barriers).

* single GPU: the peer entry point with several destinations / a column
  offset inside a wider y matches the plain GEMM bit for bit, and the device
  barrier's bounded wait gives up with a status (a peer that never arrives,
  made on the host side by a signal word nothing sets);
* two GPUs (skipped with fewer): two NCCL ranks, each rank's y equals the
  concatenation of the per-shard plain GEMMs bit for bit (same shard shape,
  same kernel plan), and matches the oracle within the kernel tolerance.
"""
import os
import socket

import pytest
import torch

from tests.helpers import w4a16_inputs

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("M", [1, 16, 32, 33, 160, 1024])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_peer_entry_single_gpu_offsets(M, dtype):
    from kernelbench_harbor_b200 import ops
    x, q, s, z = (t.cuda() for t in w4a16_inputs(M, 1024, 512, 128, dtype, seed=11))
    ref = ops.w4a16_gemm(x, q, s, z, 128)
    # two destinations, each [M, 1536] with this shard at columns [512, 1024)
    ya = torch.full((M, 1536), 7.0, dtype=x.dtype, device="cuda")
    yb = torch.full((M, 1536), -3.0, dtype=x.dtype, device="cuda")
    ops.w4a16_gemm_peers(x, q, s, z, 128, [ya.data_ptr(), yb.data_ptr()], 1536, 512)
    torch.cuda.synchronize()
    for y in (ya, yb):
        assert torch.equal(y[:, 512:1024], ref)
        assert torch.all(y[:, :512] == y[0, 0]) and torch.all(y[:, 1024:] == y[0, 0])
    assert ops.device_status() == 0


def test_peer_entry_argument_errors():
    from kernelbench_harbor_b200 import _lib, ops
    x, q, s, z = (t.cuda() for t in w4a16_inputs(16, 256, 256, 128, "fp16", seed=1))
    y = torch.empty((16, 512), dtype=torch.float16, device="cuda")
    for ldy, col0 in ((512, 300), (500, 0), (512, 384)):
        with pytest.raises(_lib.B200QError):
            ops.w4a16_gemm_peers(x, q, s, z, 128, [y.data_ptr()], ldy, col0)
    with pytest.raises(_lib.B200QError):
        ops.w4a16_gemm_peers(x, q, s, z, 128, [y.data_ptr()] * 9, 512, 0)


def test_barrier_timeout_sets_status():
    """Rank 0 of a 2-rank barrier whose peer never signals: the wait ends
    after its limit (shortened to 300 ms for the test) with
    B200Q_DEV_ERR_TIMEOUT, and the context stays usable.  Both 'pads' are
    local buffers; nothing faults or hangs."""
    from kernelbench_harbor_b200 import _lib, ops
    L = _lib.lib()
    mine = torch.zeros(64, dtype=torch.int32, device="cuda")
    peer = torch.zeros(64, dtype=torch.int32, device="cuda")
    ops.device_status()  # clear
    old = L.b200q_set_peer_barrier_timeout_ms(300)
    try:
        ops.peer_barrier([mine.data_ptr(), peer.data_ptr()], 0, torch.device("cuda", 0))
        torch.cuda.synchronize()
    finally:
        L.b200q_set_peer_barrier_timeout_ms(old)
    assert int(peer[16]) == 1 and int(mine[61]) == 1  # our epoch was published
    assert ops.device_status() & 1
    # the context still runs kernels
    assert torch.ones(4, device="cuda").sum().item() == 4


def _two_rank_worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from kernelbench_harbor_b200 import ops, parallel
        from tests.helpers import torch_ref_fp32
        mod = parallel.PeerGatherW4A16(128)
        worst = 0.0
        for M, dtype in ((16, "fp16"), (160, "fp16"), (1024, "bf16"), (16, "fp16")):
            x, q, s, z = w4a16_inputs(M, 1024, 1024, 128, dtype, seed=21 + M)
            xd, qd, sd, zd = (t.cuda() for t in (x, q, s, z))
            shards = [parallel.shard_weights(qd, sd, zd, world, r) for r in range(world)]
            expect = torch.cat([ops.w4a16_gemm(xd, *sh, 128) for sh in shards], dim=1)
            for _ in range(3):  # repeated calls reuse the buffers and pads
                y = mod(xd, *shards[rank])
            torch.cuda.synchronize()
            if not torch.equal(y, expect):
                raise AssertionError(f"rank {rank} M={M}: fused gather differs from per-shard GEMMs")
            gt = torch_ref_fp32(x, q, s, z, 128)
            err = (y.float().cpu() - gt).abs().max().item() / max(gt.abs().max().item(), 1e-6)
            worst = max(worst, err)
        if ops.device_status() != 0:
            raise AssertionError("device status set")
        q_out.put((rank, "ok", worst))
    except Exception as e:  # reported to the parent
        q_out.put((rank, repr(e), 0.0))
    finally:
        dist.destroy_process_group()


def test_two_gpu_fused_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, msg, worst in res:
        assert msg == "ok", f"rank {rank}: {msg}"
        assert worst < 2e-2


def test_mxfp8_peer_entry_single_gpu_offsets():
    from kernelbench_harbor_b200 import ops
    from tests.test_mxfp8 import _inputs
    for M in (128, 256):
        ac, asc, bc, bsc = (t.cuda() for t in _inputs(M, 512, 1024, seed=3 + M))
        ref = ops.mxfp8_gemm(ac, asc, bc, bsc)
        ya = torch.full((M, 1536), 7.0, dtype=torch.float16, device="cuda")
        yb = torch.full((M, 1536), -3.0, dtype=torch.float16, device="cuda")
        ops.mxfp8_gemm_peers(ac, asc, bc, bsc, [ya.data_ptr(), yb.data_ptr()], 1536, 512)
        torch.cuda.synchronize()
        for y in (ya, yb):
            assert torch.equal(y[:, 512:1024], ref)
            assert torch.all(y[:, :512] == 7.0 if y is ya else y[:, :512] == -3.0)
    assert ops.device_status() == 0


def _mxfp8_worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from kernelbench_harbor_b200 import ops, parallel
        from tests.test_mxfp8 import _inputs
        mod = parallel.PeerGatherMXFP8()
        for M, N in ((128, 1024), (512, 2048), (128, 1024)):
            ac, asc, bc, bsc = (t.cuda() for t in _inputs(M, N, 2048, seed=5 + M))
            n = N // world
            expect = torch.cat([ops.mxfp8_gemm(ac, asc, bc[r * n:(r + 1) * n].contiguous(),
                                               bsc[r * n:(r + 1) * n].contiguous()) for r in range(world)], dim=1)
            mine = (bc[rank * n:(rank + 1) * n].contiguous(), bsc[rank * n:(rank + 1) * n].contiguous())
            for _ in range(3):
                y = mod(ac, asc, *mine)
            torch.cuda.synchronize()
            if not torch.equal(y, expect):
                raise AssertionError(f"rank {rank} M={M}: fused gather differs from per-shard GEMMs")
        if ops.device_status() != 0:
            raise AssertionError("device status set")
        q_out.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q_out.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_gpu_mxfp8_fused_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mxfp8_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, msg in res:
        assert msg == "ok", f"rank {rank}: {msg}"
