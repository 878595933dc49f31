"""Expert-parallel quantised MoE on two GPUs (NCCL all-to-all dispatch and
return, local experts as grouped W4A16 GEMMs): each rank's output equals the
single-GPU grouped module on the same tokens bit for bit (every row's
arithmetic is the same kernel over the same weights in the same K order).
Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(E, D, H, G, seed):
    from tests.helpers import w4a16_inputs
    out = []
    for (k, n, off) in ((D, H, 0), (D, H, 1), (H, D, 2)):
        qs, ss, zs = [], [], []
        for e in range(E):
            _, q, s, z = w4a16_inputs(1, k, n, G, "fp16", seed=seed + 10 * e + off)
            qs.append(q), ss.append(s), zs.append(z)
        out += [torch.stack(qs), torch.stack(ss), torch.stack(zs)]
    return out


def _worker(rank, world, port, q_out, padded=True):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from kernelbench_harbor_b200 import parallel
        from kernelbench_harbor_b200.modules import QuantizedMoE
        T, D, H, E, G = 256, 512, 1024, 8, 128
        gen = torch.Generator().manual_seed(31)
        x = torch.randn(T, D, generator=gen).half().cuda()
        logits = torch.randn(T, E, generator=gen).half().cuda()
        w = [t.cuda() for t in _weights(E, D, H, G, 70)]
        ref = QuantizedMoE()(x, logits, *w)
        tl = T // world
        mine = slice(rank * tl, (rank + 1) * tl)
        epr = E // world
        local_w = [t[rank * epr:(rank + 1) * epr].contiguous() for t in w]
        mod = parallel.ExpertParallelMoE(E, padded=padded)
        for _ in range(2):
            y = mod(x[mine].contiguous(), logits[mine].contiguous(), local_w)
        torch.cuda.synchronize()
        if not torch.equal(y, ref[mine]):
            d = (y.float() - ref[mine].float()).abs().max().item()
            raise AssertionError(f"rank {rank}: EP output differs from single-GPU (max {d})")
        q_out.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q_out.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("padded", [True, False])
def test_ep_moe_two_gpus(padded):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out, padded)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, msg in res:
        assert msg == "ok", f"rank {rank}: {msg}"
