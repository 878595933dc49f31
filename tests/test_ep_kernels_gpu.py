"""The expert-parallel exchange kernels (ep_pack, ep_regroup, ep_gather) on
one GPU: two ranks are emulated by exchanging the send buffers' blocks by
hand, and every row is checked against the routing (which token, which local
expert, which slot), the regrouping against a stable sort by expert, and the
gathers both ways."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("P,E,T", [(2, 8, 64), (4, 8, 32), (8, 8, 16), (2, 64, 40)])
def test_ep_exchange_kernels(dtype, P, E, T):
    from kernelbench_harbor_b200 import ops
    D, C, epr = 256, 2 * T, E // P
    g = torch.Generator(device="cuda").manual_seed(P * 100 + E + T)
    xs = [torch.randn(T, D, generator=g, device="cuda").to(dtype) for _ in range(P)]
    lg = [torch.randn(T, E, generator=g, device="cuda").to(dtype) for _ in range(P)]
    sends, slots, routes = [], [], []
    for r in range(P):
        topi, gates, offsets, slot_token, token_slot = ops.moe_route(lg[r])
        send, pair_slot = ops.ep_pack(xs[r], offsets, slot_token, token_slot, E, P, C)
        sends.append(send), slots.append(pair_slot), routes.append(topi)
        # every routed pair sits in the slot pair_slot names, with its local expert id
        for t in range(T):
            for k in range(2):
                s = int(pair_slot[t, k])
                e = int(topi[t, k])
                assert s // C == e // epr
                assert torch.equal(send[s, :D], xs[r][t])
                assert int(send[s, D].float()) == e - (e // epr) * epr
        # empty slots carry -1
        ids = send[:, D].float().long().cpu()
        assert int((ids >= 0).sum()) == 2 * T
    for d in range(P):
        recv = torch.cat([sends[s][d * C:(d + 1) * C] for s in range(P)])
        loc, src, pos = ops.ep_regroup(recv, epr)
        ids = recv[:, D].float().long()
        real = (ids >= 0).nonzero().flatten()
        order = real[torch.argsort(ids[real], stable=True)]
        n = order.numel()
        assert int(loc[-1]) == n
        assert torch.equal(src[:n].long(), order) and bool((src[n:] == -1).all())
        assert torch.equal(torch.bincount(ids[real], minlength=epr).cumsum(0).int(), loc[1:])
        for j, r in enumerate(order.tolist()):
            assert int(pos[r]) == j
        assert bool((pos[ids < 0] == -1).all())
        rows = torch.zeros((P * C, D), dtype=dtype, device="cuda")
        ops.ep_gather(recv, src, D, rows)
        assert torch.equal(rows[:n], recv[order, :D])
        back = torch.zeros((P * C, D), dtype=dtype, device="cuda")
        ops.ep_gather(rows, pos, D, back)
        assert torch.equal(back[real], recv[real, :D])
    assert ops.device_status() == 0
