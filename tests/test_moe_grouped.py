"""Grouped expert GEMM (all experts in one launch, rows grouped by the routing
kernel) and its fused SiLU * mul epilogue.

* the fused gate/up launch equals the unfused grouped gate and up GEMMs
  followed by silu_mul (same rounding points; the unfused launches may
  split K, so up to one rounding of g and u apart);
* every expert's rows of the grouped GEMM match that expert's plain W4A16
  GEMM against the fp32 ground truth (oracle restatement of the dequant);
* ragged and skewed groupings: empty experts, one expert taking every row,
  row counts that are not multiples of the 128-row tile, bf16, group 32 / 64
  (two scale rows per 64-deep stage);
* split-K grouped launches (few expert tiles, long K) are deterministic;
* the grouped MoE module equals the per-expert (unfused) module within the
  rounding of the split-K reductions the per-expert path may choose.
"""
import pytest
import torch

from tests.helpers import torch_ref_fp32, w4a16_inputs

pytestmark = pytest.mark.gpu


def _stacked(E, K, N, group, dtype, seed):
    qs, ss, zs = [], [], []
    for e in range(E):
        _, q, s, z = w4a16_inputs(1, K, N, group, dtype, seed=seed + e)
        qs.append(q)
        ss.append(s)
        zs.append(z)
    return [torch.stack(t).cuda() for t in (qs, ss, zs)]


def _offsets(counts):
    off = [0]
    for c in counts:
        off.append(off[-1] + c)
    return torch.tensor(off, dtype=torch.int32, device="cuda")


CASES = [
    # counts per expert, K, N, group, dtype
    ([130, 0, 7, 256, 129, 1, 0, 64], 512, 768, 128, "fp16"),
    ([0, 0, 0, 300], 256, 512, 64, "fp16"),
    ([17, 33, 1, 128], 1024, 256, 32, "bf16"),
    ([128] * 8, 4096, 1024, 128, "fp16"),
    # one expert with ~128 rows and a long K (an expert-parallel rank's down
    # projection): the grouped launch splits K over a cluster
    ([120], 14336, 4096, 128, "fp16"),
    # an expert-parallel rank of 2: four experts of ~256 rows (two 128-row
    # blocks per tile), long K, a 2-way split
    ([250, 262, 238, 274], 14336, 4096, 128, "fp16"),
]


@pytest.mark.parametrize("counts,K,N,group,dtype", CASES)
def test_grouped_matches_per_expert_ground_truth(counts, K, N, group, dtype):
    from kernelbench_harbor_b200 import ops
    E, rows = len(counts), sum(counts)
    x, _, _, _ = w4a16_inputs(rows, K, 32, group, dtype, seed=7)
    x = x.cuda()
    q, s, z = _stacked(E, K, N, group, dtype, seed=100)
    off = _offsets(counts)
    y = ops.moe_grouped_gemm(x, off, q, s, z, group)
    torch.cuda.synchronize()
    o = off.tolist()
    for e in range(E):
        if counts[e] == 0:
            continue
        xe = x[o[e]:o[e + 1]]
        gt = torch_ref_fp32(xe.cpu(), q[e].cpu(), s[e].cpu(), z[e].cpu(), group)
        ye = y[o[e]:o[e + 1]].float().cpu()
        tol = 2e-2 if dtype == "bf16" else 1e-2
        scale = gt.abs().max().item()
        assert (ye - gt).abs().max().item() <= tol * max(scale, 1.0), f"expert {e}"
        # and the plain GEMM on the same rows agrees to its rounding
        yp = ops.w4a16_gemm(xe, q[e], s[e], z[e], group).float().cpu()
        assert (ye - yp).abs().max().item() <= tol * max(scale, 1.0)


@pytest.mark.parametrize("counts,K,N,group,dtype", CASES)
def test_fused_glu_bit_exact_vs_unfused(counts, K, N, group, dtype):
    from kernelbench_harbor_b200 import ops
    E, rows = len(counts), sum(counts)
    x, _, _, _ = w4a16_inputs(rows, K, 32, group, dtype, seed=8)
    x = x.cuda()
    gq, gs, gz = _stacked(E, K, N, group, dtype, seed=200)
    uq, us, uz = _stacked(E, K, N, group, dtype, seed=300)
    off = _offsets(counts)
    h = ops.moe_grouped_gemm(x, off, gq, gs, gz, group, up=(uq, us, uz))
    hg = ops.moe_grouped_gemm(x, off, gq, gs, gz, group)
    hu = ops.moe_grouped_gemm(x, off, uq, us, uz, group)
    ref = ops.silu_mul(hg, hu)
    torch.cuda.synchronize()
    # the unfused grouped GEMMs may split K over a cluster (few expert tiles)
    # where the fused gate/up launch does not: the fp32 sums then differ in
    # order, so g and u can differ by one rounding; otherwise the two are the
    # same arithmetic
    top = ref.float().abs().max().item()
    torch.testing.assert_close(h.float(), ref.float(), rtol=5e-3, atol=5e-3 * max(top, 1.0))
    assert ops.device_status() == 0


def test_grouped_moe_module_vs_per_expert():
    from kernelbench_harbor_b200.modules import QuantizedMoE
    T, D, H, E, G = 200, 1024, 2048, 8, 128
    gen = torch.Generator().manual_seed(13)
    x = torch.randn(T, D, generator=gen).half().cuda()
    logits = torch.randn(T, E, generator=gen).half().cuda()
    gq, gs, gz = _stacked(E, D, H, G, "fp16", seed=400)
    uq, us, uz = _stacked(E, D, H, G, "fp16", seed=500)
    dq, ds, dz = _stacked(E, H, D, G, "fp16", seed=600)
    args = (x, logits, gq, gs, gz, uq, us, uz, dq, ds, dz)
    y = QuantizedMoE(grouped=True)(*args).float()
    yr = QuantizedMoE(grouped=False)(*args).float()
    torch.testing.assert_close(y, yr, rtol=1e-2, atol=1e-2 * yr.abs().mean().item())


def test_grouped_moe_cuda_graph():
    """No host synchronisation inside the grouped forward: it captures."""
    from kernelbench_harbor_b200.modules import QuantizedMoE
    T, D, H, E, G = 64, 512, 1024, 4, 128
    gen = torch.Generator().manual_seed(14)
    x = torch.randn(T, D, generator=gen).half().cuda()
    logits = torch.randn(T, E, generator=gen).half().cuda()
    w = _stacked(E, D, H, G, "fp16", 1) + _stacked(E, D, H, G, "fp16", 2) + _stacked(E, H, D, G, "fp16", 3)
    mod = QuantizedMoE()
    y0 = mod(x, logits, *w)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y1 = mod(x, logits, *w)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


def test_grouped_split_k_deterministic():
    from kernelbench_harbor_b200 import ops
    x, _, _, _ = w4a16_inputs(120, 14336, 32, 128, "fp16", seed=9)
    q, s, z = _stacked(1, 14336, 4096, 128, "fp16", seed=300)
    off = _offsets([120])
    ys = [ops.moe_grouped_gemm(x.cuda(), off, q, s, z, 128) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    assert ops.device_status() == 0
