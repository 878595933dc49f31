"""MXFP8 block-scaled GEMM (tcgen05 kind::mxf8f6f4.block_scale) against the
fp64 oracle of the same OCP-MX operands.  The quantiser is pinned against the
e4m3 code table of the reference FP8 module's golden vectors and torch's
float8_e4m3fn."""
import numpy as np
import pytest
import torch

from oracle import mxfp8 as o
from tests.helpers import golden_cases

TOL = dict(rtol=1e-2, atol=1e-2)


def test_e4m3_table_matches_reference_golden():
    d = np.load(golden_cases("fp8_block32")[0])
    t = d["e4m3_table"]
    assert np.array_equal(np.nan_to_num(t, nan=1234.0), np.nan_to_num(o.E4M3, nan=1234.0))


def test_quantizer_blocks_and_saturation():
    from kernelbench_harbor_b200.mx import dequantize_mxfp8, quantize_mxfp8
    g = torch.Generator().manual_seed(0)
    v = torch.randn(16, 256, generator=g)
    v[0, :32] = 0.0          # all-zero block
    v[1, 5] = 1e4            # one large outlier in a block
    c, s = quantize_mxfp8(v)
    assert c.shape == (16, 256) and s.shape == (16, 8)
    dq = dequantize_mxfp8(c, s)
    assert np.allclose(o.dequant(c.numpy(), s.numpy()), dq.numpy())
    assert dq[0, :32].abs().max() == 0
    # per block: |element| <= 448 * scale and relative error of e4m3 rounding
    blk = v.reshape(16, 8, 32)
    rel = ((dq.reshape(16, 8, 32) - blk).abs() / blk.abs().amax(-1, keepdim=True).clamp(min=1e-30)).max()
    assert rel < 2 ** -3


def _inputs(M, N, K, seed):
    from kernelbench_harbor_b200.mx import quantize_mxfp8
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).half()
    b = (torch.randn(N, K, generator=g) * 0.02).half()
    return (*quantize_mxfp8(a), *quantize_mxfp8(b))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (128, 4096, 14336), (4096, 4096, 14336), (1, 512, 256),
                                   (200, 768, 1024), (128, 96, 512)])
def test_gpu_mxfp8_vs_oracle(M, N, K):
    from kernelbench_harbor_b200 import ops
    ac, asc, bc, bsc = _inputs(M, N, K, seed=M + N + K)
    y = ops.mxfp8_gemm(ac.cuda(), asc.cuda(), bc.cuda(), bsc.cuda()).float()
    if M * N * K <= 128 * 4096 * 14336:
        ref = torch.from_numpy(o.gemm_fp32(ac.numpy(), asc.numpy(), bc.numpy(), bsc.numpy()))
    else:
        from kernelbench_harbor_b200.mx import dequantize_mxfp8
        torch.backends.cuda.matmul.allow_tf32 = False
        ref = (dequantize_mxfp8(ac.cuda(), asc.cuda()) @ dequantize_mxfp8(bc.cuda(), bsc.cuda()).t()).cpu()
    torch.testing.assert_close(y.cpu(), ref, **TOL)
    assert ops.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 4096, 14336), (128, 512, 4096)])
def test_gpu_mxfp8_split_k_deterministic(M, N, K):
    """Split-K tiles (few tiles, long K) are reduced over DSMEM in rank order:
    repeated calls give identical bits."""
    from kernelbench_harbor_b200 import ops
    ac, asc, bc, bsc = (t.cuda() for t in _inputs(M, N, K, seed=77))
    ys = [ops.mxfp8_gemm(ac, asc, bc, bsc) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    assert ops.device_status() == 0
