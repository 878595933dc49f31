"""W8A8 GEMM: oracle pinned to the reference module's golden vectors (CPU) and
the tcgen05 kind::i8 kernel against the exact oracle (GPU)."""
import numpy as np
import pytest
import torch

from oracle import w8a8 as o
from tests.helpers import golden_cases

W8 = golden_cases("w8a8_")
TOL = dict(rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("path", W8, ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_reference(path):
    d = np.load(path)
    ym = o.forward_module(d["x_int8"], d["w_int8"], d["x_scale"], d["w_scale"])
    np.testing.assert_array_equal(ym, d["y_module"])
    ye = o.forward_exact(d["x_int8"], d["w_int8"], d["x_scale"], d["w_scale"])
    np.testing.assert_allclose(ye.astype(np.float32), d["y_fp32"], **TOL)


def test_smoothquant_prepare_shapes_and_ranges():
    from kernelbench_harbor_b200.quant import smoothquant_inputs
    xq, wq, xs, wsc, x, w = smoothquant_inputs(8, 256, 64, seed=1)
    assert xq.dtype == torch.int8 and wq.shape == (256, 64) and xs.shape == (8, 1) and wsc.shape == (1, 64)
    assert int(xq.abs().max()) <= 127 and int(wq.abs().max()) == 127
    # the quantised product approximates the fp32 product of the smoothed operands
    y = (xq.float() @ wq.float()) * xs.float() * wsc.float()
    ref = x.float() @ w.float().t()
    assert torch.linalg.norm(y - ref) / torch.linalg.norm(ref) < 0.05


@pytest.mark.gpu
@pytest.mark.parametrize("path", W8, ids=lambda p: p.split("/")[-1][:-4])
def test_gpu_golden(path):
    from kernelbench_harbor_b200 import ops
    d = np.load(path)
    args = [torch.from_numpy(d[k]).cuda() for k in ("x_int8", "w_int8", "x_scale", "w_scale")]
    y = ops.w8a8_gemm(*args).float().cpu().numpy()
    np.testing.assert_allclose(y, d["y_fp32"], **TOL)
    ye = o.forward_exact(d["x_int8"], d["w_int8"], d["x_scale"], d["w_scale"]).astype(np.float32)
    np.testing.assert_allclose(y, ye, rtol=2e-3, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(16, 14336, 4096), (512, 14336, 4096), (1, 4096, 6144), (33, 4096, 14336),
                                   (300, 3584, 18944), (16, 29568, 8192)])
def test_gpu_smoothquant_configs(M, K, N):
    from kernelbench_harbor_b200 import ops
    from kernelbench_harbor_b200.quant import smoothquant_inputs
    xq, wq, xs, wsc, _, _ = smoothquant_inputs(M, K, N, seed=M + N)
    y = ops.w8a8_gemm(xq.cuda(), wq.cuda(), xs.cuda(), wsc.cuda()).float().cpu().numpy()
    ye = o.forward_exact(xq.numpy(), wq.numpy(), xs.numpy(), wsc.numpy()).astype(np.float32)
    np.testing.assert_allclose(y, ye, rtol=2e-3, atol=2e-3)
    assert ops.device_status() == 0


@pytest.mark.gpu
def test_gpu_deterministic_split_k():
    from kernelbench_harbor_b200 import ops
    from kernelbench_harbor_b200.quant import smoothquant_inputs
    xq, wq, xs, wsc, _, _ = [t.cuda() for t in smoothquant_inputs(16, 14336, 4096, seed=3)]
    a = ops.w8a8_gemm(xq, wq, xs, wsc)
    b = ops.w8a8_gemm(xq, wq, xs, wsc)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_gpu_module_dropin():
    from kernelbench_harbor_b200.modules import W8A8Linear
    from kernelbench_harbor_b200.quant import smoothquant_inputs
    xq, wq, xs, wsc, _, _ = [t.cuda() for t in smoothquant_inputs(64, 4096, 4096, seed=4)]
    y = W8A8Linear()(xq, wq, xs, wsc)
    ye = o.forward_exact(xq.cpu().numpy(), wq.cpu().numpy(), xs.cpu().numpy(), wsc.cpu().numpy())
    np.testing.assert_allclose(y.float().cpu().numpy(), ye.astype(np.float32), rtol=2e-3, atol=2e-3)
