"""W4A16 dequant-GEMM on the GPU through the C ABI, against the oracle.

Tolerance: allclose(rtol=1e-2, atol=1e-2) against the fp32 ground truth (the
benchmark's stated bar), plus a tighter check against the oracle's
reference-module output (same fp16 dequantised weight, fp32 accumulation)."""
import numpy as np
import pytest
import torch

from oracle import w4a16 as o
from tests.helpers import TOL, check_w4a16, golden_cases, load_case, np_to_torch, torch_ref_fp32, w4a16_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import ops as _ops
    return _ops


def _run(ops, x, q, s, z, group):
    y = ops.w4a16_gemm(x, q, s, z, group)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return y


@pytest.mark.parametrize("path", golden_cases("w4a16_"), ids=lambda p: p.split("/")[-1][:-4])
def test_golden(ops, path):
    d, m = load_case(path)
    if m["N"] % 32:
        pytest.skip("N not a multiple of 32")
    dt = m["dtype"]
    x, q, s, z = (np_to_torch(d[k], dt if k in ("x", "scales", "zeros") else None).cuda()
                  for k in ("x", "qweight", "scales", "zeros"))
    y = _run(ops, x, q, s, z, m["group"]).float().cpu().numpy()
    assert y.shape == (m["M"], m["N"])
    np.testing.assert_allclose(y, d["y_fp32"], **TOL)
    ym = o.to_f32(d["y_module"], dt)
    # the module rounds each weight to x's dtype before an fp32-accumulated
    # matmul; the kernels keep (nib - z) * s in fp32 (decode) or round it the
    # same way (tensor-core path): within a few output ulps of the module
    top = float(np.abs(ym).max())
    ulp = 2.0 ** (np.floor(np.log2(top)) - (10 if dt == "fp16" else 7))
    assert np.abs(y - ym).max() <= 4 * ulp + 1e-3


@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 31, 32, 33, 64, 100])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_ragged_m(ops, M, dtype):
    x, q, s, z = w4a16_inputs(M, 1024, 512, 128, dtype, seed=M, device="cuda")
    y = _run(ops, x, q, s, z, 128)
    assert y.dtype == x.dtype
    if dtype == "fp16":
        ref = o.forward_fp32(x.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy(), z.cpu().numpy(), 128)
        np.testing.assert_allclose(y.float().cpu().numpy(), ref, **TOL)
    check_w4a16(y, x, q, s, z, 128)


@pytest.mark.parametrize("group", [32, 64, 128, 256])
def test_groups(ops, group):
    x, q, s, z = w4a16_inputs(16, 2048, 768, group, "fp16", seed=group, device="cuda")
    y = _run(ops, x, q, s, z, group)
    ref = torch_ref_fp32(x, q, s, z, group)
    torch.testing.assert_close(y.float(), ref, **TOL)


@pytest.mark.parametrize("K,N", [(128, 32), (384, 96), (4096, 14336), (14336, 4096), (3584, 18944),
                                 (29568, 8192)])
def test_reference_layer_shapes(ops, K, N):
    x, q, s, z = w4a16_inputs(16, K, N, 128, "fp16", seed=K + N, device="cuda")
    y = _run(ops, x, q, s, z, 128)
    torch.testing.assert_close(y.float(), torch_ref_fp32(x, q, s, z, 128), **TOL)


# the reference's whole W4A16 task grid (generate_tasks.py:480-489, 534-541):
# every layer at g64 fp16, g128 fp16 and g128 bf16, decode M=16
LAYERS = [(4096, 14336), (14336, 4096), (8192, 28672), (28672, 8192), (3584, 18944), (18944, 3584),
          (8192, 29568), (29568, 8192)]


def _gpu_inputs(M, K, N, group, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nib = torch.randint(0, 16, (K, N), generator=g, device="cuda", dtype=torch.int32)
    q = torch.zeros(K, N // 8, dtype=torch.int32, device="cuda")
    for i in range(8):
        q |= nib[:, i::8] << (4 * i)
    dt = torch.float16 if dtype == "fp16" else torch.bfloat16
    x = torch.randn(M, K, generator=g, device="cuda").to(dt)
    s = (torch.rand(K // group, N, generator=g, device="cuda") * 0.018 + 0.002).to(dt)
    z = torch.randint(0, 16, (K // group, N), generator=g, device="cuda").to(dt)
    return x, q, s, z


@pytest.mark.parametrize("K,N", LAYERS)
@pytest.mark.parametrize("group,dtype", [(64, "fp16"), (128, "fp16"), (128, "bf16")])
def test_reference_task_grid(ops, K, N, group, dtype):
    x, q, s, z = _gpu_inputs(16, K, N, group, dtype, seed=K * 7 + N + group)
    y = _run(ops, x, q, s, z, group)
    check_w4a16(y, x, q, s, z, group)


def test_benchmark_decode_config_vs_oracle(ops):
    """The benchmark's decode configuration: M=16, K=14336, N=4096, g128, against the numpy oracle."""
    x, q, s, z = w4a16_inputs(16, 14336, 4096, 128, "fp16", seed=1016, device="cuda")
    y = _run(ops, x, q, s, z, 128).float().cpu().numpy()
    ref = o.forward_fp32(x.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy(), z.cpu().numpy(), 128)
    np.testing.assert_allclose(y, ref, **TOL)


def test_reference_scale_distribution(ops):
    """The reference's own get_inputs draws scales as randn*0.01 (signed)."""
    x, q, s, z = w4a16_inputs(16, 14336, 4096, 128, "fp16", seed=5, device="cuda", dist="ref")
    y = _run(ops, x, q, s, z, 128)
    torch.testing.assert_close(y.float(), torch_ref_fp32(x, q, s, z, 128), **TOL)


def test_deterministic_and_workspace_reusable(ops):
    x, q, s, z = w4a16_inputs(16, 14336, 4096, 128, "fp16", seed=9, device="cuda")
    a = _run(ops, x, q, s, z, 128)
    b = _run(ops, x, q, s, z, 128)
    assert torch.equal(a, b)


def test_empty_m(ops):
    x, q, s, z = w4a16_inputs(0, 256, 64, 128, "fp16", device="cuda")
    y = ops.w4a16_gemm(x, q, s, z, 128)
    assert y.shape == (0, 64)


def test_module_dropin(ops):
    from kernelbench_harbor_b200.modules import ModelNew
    x, q, s, z = w4a16_inputs(16, 1024, 256, 64, "fp16", seed=3, device="cuda")
    y = ModelNew()(x, q, s, z)
    torch.testing.assert_close(y.float(), torch_ref_fp32(x, q, s, z, 64), **TOL)


@pytest.mark.parametrize("M,K,N,group,dtype", [
    (128, 14336, 4096, 128, "fp16"),   # the benchmark's M=128 sweep point (split-K tiles)
    (256, 1024, 512, 128, "fp16"),
    (300, 2048, 768, 64, "fp16"),      # ragged M tile, ragged N tile (768 = 3 x 256)
    (129, 4096, 1024, 32, "bf16"),
    (512, 4096, 1024, 256, "bf16"),
    (1024, 14336, 4096, 128, "fp16"),  # the benchmark's M=1024 sweep point
])
def test_tensor_core_path(ops, M, K, N, group, dtype):
    x, q, s, z = w4a16_inputs(M, K, N, group, dtype, seed=M + K, device="cuda")
    y = _run(ops, x, q, s, z, group)
    check_w4a16(y, x, q, s, z, group)


@pytest.mark.parametrize("M,K,N,group,dtype", [
    (768, 2048, 4096, 128, "fp16"),    # 48 256-row tiles x 3-way split
    (1000, 4096, 4096, 64, "bf16"),    # ragged 256-row tiles, 2-way split
    (1024, 1024, 4096, 32, "fp16"),    # short K, two scale rows per stage
    (300, 2048, 768, 128, "fp16"),     # ragged rows and columns, 8-way (or as co-resident) split
])
def test_split_256_row_tiles(ops, M, K, N, group, dtype):
    """256-row tiles whose K ranges form a cluster: the partial tiles are
    reduced over DSMEM in two passes of one 128-row block, with uneven row
    ownership when the cluster size does not divide 128."""
    x, q, s, z = w4a16_inputs(M, K, N, group, dtype, seed=M + N, device="cuda")
    y = _run(ops, x, q, s, z, group)
    check_w4a16(y, x, q, s, z, group)
    y2 = _run(ops, x, q, s, z, group)
    assert torch.equal(y, y2)  # deterministic reduction order
    ws = ops.workspace(torch.device("cuda", torch.cuda.current_device()), 0)
    torch.cuda.synchronize()
    assert int(ws.count_nonzero()) == 0, "the split left the workspace dirty"


def test_tensor_core_full_config(ops):
    """The benchmark's compute-bound configuration, M=4096, against the fp32 torch reference."""
    x, q, s, z = w4a16_inputs(4096, 14336, 4096, 128, "fp16", seed=4096, device="cuda")
    y = _run(ops, x, q, s, z, 128)
    torch.testing.assert_close(y.float(), torch_ref_fp32(x, q, s, z, 128), **TOL)


def test_workspace_left_zeroed(ops):
    """Every kernel returns the workspace it used to zero, so kernels of
    different shapes can share it (decode split-K slots, tensor-core split-K
    accumulator and tickets)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    for M in (16, 128, 5, 200):
        x, q, s, z = w4a16_inputs(M, 4096, 1024, 128, "fp16", seed=M, device="cuda")
        _run(ops, x, q, s, z, 128)
        ws = ops.workspace(dev, 0)
        torch.cuda.synchronize()
        assert int(ws.count_nonzero()) == 0, f"workspace dirty after M={M}"
