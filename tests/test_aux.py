"""The rows next to the W4A16 path: GPU weight packer, fused SiLU * mul + fp8
quantisation (FUSED_SILU_REF), the quantised MoE drop-in for FUSED_QMOE_REF
(int8 symmetric weights) and the multi-LoRA quantised linear (LORA_REF).

CPU tests pin the oracles against the reference modules' golden vectors; GPU
tests compare the kernels with the oracles / golden vectors and with fp32
torch references at the benchmark configurations."""
import os

import numpy as np
import pytest
import torch

from oracle import lora as olora
from oracle import silu_fp8 as osilu
from oracle import w4a16 as o4
from oracle.w4a16 import bf16_bits_to_f32
from tests.conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _silu_cases():
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith("silu_fp8_"))


def _f32(arr, dtype):
    return bf16_bits_to_f32(arr) if dtype == "bf16" else arr.astype(np.float32)


def _fp8_close(got, want, scale_rows):
    """Equal to float32 rounding (a group's scale may differ in its last bit
    when exp does) except a small fraction of elements one e4m3 step apart
    (exp's last bit can move a value across an e4m3 rounding boundary)."""
    diff = np.abs(got - want)
    step = np.repeat(scale_rows, 128, axis=1) * 32.0  # > one e4m3 step at the top of the range
    assert np.all(diff <= step + 1e-12)
    assert np.mean(diff > 1e-6 * np.abs(want) + 1e-30) < 0.01


# ---------------------------------------------------------------- CPU: oracles vs golden
@pytest.mark.parametrize("name", _silu_cases())
def test_silu_fp8_oracle_matches_reference(name):
    d = _load(name)
    dtype = "bf16" if "bf16" in name else "fp16"
    y = _f32(d["y"], dtype)
    got = osilu.forward(y)
    H = y.shape[1] // 2
    amax = np.abs(d["out"].reshape(y.shape[0], H // 128, 128)).max(axis=-1) / 448.0
    _fp8_close(got, d["out"], amax)


def test_e4m3_round_ties_to_even():
    from oracle.mxfp8 import E4M3
    t = torch.tensor([0.0, 1.0625, 1.1875, 448.0, -0.001953125, 300.0, 17.0, 0.013671875])
    want = t.to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(osilu.e4m3_round(t.numpy()), want)
    assert np.isnan(E4M3[0x7F])


def test_lora_oracle_matches_reference():
    d = _load("lora_t16_d256_n128_r16.npz")
    got = olora.forward(d["x"], d["qweight"], d["scales"], d["A"], d["B"], d["lora_ids"])
    np.testing.assert_allclose(got.astype(np.float32), d["y_module"].astype(np.float32), rtol=2e-3, atol=2e-3)
    gt = olora.forward_fp32(d["x"], d["qweight"], d["scales"], d["A"], d["B"], d["lora_ids"])
    np.testing.assert_allclose(gt, d["y_fp32"], rtol=1e-4, atol=1e-4)


def test_signed_pack_is_offset_unsigned_pack():
    g = np.random.default_rng(3)
    q = g.integers(-8, 8, size=(16, 64))
    packed = o4.pack(q + 8)
    np.testing.assert_array_equal(o4.unpack(packed).astype(np.int64) - 8, q)


# ---------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(1, 8), (64, 256), (4096, 14336), (3, 1408)])
def test_pack_unsigned_bit_exact(K, N):
    from kernelbench_harbor_b200 import ops
    g = torch.Generator().manual_seed(K + N)
    nib = torch.randint(0, 16, (K, N), generator=g, dtype=torch.int64)
    got = ops.pack_int4(nib.to(torch.uint8).cuda(), offset=0).cpu().numpy()
    np.testing.assert_array_equal(got, o4.pack(nib.numpy()))
    assert ops.device_status() == 0


@pytest.mark.gpu
def test_pack_signed_and_range_status():
    from kernelbench_harbor_b200 import ops
    q = torch.randint(-8, 8, (32, 64), dtype=torch.int8)
    got = ops.pack_int4(q.cuda(), offset=8).cpu().numpy()
    np.testing.assert_array_equal(o4.unpack(got).astype(np.int64) - 8, q.numpy())
    assert ops.device_status() == 0
    bad = q.clone()
    bad[3, 5] = 9  # 9 + 8 does not fit 4 bits
    ops.pack_int4(bad.cuda(), offset=8)
    assert ops.device_status() & 2


@pytest.mark.gpu
@pytest.mark.parametrize("name", _silu_cases())
def test_silu_fp8_vs_reference_golden(name):
    from kernelbench_harbor_b200.modules import FusedSiluFp8
    d = _load(name)
    dtype = "bf16" if "bf16" in name else "fp16"
    if dtype == "bf16":
        y = torch.from_numpy(d["y"].view(np.int16)).view(torch.bfloat16)
    else:
        y = torch.from_numpy(d["y"])
    got = FusedSiluFp8()(y.cuda()).cpu().numpy()
    T, H = got.shape
    amax = np.abs(d["out"].reshape(T, H // 128, 128)).max(axis=-1) / 448.0
    _fp8_close(got, d["out"], amax)


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,dtype", [(256, 1408, torch.float16), (512, 2560, torch.float16),
                                       (512, 14336, torch.bfloat16)])
def test_silu_fp8_benchmark_configs(T, H, dtype):
    """The reference's configurations (generate_tasks.py:351-355): the kernel
    against the oracle, its codes / scales against the dequantised output, and
    cosine similarity with the unquantised activation (how the reference
    grades this family)."""
    from kernelbench_harbor_b200 import ops
    g = torch.Generator().manual_seed(T + H)
    y = torch.randn(T, 2 * H, generator=g).to(dtype)
    out, q, sc = ops.silu_mul_fp8(y.cuda(), codes=True)
    out, q, sc = out.cpu(), q.cpu(), sc.cpu()
    torch.testing.assert_close(out, (q.float().reshape(T, H // 128, 128) * sc[:, :, None]).reshape(T, H))
    want = osilu.forward(y.float().numpy())
    _fp8_close(out.numpy(), want, sc.numpy())
    yf = y.float()
    act = torch.nn.functional.silu(yf[:, :H]) * yf[:, H:]
    assert torch.nn.functional.cosine_similarity(out.flatten(), act.flatten(), dim=0).item() > 0.999


@pytest.mark.gpu
def test_fused_qmoe_vs_reference_golden():
    from kernelbench_harbor_b200.modules import FusedQMoE
    d = _load("moe_routing.npz")
    args = [torch.from_numpy(d[k]).cuda() for k in ("qmoe_x", "qmoe_qweight", "qmoe_scales", "qmoe_logits")]
    y = FusedQMoE()(*args).float().cpu().numpy()
    np.testing.assert_allclose(y, d["qmoe_y_fp32"], rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(y, d["qmoe_y_module"].astype(np.float32), rtol=1e-2, atol=1e-2)


def _qmoe_ref(x, qweight, scales, logits, module_rounding):
    """FUSED_QMOE_REF.forward on the GPU with fp32 arithmetic: as the grader's
    ground truth, or (module_rounding) rounding where the module in x.dtype
    rounds (dequantised weight, each expert output, the gated products and
    their sum)."""
    T, D = x.shape
    E, _, N = qweight.shape
    dt = x.dtype
    probs = torch.softmax(logits.float(), dim=-1)
    topv, topi = probs.topk(2, dim=-1)
    topv = topv / topv.sum(dim=-1, keepdim=True)
    w = (qweight.reshape(E, D // 128, 128, N).float() * scales.float()[:, :, None, :]).reshape(E, D, N)
    if module_rounding:
        w = w.to(dt).float()
        topv = topv.to(dt).float()
    sel = torch.zeros(T, 2, N, device=x.device)
    for k in range(2):
        for e in range(E):
            rows = torch.nonzero(topi[:, k] == e).flatten()
            if rows.numel():
                o = x[rows].float() @ w[e]
                sel[rows, k] = o.to(dt).float() if module_rounding else o
    if not module_rounding:
        return (sel * topv[:, :, None]).sum(dim=1)
    p = (sel * topv[:, :, None]).to(dt).float()
    return (p[:, 0] + p[:, 1]).to(dt).float()


@pytest.mark.gpu
@pytest.mark.parametrize("D,E,N,dtype", [(2048, 64, 1408, torch.float16), (4096, 8, 14336, torch.float16),
                                         (2048, 60, 1408, torch.bfloat16)])
def test_fused_qmoe_benchmark_configs(D, E, N, dtype):
    from kernelbench_harbor_b200.modules import FusedQMoE
    torch.backends.cuda.matmul.allow_tf32 = False
    T = 256
    g = torch.Generator().manual_seed(D + E)
    x = torch.randn(T, D, generator=g).to(dtype).cuda()
    qweight = torch.randint(-8, 8, (E, D, N), generator=g, dtype=torch.int8).cuda()
    scales = (torch.randn(E, D // 128, N, generator=g) * 0.01).to(dtype).cuda()
    logits = torch.randn(T, E, generator=g).to(dtype).cuda()
    y = FusedQMoE()(x, qweight, scales, logits).float()
    ref_mod = _qmoe_ref(x, qweight, scales, logits, True)
    # bf16: the two gated products are rounded to 8 significant bits before
    # their sum, so where they cancel one ulp of a product (of the size of
    # the largest outputs) is the resolution; fp16 keeps the plain 1e-2
    atol = 1e-2 * max(1.0, ref_mod.abs().max().item()) if dtype == torch.bfloat16 else 1e-2
    torch.testing.assert_close(y, ref_mod, rtol=1e-2, atol=atol)
    ref32 = _qmoe_ref(x, qweight, scales, logits, False)
    tol = 3e-2 if dtype == torch.bfloat16 else 1e-2
    torch.testing.assert_close(y, ref32, rtol=tol, atol=max(tol, atol))


@pytest.mark.gpu
def test_lora_vs_reference_golden():
    from kernelbench_harbor_b200.modules import MultiLoRAW4
    d = _load("lora_t16_d256_n128_r16.npz")
    args = [torch.from_numpy(d[k]).cuda() for k in ("x", "qweight", "scales", "A", "B", "lora_ids")]
    y = MultiLoRAW4()(*args).float().cpu().numpy()
    np.testing.assert_allclose(y, d["y_fp32"], rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(y, d["y_module"].astype(np.float32), rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("D,N,r,L,dtype", [(4096, 4096, 16, 8, torch.float16), (3584, 3584, 32, 8, torch.float16),
                                           (4096, 4096, 64, 4, torch.bfloat16)])
def test_lora_benchmark_configs(D, N, r, L, dtype):
    from kernelbench_harbor_b200 import ops
    from kernelbench_harbor_b200.modules import MultiLoRAW4
    torch.backends.cuda.matmul.allow_tf32 = False
    T = 64
    g = torch.Generator().manual_seed(D + r)
    x = torch.randn(T, D, generator=g).to(dtype).cuda()
    qweight = torch.randint(-8, 8, (D, N), generator=g, dtype=torch.int8).cuda()
    scales = (torch.randn(D // 128, N, generator=g) * 0.01).to(dtype).cuda()
    A = (torch.randn(L, D, r, generator=g) * 0.02).to(dtype).cuda()
    B = (torch.randn(L, r, N, generator=g) * 0.02).to(dtype).cuda()
    ids = torch.randint(0, L, (T,), generator=g).cuda()
    ids[0] = L - 1
    y = MultiLoRAW4()(x, qweight, scales, A, B, ids).float()
    w = (qweight.float().reshape(D // 128, 128, N) * scales.float()[:, None, :]).reshape(D, N)
    ref = x.float() @ w + torch.einsum("tr,trn->tn", torch.einsum("td,tdr->tr", x.float(), A[ids].float()),
                                       B[ids].float())
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-2
    torch.testing.assert_close(y, ref, rtol=tol, atol=tol)
    assert ops.device_status() == 0
    bad = ids.clone()
    bad[5] = L  # out of range: status bit, the token gets the base product only
    ops.lora_shrink(x, A, bad)
    assert ops.device_status() & 2
