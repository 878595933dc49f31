"""Integer unpacking and dequantisation on the GPU, bit for bit.

The reference unpacks with an arithmetic shift and a 4-bit mask
(generate_tasks.py:55-57) and forms w = (nib - z) * s in the activation dtype
(:58-61).  With identity activations, y = I . W reads the dequantised weight
back through the whole kernel: the unpack, the zero subtraction and the
multiply by the scale.  Both kernels are checked: the decode kernel (M <= 16,
K read in slices of 16 identity rows) and the tcgen05 kernel (M = K >= 17).
The expected values are the reference module's own dequantised weights
(``w_dequant`` in the golden fixtures, made by tests/golden/make_golden.py
from the unmodified reference module) and, for the known-answer words
(0x80000000, 0xFFFFFFFF, 0x76543210, ...), the nibbles themselves."""
import numpy as np
import pytest
import torch

from tests.helpers import golden_cases, load_case, np_to_torch, tdt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import ops as _ops
    return _ops


def _read_back(ops, q, s, z, group, dtype, path):
    """W [K, N] as the kernel sees it, through identity activations."""
    K = q.shape[0]
    eye = torch.eye(K, dtype=tdt(dtype), device="cuda")
    if path == "tc":
        y = ops.w4a16_gemm(eye, q, s, z, group)
    else:
        y = torch.cat([ops.w4a16_gemm(eye[k0:k0 + 16].contiguous(), q, s, z, group) for k0 in range(0, K, 16)])
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return y


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy()


CASES = [p for p in golden_cases("w4a16_m16_k256_n128_")]


@pytest.mark.parametrize("path", ["decode", "tc"])
@pytest.mark.parametrize("case", CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_dequant_bit_exact(ops, case, path):
    d, m = load_case(case)
    dt = m["dtype"]
    q = np_to_torch(d["qweight"]).cuda()
    s = np_to_torch(d["scales"], dt).cuda()
    z = np_to_torch(d["zeros"], dt).cuda()
    w = _read_back(ops, q, s, z, m["group"], dt, path)
    expect = d["w_dequant"].view(np.int16)
    got = _bits(w)
    assert got.shape == expect.shape
    bad = np.argwhere(got != expect)
    assert bad.size == 0, f"{len(bad)} weights differ, first at {bad[0].tolist()}"


@pytest.mark.parametrize("path", ["decode", "tc"])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_unpack_known_answers(ops, path, dtype):
    d, _ = load_case(golden_cases("unpack_kat")[0])
    q = torch.from_numpy(d["qweight"].copy()).cuda()
    K, N = d["nib"].shape
    s = torch.ones(1, N, dtype=tdt(dtype), device="cuda")
    z = torch.zeros(1, N, dtype=tdt(dtype), device="cuda")
    w = _read_back(ops, q, s, z, K, dtype, path)
    assert torch.equal(w.float().cpu(), torch.from_numpy(d["nib"].astype(np.float32)))


@pytest.mark.parametrize("path", ["decode", "tc"])
def test_signed_words_with_zero_points(ops, path):
    """Words with the sign bit set: the arithmetic shift's sign extension is
    masked away, so the top nibble stays 8..15; every zero point 0..15."""
    K, N = 128, 256
    g = torch.Generator().manual_seed(7)
    nib = torch.randint(0, 16, (K, N), generator=g)
    nib[:, 7::8] = torch.randint(8, 16, (K, N // 8), generator=g)  # top nibble >= 8: negative int32
    packed = torch.zeros(K, N // 8, dtype=torch.int64)
    for i in range(8):
        packed |= nib[:, i::8] << (4 * i)
    q = packed.to(torch.int32).cuda()  # wraps to negative words
    assert int((q < 0).sum()) == K * N // 8
    z = (torch.arange(N) % 16).reshape(1, N).to(torch.float16).cuda()
    s = torch.full((1, N), 0.25, dtype=torch.float16).cuda()
    w = _read_back(ops, q, s, z, K, "fp16", path)
    expect = ((nib.float() - z.float().cpu()) * 0.25).to(torch.float16)
    assert torch.equal(w.cpu(), expect)
