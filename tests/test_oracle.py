"""The numpy oracle against the reference's own outputs (golden fixtures made
by tests/golden/make_golden.py from the reference modules)."""
import numpy as np
import pytest
import torch

from oracle import w4a16 as o
from tests.helpers import golden_cases, load_case, torch_ref_fp32, np_to_torch

W4 = golden_cases("w4a16_")


def test_golden_fixtures_present():
    assert len(W4) >= 7


@pytest.mark.parametrize("path", W4, ids=lambda p: p.split("/")[-1][:-4])
def test_pack_unpack_bit_exact(path):
    d, m = load_case(path)
    assert (o.unpack(d["qweight"]) == d["nib"]).all()
    assert (o.pack(d["nib"]) == d["qweight"]).all()


@pytest.mark.parametrize("path", W4, ids=lambda p: p.split("/")[-1][:-4])
def test_dequant_matches_reference_module_bits(path):
    d, m = load_case(path)
    w = o.dequant(d["qweight"], d["scales"], d["zeros"], m["group"], m["dtype"])
    ref = o.to_f32(d["w_dequant"], m["dtype"])
    # identical values (the reference's identity-matmul readback turns -0 into +0)
    assert np.array_equal(w, ref)


@pytest.mark.parametrize("path", W4, ids=lambda p: p.split("/")[-1][:-4])
def test_forward_matches_reference(path):
    d, m = load_case(path)
    args = (d["x"], d["qweight"], d["scales"], d["zeros"], m["group"], m["dtype"])
    y32 = o.forward_fp32(*args)
    np.testing.assert_allclose(y32, d["y_fp32"], rtol=1e-5, atol=1e-4)
    ym = o.to_f32(o.forward_module(*args), m["dtype"])
    ref = o.to_f32(d["y_module"], m["dtype"])
    # one rounding of differently-ordered fp32 sums: at most one output ulp apart
    big = np.maximum(np.abs(ym), np.abs(ref))
    ulp = np.spacing(big.astype(np.float16)).astype(np.float32) if m["dtype"] == "fp16" else big * 2.0 ** -7
    assert (np.abs(ym - ref) <= ulp * 1.0001).all()


def test_unpack_kat():
    d = np.load(golden_cases("unpack_kat")[0])
    assert (o.unpack(d["qweight"]) == d["nib"]).all()
    # explicit words: sign bit, all ones, ascending nibbles
    q = np.array([[np.uint32(0x80000000).view(np.int32), np.uint32(0xFFFFFFFF).view(np.int32),
                   np.int32(0x76543210)]], dtype=np.int32)
    u = o.unpack(q)
    assert list(u[0, :8]) == [0, 0, 0, 0, 0, 0, 0, 8]
    assert list(u[0, 8:16]) == [15] * 8
    assert list(u[0, 16:24]) == list(range(8))


def test_torch_fp32_reference_matches_oracle():
    """The torch fp32 helper used by the full-size GPU tests agrees with the
    oracle (checked on the CPU)."""
    for path in W4[:4]:
        d, m = load_case(path)
        if m["dtype"] != "fp16":
            continue
        y = torch_ref_fp32(np_to_torch(d["x"]), np_to_torch(d["qweight"]), np_to_torch(d["scales"]),
                           np_to_torch(d["zeros"]), m["group"]).numpy()
        np.testing.assert_allclose(y, d["y_fp32"], rtol=1e-5, atol=1e-4)


def test_algorithmic_bytes_matches_benchmark_figure():
    assert o.algorithmic_bytes(16, 4096, 14336, 128) == 31_784_960
    assert o.flops(4096, 4096, 14336) == 481_036_337_152
