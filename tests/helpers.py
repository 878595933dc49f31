"""Shared test helpers: seeded input builders (the reference recipe of
QUANT_REF.get_inputs, generate_tasks.py:63-73, on a seeded generator) and a
torch fp32 reference of the same op for sizes the numpy oracle is too slow for."""
from __future__ import annotations

import glob
import json
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = dict(rtol=1e-2, atol=1e-2)  # the benchmark's stated allclose tolerance for fp16 outputs


def golden_cases(prefix: str):
    return sorted(glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def load_case(path: str):
    d = dict(np.load(path))
    meta = json.loads(str(d.pop("meta"))) if "meta" in d else {}
    return d, meta


def np_to_torch(a: np.ndarray, dtype: str | None = None) -> torch.Tensor:
    if dtype == "bf16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a).copy())


def tdt(dtype: str) -> torch.dtype:
    return {"fp16": torch.float16, "bf16": torch.bfloat16}[dtype]


def w4a16_inputs(M, K, N, group=128, dtype="fp16", seed=0, device="cpu", dist="bj"):
    g = torch.Generator().manual_seed(seed)
    nib = torch.randint(0, 16, (K, N), generator=g, dtype=torch.int64)
    packed = torch.zeros(K, N // 8, dtype=torch.int64)
    for i in range(8):
        packed |= nib[:, i::8] << (4 * i)
    qweight = packed.to(torch.int32)
    x = torch.randn(M, K, generator=g).to(tdt(dtype))
    if dist == "bj":
        scales = (torch.rand(K // group, N, generator=g) * 0.018 + 0.002).to(tdt(dtype))
    else:
        scales = (torch.randn(K // group, N, generator=g) * 0.01).to(tdt(dtype))
    zeros = torch.randint(0, 16, (K // group, N), generator=g).to(tdt(dtype))
    return [t.to(device) for t in (x, qweight, scales, zeros)]


def torch_ref_fp32(x, qweight, scales, zeros, group):
    """fp32 ground truth in torch, any device: unpack by arithmetic shift and
    mask (generate_tasks.py:55-57), (w - z) * s in fp32, fp32 matmul."""
    K = qweight.shape[0]
    N = qweight.shape[1] * 8
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int32)
    w = ((qweight.unsqueeze(-1) >> shifts) & 0xF).reshape(K, N).float()
    g = K // group
    s = scales.float().reshape(g, 1, N).expand(g, group, N).reshape(K, N)
    z = zeros.float().reshape(g, 1, N).expand(g, group, N).reshape(K, N)
    wd = (w - z) * s
    if x.is_cuda:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            return x.float() @ wd
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
    return x.float() @ wd


def torch_ref_module(x, qweight, scales, zeros, group):
    """The reference module's own numerics (generate_tasks.py:55-61): the
    dequantised weight is rounded to x.dtype exactly as QUANT_REF does it
    ((w - ze) then * se, each in x.dtype); the product accumulates in fp32 and
    is returned in fp32 (before the module's final rounding to x.dtype)."""
    K = qweight.shape[0]
    N = qweight.shape[1] * 8
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int32)
    w = ((qweight.unsqueeze(-1) >> shifts) & 0xF).reshape(K, N).to(x.dtype)
    g = K // group
    se = scales.reshape(g, 1, N).expand(g, group, N).reshape(K, N).to(x.dtype)
    ze = zeros.reshape(g, 1, N).expand(g, group, N).reshape(K, N).to(x.dtype)
    wd = ((w - ze) * se).float()
    if x.is_cuda:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            return x.float() @ wd
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
    return x.float() @ wd


def check_w4a16(y, x, qweight, scales, zeros, group):
    """fp16: allclose(1e-2) against the fp32 ground truth.  bf16 through the
    decode kernel (M <= 16), which applies the scales in fp32: allclose(1e-2)
    against the fp32 ground truth as well.  bf16 through the tensor-core kernel,
    which rounds each weight to bf16 (8 significant bits) exactly as the
    reference module does: allclose(1e-2) against that module's numerics and,
    against the fp32 ground truth, allclose(5e-2) with the absolute part
    growing as sqrt(K / 4096) (independent weight roundings add up as a random
    walk over the K products: at K = 29568 the module itself is ~0.09 off)."""
    ref32 = torch_ref_fp32(x, qweight, scales, zeros, group)
    if x.dtype == torch.float16 or x.shape[0] < 17:
        torch.testing.assert_close(y.float(), ref32, **TOL)
    else:
        torch.testing.assert_close(y.float(), torch_ref_module(x, qweight, scales, zeros, group), **TOL)
        K = x.shape[1]
        torch.testing.assert_close(y.float(), ref32, rtol=5e-2, atol=5e-2 * max(1.0, (K / 4096) ** 0.5))


def torch_dequant_fp32(qweight, scales, zeros, group):
    """fp32 weight [K, N] = (unpack(qweight) - z) * s (generate_tasks.py:55-61 in fp32)."""
    K = qweight.shape[0]
    N = qweight.shape[1] * 8
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int32)
    w = ((qweight.unsqueeze(-1) >> shifts) & 0xF).reshape(K, N).float()
    g = K // group
    s = scales.float().reshape(g, 1, N).expand(g, group, N).reshape(K, N)
    z = zeros.float().reshape(g, 1, N).expand(g, group, N).reshape(K, N)
    return (w - z) * s
