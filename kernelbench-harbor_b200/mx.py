"""OCP Microscaling (MX v1.0) FP8 quantiser for the MXFP8 GEMM's inputs.

Blocks of 32 consecutive elements along the last axis share one E8M0 scale
2^X with X = floor(log2(amax)) - 8 (8 = exponent of e4m3's largest normal,
448); elements are v / 2^X rounded to nearest even in e4m3 and saturated to
+-448.  Returns (codes uint8 [R, K], scales uint8 [R, K/32], biased by 127).
"""
from __future__ import annotations

import torch

E4M3_EMAX = 8


def quantize_mxfp8(v: torch.Tensor):
    R, K = v.shape
    if K % 32:
        raise ValueError("K must be a multiple of 32")
    vf = v.float().reshape(R, K // 32, 32)
    amax = vf.abs().amax(dim=-1)
    # exact floor(log2(amax)) from the fp32 exponent field (amax = 0 -> smallest scale)
    bits = amax.view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 127
    x = torch.where(amax > 0, e - E4M3_EMAX, torch.full_like(e, -127))
    x = x.clamp(-127, 127)
    scale = torch.exp2(x.float())
    q = (vf / scale.unsqueeze(-1)).clamp(-448.0, 448.0)
    codes = q.to(torch.float8_e4m3fn).view(torch.uint8).reshape(R, K)
    return codes.contiguous(), (x + 127).to(torch.uint8).contiguous()


def dequantize_mxfp8(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    v = codes.view(torch.float8_e4m3fn).float()
    s = torch.exp2(scales.float() - 127.0)
    return v * s.repeat_interleave(32, dim=-1)
