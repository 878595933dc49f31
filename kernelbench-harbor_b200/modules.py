"""Drop-in replacements for the reference operator modules.

``ModelNew`` keeps the reference contract (common/kb_verifier.py:186-201): a
constructor without arguments and ``forward`` with exactly the signature of the
reference ``Model.forward``, returning the same shape.  The group size of the
reference module is a module constant (``GROUP``, generate_tasks.py:48); here it
is recovered from the scales' shape, so one class serves the g64 and g128
tasks.  Output dtype is x's dtype, as the reference module returns."""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops


class W4A16Linear(nn.Module):
    """Packed-asymmetric W4A16 (GPTQ-style) linear: QUANT_REF.forward,
    generate_tasks.py:54-61.  x:[..., K]; qweight:[K, N//8] int32;
    scales, zeros:[K//GROUP, N]."""

    def forward(self, x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                zeros: torch.Tensor) -> torch.Tensor:
        K = qweight.shape[0]
        if scales.shape[0] == 0 or K % scales.shape[0]:
            raise ValueError(f"scales rows ({scales.shape[0]}) must divide K ({K})")
        group = K // scales.shape[0]
        lead = x.shape[:-1]
        y = ops.w4a16_gemm(x.reshape(-1, K), qweight, scales, zeros, group)
        return y.reshape(*lead, y.shape[-1])


class W8A8Linear(nn.Module):
    """W8A8 SmoothQuant linear: W8A8_REF.forward, generate_tasks.py:204-206.
    x_int8:[M,K] int8; w_int8:[K,N] int8; x_scale:[M,1] fp16; w_scale:[1,N]
    fp16; returns fp16 [M,N]."""

    def forward(self, x_int8, w_int8, x_scale, w_scale):
        return ops.w8a8_gemm(x_int8, w_int8, x_scale, w_scale)


# the reference harness imports the replacement as ``ModelNew``
ModelNew = W4A16Linear
