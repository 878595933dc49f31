"""torch-CPU restatement of the reference modules' op sequences -- TEST/BASELINE ONLY.

Used as the timed CPU baseline (``bench.py`` ``cpu_baseline`` and
``--impl reference``): the reference cannot travel to the GPU box (it is a
Python checkout), so its ``Model.forward`` is restated here op for op, in the
same dtypes, so that its CPU cost is the reference's CPU cost.

* ``w4a16_forward``  -- QUANT_REF.forward, generate_tasks.py:54-61: unpack via
  int32 shifts [K, N/8, 8], cast to x.dtype, scales/zeros materialised to
  [K, N] by expand+reshape, (w - ze) * se, torch.matmul in x.dtype.
* ``w8a8_forward``   -- W8A8_REF.forward, generate_tasks.py:204-206.
"""
from __future__ import annotations

import torch


def w4a16_forward(x, qweight, scales, zeros, group: int):
    K = qweight.shape[0]
    N = qweight.shape[1] * 8
    shifts = torch.arange(0, 32, 4, device=x.device, dtype=torch.int32)
    w = ((qweight.unsqueeze(-1) >> shifts) & 0xF).reshape(K, N).to(x.dtype)
    g = K // group
    se = scales.reshape(g, 1, N).expand(g, group, N).reshape(K, N).to(x.dtype)
    ze = zeros.reshape(g, 1, N).expand(g, group, N).reshape(K, N).to(x.dtype)
    return torch.matmul(x, (w - ze) * se)


def w8a8_forward(x_int8, w_int8, x_scale, w_scale):
    acc = torch.matmul(x_int8.float(), w_int8.float())
    return (acc * x_scale.float() * w_scale.float()).to(torch.float16)
