"""Weight / activation quantisers that produce the inputs of the sibling ops.

The reference modules take already-quantised tensors; the benchmark describes
how they are made.  These builders are part of the library so a caller can go
from fp16 activations and fp16 master weights to the ops' inputs.

* ``smoothquant_prepare`` -- W8A8 SmoothQuant (alpha = 0.5): per input channel
  j, s_j = max|x_j|^0.5 / max|W_j|^0.5; x' = x / s, W' = W * s; dynamic
  per-token symmetric int8 for x' (scale = max|x'_m| / 127, round half to even,
  clamp to +-127) and per-output-channel symmetric int8 for W'.  Computed in
  fp32; scales are returned in fp16 as the W8A8 op consumes them.
"""
from __future__ import annotations

import torch


def _sym_int8(a: torch.Tensor, dim: int):
    amax = a.abs().amax(dim=dim, keepdim=True).clamp(min=1e-8)
    scale = amax / 127.0
    q = torch.round(a / scale).clamp(-127, 127).to(torch.int8)  # torch.round: half to even
    return q, scale


def smoothquant_prepare(x: torch.Tensor, w_master_nk: torch.Tensor, alpha: float = 0.5):
    """x [M, K] (fp16/fp32), w_master_nk [N, K] (output rows, input columns).
    Returns x_int8 [M, K], x_scale [M, 1] fp16, w_int8 [K, N], w_scale [1, N] fp16."""
    xf = x.float()
    wf = w_master_nk.float()
    xmax = xf.abs().amax(dim=0).clamp(min=1e-5)
    wmax = wf.abs().amax(dim=0).clamp(min=1e-5)
    s = xmax.pow(alpha) / wmax.pow(1.0 - alpha)
    xq, xs = _sym_int8(xf / s, dim=1)
    wkn = (wf * s).t().contiguous()  # [K, N]
    wq, wsc = _sym_int8(wkn, dim=0)
    return xq, xs.to(torch.float16), wq.contiguous(), wsc.to(torch.float16)


def smoothquant_inputs(M: int, K: int, N: int, seed: int = 0, device="cpu", outlier_frac: float = 0.01):
    """The benchmark's W8A8 inputs: x fp16 N(0,1) with 1% of channels x20,
    master weight fp16 N(0, 0.02) [N, K], quantised by ``smoothquant_prepare``.
    Also returns the fp16 x and master weight."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    n_out = max(1, int(round(K * outlier_frac)))
    idx = torch.randperm(K, generator=g)[:n_out]
    x[:, idx] *= 20.0
    x = x.to(torch.float16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.float16)
    xq, xs, wq, wsc = smoothquant_prepare(x, w)
    return [t.to(device) for t in (xq, wq, xs, wsc)] + [x.to(device), w.to(device)]
