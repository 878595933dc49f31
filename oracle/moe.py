"""numpy oracle for top-2 routing and the quantised MoE FFN -- TEST INFRASTRUCTURE ONLY.

* ``route`` restates the routing of MOE_REF / FUSED_QMOE_REF
  (generate_tasks.py:171-173 and 368-371): softmax of the fp32-upcast logits,
  the two largest probabilities, renormalised, cast to the logits' dtype.  On
  exact ties torch.topk's order is implementation-defined; this oracle (and the
  library) take the lower expert index first.
* ``ffn_fp32`` is the ground truth of the composite FFN: per token and each of
  its two experts, SiLU(x Wg) * (x Wu) (FUSED_SILU_REF, :336-337) then . Wd,
  gated sum (:377-378), all in fp32 with the W4A16 weights dequantised in fp32
  (oracle.w4a16.dequant_fp32).
"""
from __future__ import annotations

import numpy as np

from . import w4a16


def route(logits: np.ndarray):
    l = np.asarray(logits, dtype=np.float32)
    order = np.argsort(-l, axis=1, kind="stable")[:, :2]
    m = l.max(axis=1, keepdims=True)
    e = np.exp((l - m).astype(np.float64))
    p = e / e.sum(axis=1, keepdims=True)
    topv = np.take_along_axis(p, order, axis=1)
    gates = (topv / topv.sum(axis=1, keepdims=True)).astype(np.float32)
    return order.astype(np.int32), gates


def ffn_fp32(x, logits, experts, group):
    """experts: list of E tuples (gq, gs, gz, uq, us, uz, dq, ds, dz) as numpy."""
    topi, gates = route(logits)
    xf = np.asarray(x, dtype=np.float32).astype(np.float64)
    T, D = xf.shape
    y = np.zeros((T, D), dtype=np.float64)
    cache = {}
    for e in np.unique(topi):
        gq, gs, gz, uq, us, uz, dq, ds, dz = experts[e]
        wg = w4a16.dequant_fp32(gq, gs.astype(np.float32), gz.astype(np.float32), group)
        wu = w4a16.dequant_fp32(uq, us.astype(np.float32), uz.astype(np.float32), group)
        wd = w4a16.dequant_fp32(dq, ds.astype(np.float32), dz.astype(np.float32), group)
        cache[e] = (wg.astype(np.float64), wu.astype(np.float64), wd.astype(np.float64))
    for t in range(T):
        for k in range(2):
            wg, wu, wd = cache[topi[t, k]]
            a = xf[t] @ wg
            h = a / (1.0 + np.exp(-a)) * (xf[t] @ wu)
            y[t] += gates[t, k] * (h @ wd)
    return y.astype(np.float32)
