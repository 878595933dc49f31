"""Oracle for the fused SiLU * mul + per-group fp8 quantisation -- TEST
INFRASTRUCTURE ONLY (imported by tests and never by the product).

Restates FUSED_SILU_REF.forward (generate_tasks.py:332-346) in numpy:
act = silu(gate) * up in float32 (silu(g) = g / (1 + exp(-g))); per group of
128 columns scale = max(amax(|act|) / 448, 1e-12); q = e4m3(clamp(act / scale,
+-448)) rounded to nearest, ties to even; returns q * scale (float32).  Pinned
against the reference module's outputs in tests/golden/silu_fp8_*.npz.  The
exp of numpy and of the GPU may differ in the last bit, which can move a value
across an e4m3 rounding boundary: comparisons allow one e4m3 step on a small
fraction of elements (the reference's own oracle notes the same,
common/oracles/fused_silu_fp8.py:7-10).
"""
from __future__ import annotations

import numpy as np

from oracle.mxfp8 import E4M3

GROUP = 128
FP8_MAX = np.float32(448.0)

_FINITE = np.array([c for c in range(256) if not np.isnan(E4M3[c])], dtype=np.int64)
_ORDER = np.argsort(E4M3[_FINITE], kind="stable")
_VALS = E4M3[_FINITE][_ORDER].astype(np.float64)
_CODES = _FINITE[_ORDER]


def e4m3_round(v: np.ndarray) -> np.ndarray:
    """Nearest e4m3 value (ties to the even code), v already within +-448."""
    v = np.asarray(v, dtype=np.float64)
    i = np.clip(np.searchsorted(_VALS, v), 1, len(_VALS) - 1)
    lo, hi = _VALS[i - 1], _VALS[i]
    pick_hi = (hi - v) < (v - lo)
    tie = (hi - v) == (v - lo)
    hi_even = (_CODES[i] & 1) == 0
    pick_hi = pick_hi | (tie & hi_even)
    return np.where(pick_hi, hi, lo).astype(np.float32)


def forward(y: np.ndarray) -> np.ndarray:
    """y [T, 2H] float32 (the fp16/bf16 input upcast) -> float32 [T, H]."""
    y = np.asarray(y, dtype=np.float32)
    T, H2 = y.shape
    H = H2 // 2
    gate, up = y[:, :H], y[:, H:]
    act = (gate / (np.float32(1.0) + np.exp(-gate))) * up
    a = act.reshape(T, H // GROUP, GROUP)
    scale = np.maximum(np.abs(a).max(axis=-1, keepdims=True) / FP8_MAX, np.float32(1e-12)).astype(np.float32)
    q = e4m3_round(np.clip(a / scale, -FP8_MAX, FP8_MAX))
    return (q * scale).reshape(T, H).astype(np.float32)
