"""Oracle for the multi-LoRA quantised linear -- TEST INFRASTRUCTURE ONLY.

Restates LORA_REF.forward (generate_tasks.py:405-414) in numpy with the
module's rounding points in the activation dtype: w = q * s (one rounding),
base = x @ w, lo = x @ A[id] and lo @ B[id] each rounded, y = base + lo
rounded; products accumulate in float64 here (the module accumulates in fp32
inside its matmuls, so the two agree to the output rounding).  Pinned against
the reference module's outputs in tests/golden/lora_*.npz.
"""
from __future__ import annotations

import numpy as np

GROUP = 128


def forward(x16, qweight, scales16, A16, B16, ids) -> np.ndarray:
    """fp16 arrays (float16 dtype) and int8 qweight / int ids -> float16 [T, N]."""
    D, N = qweight.shape
    w = (qweight.astype(np.float16).reshape(D // GROUP, GROUP, N) * scales16[:, None, :]).reshape(D, N)
    x = x16.astype(np.float64)
    base = (x @ w.astype(np.float64)).astype(np.float16)
    lo = np.einsum("td,tdr->tr", x, A16[ids].astype(np.float64)).astype(np.float16)
    lo2 = np.einsum("tr,trn->tn", lo.astype(np.float64), B16[ids].astype(np.float64)).astype(np.float16)
    return (base.astype(np.float32) + lo2.astype(np.float32)).astype(np.float16)


def forward_fp32(x, qweight, scales, A, B, ids) -> np.ndarray:
    """Ground truth (float inputs upcast, common/kb_verifier.py:194-196)."""
    D, N = qweight.shape
    w = (qweight.astype(np.float64).reshape(D // GROUP, GROUP, N) * scales.astype(np.float64)[:, None, :]).reshape(D, N)
    x = x.astype(np.float64)
    lo = np.einsum("td,tdr->tr", x, A[ids].astype(np.float64))
    return (x @ w + np.einsum("tr,trn->tn", lo, B[ids].astype(np.float64))).astype(np.float32)
