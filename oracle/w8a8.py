"""numpy oracle for the W8A8 GEMM -- TEST INFRASTRUCTURE ONLY.

Restates W8A8_REF.forward (generate_tasks.py:204-206):
    acc = x_int8.float() @ w_int8.float();  y = (acc * x_scale * w_scale).to(fp16)
``forward_exact`` forms the integer product exactly (float64 holds it exactly), then applies the
scales in fp64 and rounds once to fp16 -- the value the reference's fp32
matmul approximates (its fp32 accumulation of products up to 14336 * 127^2
rounds).  ``forward_module`` reproduces the fp32 accumulation order-free
(float32 matmul) for comparison with the golden vectors.
"""
from __future__ import annotations

import numpy as np


def forward_exact(x_int8, w_int8, x_scale, w_scale) -> np.ndarray:
    # int8 x int8 products summed over K < 2^38 are integers below 2^53, so a
    # float64 (BLAS) product is exact -- the same value as an int64 product
    acc = np.asarray(x_int8, dtype=np.float64) @ np.asarray(w_int8, dtype=np.float64)
    xs = np.asarray(x_scale, dtype=np.float16).astype(np.float64).reshape(-1, 1)
    ws = np.asarray(w_scale, dtype=np.float16).astype(np.float64).reshape(1, -1)
    return (acc.astype(np.float64) * xs * ws).astype(np.float32).astype(np.float16)


def forward_module(x_int8, w_int8, x_scale, w_scale) -> np.ndarray:
    acc = np.asarray(x_int8, dtype=np.float32) @ np.asarray(w_int8, dtype=np.float32)
    xs = np.asarray(x_scale, dtype=np.float16).astype(np.float32).reshape(-1, 1)
    ws = np.asarray(w_scale, dtype=np.float16).astype(np.float32).reshape(1, -1)
    return (acc * xs * ws).astype(np.float16)


def algorithmic_bytes(M: int, N: int, K: int) -> int:
    return M * K + K * N + 2 * M + 2 * N + 2 * M * N
