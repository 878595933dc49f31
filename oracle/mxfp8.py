"""Oracle for the MXFP8 block-scaled GEMM -- TEST INFRASTRUCTURE ONLY.

Parity: the reference has no MX module (its nearest is FP8_REF, a weight-only
fp8 GEMM with fp16 block scales, generate_tasks.py:218-237).  This restates
the OCP Microscaling (MX) v1.0 format the benchmark names: blocks of 32
consecutive K elements share one E8M0 scale 2^X, X = floor(log2(amax)) - 8
(8 = exponent of the largest e4m3 normal, 448), elements are v / 2^X rounded
to nearest-even e4m3 with saturation to +-448.  The e4m3 decode table and the
rounding are pinned against torch's float8_e4m3fn (an independent
implementation) and against the e4m3 code table of the reference FP8 module's
golden vectors; the GEMM is y = (A_deq . B_deq^T) in fp64, returned as fp32
(ground truth) or rounded to fp16.  Parity of the format itself is otherwise
unpinned: no reference output exists for it.
"""
from __future__ import annotations

import numpy as np


def e4m3_decode_table() -> np.ndarray:
    """fp32 value of each of the 256 e4m3fn codes (1-4-3, bias 7, no infinities,
    S.1111.111 = NaN)."""
    out = np.zeros(256, dtype=np.float32)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        e = (c >> 3) & 0xF
        m = c & 7
        if e == 15 and m == 7:
            out[c] = np.nan
        elif e == 0:
            out[c] = s * (m / 8.0) * 2.0 ** -6
        else:
            out[c] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return out


E4M3 = e4m3_decode_table()


def dequant(codes: np.ndarray, scales_e8m0: np.ndarray) -> np.ndarray:
    """codes uint8 [R, K], scales uint8 [R, K/32] -> fp64 [R, K]."""
    v = E4M3[np.asarray(codes, dtype=np.uint8)].astype(np.float64)
    s = np.exp2(np.asarray(scales_e8m0, dtype=np.float64) - 127.0)
    return v * np.repeat(s, 32, axis=1)


def gemm_fp32(a_codes, a_scales, b_codes, b_scales) -> np.ndarray:
    """y[M, N] = A . B^T with A [M, K], B [N, K] (both K-major)."""
    return (dequant(a_codes, a_scales) @ dequant(b_codes, b_scales).T).astype(np.float32)


def flops(M: int, N: int, K: int) -> int:
    return 2 * M * N * K


def algorithmic_bytes(M: int, N: int, K: int) -> int:
    return M * K + N * K + (M + N) * (K // 32) + 2 * M * N
