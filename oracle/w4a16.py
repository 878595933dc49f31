"""numpy oracle for the packed-asymmetric W4A16 group-quantised GEMM.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates QUANT_REF of
lilian-muyaoli/kernelbench-harbor, ``generate_tasks.py:45-74``:

* ``pack``      -- ``get_inputs`` packer, ``generate_tasks.py:65-69``:
                   ``packed[k, j] |= nib[k, 8j+i] << 4i`` in int64, then
                   truncated to int32 (nibble 7 >= 8 makes the word negative).
* ``unpack``    -- ``Model.forward`` unpack, ``generate_tasks.py:55-57``:
                   arithmetic ``>>`` of the signed int32 word by 0,4,..,28 then
                   ``& 0xF``; nibble i of word [k, j] is column 8j+i.
* ``dequant``   -- ``generate_tasks.py:58-61``: scale and zero rows repeated
                   GROUP times along K, ``(w - ze) * se`` evaluated in the
                   activation dtype, one rounding per op (what torch's CPU and
                   CUDA elementwise kernels do).
* ``forward_module`` -- the reference module's output in x's dtype: the
                   dequantised weight in x.dtype, then an fp32-accumulated
                   product rounded once to x.dtype.
* ``forward_fp32`` -- the grader's ground truth, ``common/kb_verifier.py:194-196``:
                   floating inputs upcast to fp32, integer tensors unchanged,
                   the same module evaluated in fp32 (accumulated here in fp64).

Everything works on numpy arrays; bf16 data is carried as ``uint16`` bit
patterns (numpy has no bfloat16) and converted with round-to-nearest-even.
"""
from __future__ import annotations

import numpy as np

SHIFTS = np.arange(0, 32, 4, dtype=np.int32)


# ----------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 (NaN kept quiet)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    out[nan] = 0x7FC0
    return out


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """Activation-dtype array (fp16 array or bf16 bit pattern) -> fp32."""
    if dtype == "bf16":
        return bf16_bits_to_f32(a)
    return np.asarray(a, dtype=np.float16).astype(np.float32)


def round_to(a32: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> activation dtype (fp16 array or bf16 bit pattern)."""
    if dtype == "bf16":
        return f32_to_bf16_bits(a32)
    return np.asarray(a32, dtype=np.float32).astype(np.float16)


# ----------------------------------------------------------------- packing
def pack(nib: np.ndarray) -> np.ndarray:
    """nib [K, N] in 0..15 -> qweight int32 [K, N//8] (generate_tasks.py:65-69)."""
    nib = np.asarray(nib, dtype=np.int64)
    K, N = nib.shape
    if N % 8:
        raise ValueError("N must be a multiple of 8")
    packed = np.zeros((K, N // 8), dtype=np.int64)
    for i in range(8):
        packed |= nib[:, i::8] << (4 * i)
    # torch's int64 -> int32 .to() keeps the low 32 bits (two's complement)
    return (packed & 0xFFFFFFFF).astype(np.uint32).view(np.int32)


def unpack(qweight: np.ndarray) -> np.ndarray:
    """qweight int32 [K, N//8] -> uint8 [K, N] (generate_tasks.py:55-57)."""
    q = np.asarray(qweight, dtype=np.int32)
    K = q.shape[0]
    w = (q[..., None] >> SHIFTS) & 0xF  # arithmetic shift on signed int32, then mask
    return w.reshape(K, q.shape[1] * 8).astype(np.uint8)


# ----------------------------------------------------------------- dequant / forward
def _expand_groups(a: np.ndarray, group: int, K: int) -> np.ndarray:
    g = K // group
    return np.repeat(a.reshape(g, 1, -1), group, axis=1).reshape(K, -1)


def dequant(qweight, scales, zeros, group: int, dtype: str = "fp16") -> np.ndarray:
    """fp32 view of the weight the reference module multiplies by, after its
    dtype roundings: w.to(dt) exact, (w - ze) rounded to dt, (*se) rounded to dt."""
    K = qweight.shape[0]
    if K % group:
        raise ValueError("K must be a multiple of the group size")
    w = unpack(qweight).astype(np.float32)
    se = _expand_groups(to_f32(scales, dtype), group, K)
    ze = _expand_groups(to_f32(zeros, dtype), group, K)
    d = to_f32(round_to(w - ze, dtype), dtype)
    return to_f32(round_to(d * se, dtype), dtype)


def dequant_fp32(qweight, scales, zeros, group: int, dtype: str = "fp16") -> np.ndarray:
    """The ground-truth weight: same formula evaluated in fp32 (no dt rounding)."""
    K = qweight.shape[0]
    w = unpack(qweight).astype(np.float32)
    se = _expand_groups(to_f32(scales, dtype), group, K)
    ze = _expand_groups(to_f32(zeros, dtype), group, K)
    return (w - ze) * se


def forward_module(x, qweight, scales, zeros, group: int, dtype: str = "fp16") -> np.ndarray:
    """Reference module output in x's dtype (fp32 accumulation, one final rounding)."""
    w = dequant(qweight, scales, zeros, group, dtype).astype(np.float64)
    y = to_f32(x, dtype).astype(np.float64) @ w
    return round_to(y.astype(np.float32), dtype)


def forward_fp32(x, qweight, scales, zeros, group: int, dtype: str = "fp16") -> np.ndarray:
    """Grader ground truth (common/kb_verifier.py:194-196), accumulated in fp64."""
    w = dequant_fp32(qweight, scales, zeros, group, dtype).astype(np.float64)
    return (to_f32(x, dtype).astype(np.float64) @ w).astype(np.float32)


def algorithmic_bytes(M: int, N: int, K: int, group: int, act_bytes: int = 2) -> int:
    """Bytes one call must move at minimum: packed weight, scales, zeros, x, y."""
    return K * N // 2 + 2 * (K // group) * N * act_bytes + M * K * act_bytes + M * N * act_bytes


def flops(M: int, N: int, K: int) -> int:
    return 2 * M * N * K
