"""C-ABI library: builds, loads, exports every symbol include/b200q.h
declares, and rejects bad arguments before touching a GPU."""
import ctypes
import os
import re

import pytest

import kernelbench_harbor_b200 as pkg
from kernelbench_harbor_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for f in os.listdir(os.path.join(REPO, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(REPO, "include", f)).read()
            syms |= set(re.findall(r"\b(b200q_\w+)\s*\(", src))
    return sorted(syms)


@pytest.fixture(scope="module")
def L():
    pkg.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    syms = declared_symbols()
    assert "b200q_w4a16_gemm" in syms
    for s in syms:
        assert hasattr(L, s), s
    # and the ctypes table covers exactly the header
    assert set(_lib.SIGNATURES) == set(syms)


def test_version(L):
    assert L.b200q_version() >= 1


def _call(L, M=16, N=4096, K=14336, group=128, dtype=0, ws_bytes=1 << 20, ptr=16):
    return L.b200q_w4a16_gemm(ptr, ptr, ptr, ptr, ptr, M, N, K, group, dtype, ptr, ws_bytes, None)


@pytest.mark.parametrize("kw,code", [
    (dict(group=100), _lib.ERR_UNSUPPORTED),
    (dict(dtype=7), _lib.ERR_UNSUPPORTED),
    (dict(N=4100), _lib.ERR_ALIGN),
    (dict(K=200), _lib.ERR_SHAPE),
    (dict(M=-1), _lib.ERR_SHAPE),
])
def test_argument_errors(L, kw, code):
    assert _call(L, **kw) == code
    assert L.b200q_last_error()


def test_empty_m_is_noop(L):
    assert _call(L, M=0) == _lib.OK


def test_workspace_size_monotone(L):
    a = L.b200q_w4a16_workspace_bytes(16, 4096, 14336, 128, 0)
    b = L.b200q_w4a16_workspace_bytes(1, 256, 128, 128, 0)
    assert a >= 256 and b >= 256


def test_python_errors_without_gpu():
    import torch
    from kernelbench_harbor_b200 import ops
    x = torch.zeros(4, 128, dtype=torch.float16)
    q = torch.zeros(128, 4, dtype=torch.int32)
    s = torch.zeros(1, 32, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.w4a16_gemm(x, q, s, s, 128)
