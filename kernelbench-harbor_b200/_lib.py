"""ctypes binding of libb200q.so (declarations mirror include/b200q.h).

The library is loaded from this package directory only.  There is no CPU or
pure-PyTorch fallback: if the shared object is missing, every op raises."""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB

OK = 0
ERR_SHAPE = -1
ERR_ALIGN = -2
ERR_UNSUPPORTED = -3
ERR_CUDA = -4
ERR_WORKSPACE = -5
ERR_DEVICE = -6

DTYPE_FP16 = 0
DTYPE_BF16 = 1

_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p
_c_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol include/b200q.h declares
SIGNATURES = {
    "b200q_version": (ctypes.c_int, []),
    "b200q_last_error": (ctypes.c_char_p, []),
    "b200q_workspace_status": (ctypes.c_int, [_c_vp, _c_vp]),
    "b200q_set_weight_prefetch": (ctypes.c_int, [ctypes.c_int]),
    "b200q_w4a16_workspace_bytes": (_c_sz, [_c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "b200q_w4a16_gemm": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                        ctypes.c_int, _c_vp, _c_sz, _c_vp]),
    "b200q_w8a8_workspace_bytes": (_c_sz, [_c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "b200q_w8a8_gemm": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_sz,
                                       _c_vp]),
    "b200q_mxfp8_workspace_bytes": (_c_sz, [_c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "b200q_mxfp8_gemm": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_sz,
                                        _c_vp]),
    "b200q_moe_route": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                                       _c_vp]),
    "b200q_moe_gather": (ctypes.c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp]),
    "b200q_ep_pack": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64,
                                     _c_i64, _c_vp, _c_vp, _c_vp]),
    "b200q_ep_regroup": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, ctypes.c_int, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp]),
    "b200q_ep_gather": (ctypes.c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_vp]),
    "b200q_silu_mul": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_i64, ctypes.c_int, _c_vp]),
    "b200q_moe_combine": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_int, _c_vp]),
    "b200q_w4a16_gemm_noalloc": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64,
                                                _c_i64, ctypes.c_int, _c_vp]),
    "b200q_w4a16_noalloc_status": (ctypes.c_int, [_c_vp]),
    "b200q_w4a16_gemm_peers": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, ctypes.c_int, _c_i64, _c_i64,
                                              _c_vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                              _c_vp, _c_sz, _c_vp]),
    "b200q_moe_grouped_gemm": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64,
                                              _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_vp, _c_sz,
                                              _c_vp]),
    "b200q_pack_int4": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, ctypes.c_int, _c_vp, _c_vp, _c_vp]),
    "b200q_silu_mul_fp8": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, ctypes.c_int, _c_vp, _c_vp, _c_vp, _c_vp]),
    "b200q_lora_shrink": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_vp,
                                         _c_vp, _c_vp]),
    "b200q_lora_expand_add": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                             ctypes.c_int, _c_vp, _c_vp]),
    "b200q_mxfp8_gemm_peers": (ctypes.c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, ctypes.c_int, _c_i64, _c_i64,
                                              _c_vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_vp, _c_sz, _c_vp]),
    "b200q_peer_barrier": (ctypes.c_int, [_c_vp, ctypes.c_int, ctypes.c_int, _c_vp, _c_vp]),
    "b200q_set_peer_barrier_timeout_ms": (_c_i64, [_c_i64]),
}

_lock = threading.Lock()
_lib = None


class B200QError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"b200q error {code}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB):
                    raise ImportError(
                        f"{LIB} is missing: build it with `python -m kernelbench_harbor_b200.build` "
                        "(there is no fallback implementation)")
                h = ctypes.CDLL(LIB)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def check(code: int) -> None:
    if code != OK:
        msg = lib().b200q_last_error().decode(errors="replace")
        raise B200QError(code, msg)
