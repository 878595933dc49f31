"""b200q: B200-native (sm_100a) quantised dequant-GEMM library.

Drop-in replacement for the hot path of lilian-muyaoli/kernelbench-harbor's
``quant_w4a16_pa`` task family (QUANT_REF, generate_tasks.py:45-74) and its
siblings.  Python is the host side only: every op calls the C-ABI shared
library ``libb200q.so`` (include/b200q.h) built from ``csrc/`` for sm_100a.
"""
from .build import LIB, build  # noqa: F401

__all__ = ["build", "LIB"]


def __getattr__(name):
    # lazy: importing the package must not require CUDA or the built library
    if name in ("ops", "modules", "_lib", "parallel"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    if name in ("ModelNew", "W4A16Linear"):
        from . import modules
        return getattr(modules, name)
    raise AttributeError(name)
