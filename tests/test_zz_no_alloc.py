"""The allocation-free entry point, b200q_w4a16_gemm_noalloc.

It exists for callers that cannot allocate device memory (a plugin inside a
host program that owns every allocation, a fixed memory budget): they pass only
inputs and outputs, and the kernel's scratch is a fixed array inside the
library.  This test calls it through the C ABI twice in a row (the array keeps
the previous call's contents) and checks each result against the regular
workspace entry point, with the tolerance the other tests use.  It sits in a
file collected last and works alone or after the other tests."""
import pytest
import torch

from tests.helpers import TOL, w4a16_inputs

pytestmark = pytest.mark.gpu


def _noalloc(L, x, q, s, z, group):
    M, K = x.shape
    N = q.shape[1] * 8
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    dt = 0 if x.dtype == torch.float16 else 1
    rc = L.b200q_w4a16_gemm_noalloc(x.data_ptr(), q.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                    M, N, K, group, dt, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.b200q_last_error().decode()
    return y


def test_noalloc_matches_workspace_entry_point_twice():
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import _lib, ops
    L = _lib.lib()
    for seed, (M, K, N, dtype) in enumerate([(16, 14336, 4096, "fp16"), (5, 4096, 1024, "bf16")]):
        x, q, s, z = w4a16_inputs(M, K, N, 128, dtype, seed=100 + seed, device="cuda")
        ref = ops.w4a16_gemm(x, q, s, z, 128)
        y1 = _noalloc(L, x, q, s, z, 128)
        y2 = _noalloc(L, x, q, s, z, 128)
        torch.cuda.synchronize()
        torch.testing.assert_close(y1.float(), ref.float(), **TOL)
        torch.testing.assert_close(y2.float(), ref.float(), **TOL)


def test_noalloc_rejects_oversize():
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import _lib
    L = _lib.lib()
    dev = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = dev.data_ptr()
    assert L.b200q_w4a16_gemm_noalloc(p, p, p, p, p, 64, 4096, 4096, 128, 0, None) == _lib.ERR_SHAPE
    assert b"M must be" in L.b200q_last_error()
    # scratch need beyond the fixed array (many strips x splits)
    assert L.b200q_w4a16_gemm_noalloc(p, p, p, p, p, 32, 1 << 30, 4096, 128, 0, None) == _lib.ERR_SHAPE
    assert b"scratch" in L.b200q_last_error()
