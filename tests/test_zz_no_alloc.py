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
    cases = [(16, 14336, 4096, 128, "fp16"), (5, 4096, 1024, 128, "bf16"),
             # 17..32 rows: the two-row-block variant, which only this entry point uses
             (17, 4096, 1024, 64, "fp16"), (32, 2048, 768, 32, "bf16"), (32, 14336, 4096, 128, "fp16")]
    for seed, (M, K, N, group, dtype) in enumerate(cases):
        x, q, s, z = w4a16_inputs(M, K, N, group, dtype, seed=100 + seed, device="cuda")
        ref = ops.w4a16_gemm(x, q, s, z, group)
        y1 = _noalloc(L, x, q, s, z, group)
        y2 = _noalloc(L, x, q, s, z, group)
        torch.cuda.synchronize()
        assert L.b200q_w4a16_noalloc_status(torch.cuda.current_stream().cuda_stream) == 0
        # bf16: the workspace entry point's tensor-core path (M >= 17) rounds
        # each weight to bf16 like the reference module, the decode path keeps
        # it in fp32, so the two are compared at the bf16 bar of the other tests
        tol = TOL if dtype == "fp16" else dict(rtol=5e-2, atol=5e-2)
        torch.testing.assert_close(y1.float(), ref.float(), **tol)
        torch.testing.assert_close(y2.float(), ref.float(), **tol)
        assert torch.equal(y1, y2)


def test_noalloc_rejects_oversize():
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import _lib
    L = _lib.lib()
    dev = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = dev.data_ptr()
    assert L.b200q_w4a16_gemm_noalloc(p, p, p, p, p, 64, 4096, 4096, 128, 0, None) == _lib.ERR_SHAPE
    assert b"M must be" in L.b200q_last_error()
    # N beyond the supported range
    assert L.b200q_w4a16_gemm_noalloc(p, p, p, p, p, 32, (1 << 30) + 32, 4096, 128, 0, None) == _lib.ERR_SHAPE
    assert b"too large" in L.b200q_last_error()
    # K beyond the 32-bit range the kernels index with
    assert L.b200q_w4a16_gemm_noalloc(p, p, p, p, p, 16, 4096, 1 << 31, 128, 0, None) == _lib.ERR_SHAPE
    assert b"too large" in L.b200q_last_error()
