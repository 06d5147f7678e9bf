"""jx_gemm_f32_noalloc: the GEMM entry point that allocates nothing.

It exists for callers that cannot let a library allocate device memory: a
process whose own arena or caching allocator already owns the GPU's memory, a
latency-critical loop that cannot afford an allocator call, or a plugin host
that forbids hidden allocations.  Its workspace is a fixed 64 MiB device array
inside the library.  This test calls it through the C ABI and checks it
against the allocating entry point jx_gemm_f32 (normwise <= 1e-5, the GEMM
tests' tolerance) on two calls in a row, so the second call runs on the
array the first one left behind.  It also checks that a problem too large for
the array is refused.

The file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


def _noalloc(jx, A, B, Cp, M, N, K, batch=1, sA=0, sB=0, sC=0, stream=None):
    jx.call("jx_gemm_f32_noalloc", A, B, Cp, M, N, K, 0, 0, K, N, N, batch, sA, sB, sC, stream)


def test_noalloc_matches_allocating_gemm_twice(jx, dev):
    rng = np.random.default_rng(21)
    # two calls in a row with different shapes: the second one reuses (and must
    # fully overwrite) the workspace contents the first one left
    for (M, N, K, batch) in ((300, 520, 1000, 1), (96, 200, 130, 3)):
        a = rng.uniform(-1, 1, (batch, M, K)).astype(np.float32)
        b = rng.uniform(-1, 1, (batch, K, N)).astype(np.float32)
        A, B = dev.put(a), dev.put(b)
        C_ref = dev.full((batch, M, N), np.nan)
        C_new = dev.full((batch, M, N), np.nan)
        jx.gemm(A.data_ptr(), B.data_ptr(), C_ref.data_ptr(), M, N, K, batch=batch, strideA=M * K,
                strideB=K * N, strideC=M * N, stream=dev.stream)
        _noalloc(jx, A.data_ptr(), B.data_ptr(), C_new.data_ptr(), M, N, K, batch, M * K, K * N, M * N,
                 dev.stream)
        ref, got = dev.get(C_ref), dev.get(C_new)
        assert np.isfinite(got).all()
        for i in range(batch):
            assert normwise_rel(got[i], ref[i]) <= 1e-5
            exact = a[i].astype(np.float64) @ b[i].astype(np.float64)
            assert normwise_rel(got[i], exact) <= 1e-5


def test_noalloc_rejects_problems_beyond_the_fixed_workspace(jx, dev):
    M = N = K = 4096  # needs 2*(M+N)*K floats = 256 MiB > 64 MiB
    with pytest.raises(jx.JaxRsError) as e:
        _noalloc(jx, 16, 16, 16, M, N, K)
    assert e.value.status == jx.JX_EINVAL
    assert "maximum" in e.value.message
