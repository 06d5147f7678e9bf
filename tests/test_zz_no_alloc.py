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


def _noalloc(jx, A, B, Cp, M, N, K, batch=1, sA=0, sB=0, sC=0, stream=None, transA=0, transB=0):
    lda = M if transA else K
    ldb = K if transB else N
    jx.call("jx_gemm_f32_noalloc", A, B, Cp, M, N, K, transA, transB, lda, ldb, N, batch, sA, sB, sC, stream)


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


@pytest.mark.parametrize("transA,transB", [(1, 0), (0, 1), (1, 1)])
def test_noalloc_transposed_operands(jx, dev, transA, transB):
    """The transposing split pass writes into the fixed array too: K not a
    multiple of 32 (zero padding up to the k-block) and a batch offset."""
    rng = np.random.default_rng(22 + 2 * transA + transB)
    M, N, K, batch = 136, 264, 77, 2
    a = rng.uniform(-1, 1, (batch, K, M) if transA else (batch, M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (batch, N, K) if transB else (batch, K, N)).astype(np.float32)
    A, B = dev.put(a), dev.put(b)
    for _ in range(2):  # twice in a row on the same array
        C_ref = dev.full((batch, M, N), np.nan)
        C_new = dev.full((batch, M, N), np.nan)
        jx.gemm(A.data_ptr(), B.data_ptr(), C_ref.data_ptr(), M, N, K, transA=bool(transA), transB=bool(transB),
                batch=batch, strideA=M * K, strideB=K * N, strideC=M * N, stream=dev.stream)
        _noalloc(jx, A.data_ptr(), B.data_ptr(), C_new.data_ptr(), M, N, K, batch, M * K, K * N, M * N,
                 dev.stream, transA, transB)
        ref, got = dev.get(C_ref), dev.get(C_new)
        for i in range(batch):
            ai = a[i].T if transA else a[i]
            bi = b[i].T if transB else b[i]
            assert normwise_rel(got[i], ref[i]) <= 1e-5
            assert normwise_rel(got[i], ai.astype(np.float64) @ bi.astype(np.float64)) <= 1e-5


def test_noalloc_empty_contraction_zero_fills(jx, dev):
    """K == 0 gives C = 0, as jx_gemm_f32 does."""
    M, N = 5, 7
    C_new = dev.full((M, N), np.nan)
    _noalloc(jx, 16, 16, C_new.data_ptr(), M, N, 0, stream=dev.stream)
    assert (dev.get(C_new) == 0).all()


def test_noalloc_error_word_reaches_device_status(jx, dev):
    """A timed-out wait inside this entry point's launches is flagged in its
    own fixed device word; jx_device_status must report and clear it.  The
    flag is planted through the test hook (no wait is made to run out)."""
    jx.device_status()  # clear whatever an earlier test left
    jx.call("jx_selftest_noalloc_flag", jx.DEVERR_TIMEOUT)
    assert jx.device_status() & jx.DEVERR_TIMEOUT
    assert jx.device_status() == 0
