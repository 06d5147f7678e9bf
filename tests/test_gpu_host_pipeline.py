"""Host-buffer entry points with overlapped transfers (jx_gemm_f32_host,
jx_tape_run_host, jx_fft*_c2c_f32_host): the same results as the device-buffer
calls, with pinned, registered and pageable host memory, for ragged block
splits."""
import ctypes as C

import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


def _ptr(a):
    return a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr()


@pytest.mark.parametrize("M,N,K,block", [(1000, 520, 300, 0), (1000, 520, 300, 128), (257, 64, 33, 100),
                                         (4096, 1024, 2048, 0)])
@pytest.mark.parametrize("pinned", [True, False])
def test_gemm_host_matches_oracle(jx, dev, oracle, M, N, K, block, pinned):
    import torch
    rng = np.random.default_rng(M + N + K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    if pinned:
        A, B = torch.from_numpy(a).pin_memory(), torch.from_numpy(b).pin_memory()
        Cm = torch.full((M, N), float("nan")).pin_memory()
    else:
        A, B, Cm = a, b, np.full((M, N), np.nan, np.float32)
    jx.call("jx_gemm_f32_host", _ptr(A), _ptr(B), _ptr(Cm), M, N, K, K, N, N, block, dev.stream)
    dev.sync()
    c = Cm.numpy() if pinned else Cm
    rows = np.unique(np.linspace(0, M - 1, 12).astype(int))
    ref = oracle.matmul(a[rows], b, nthreads=8)
    assert normwise_rel(c[rows], ref) <= 1e-5
    assert np.isfinite(c).all()


@pytest.mark.parametrize("n,block", [(1, 0), (1000, 256), (1 << 20, 100000), (3_000_001, 0)])
def test_tape_run_host_matches_device_run(jx, dev, oracle, n, block):
    from test_gpu_elementwise import chain_tape, _close
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    y = np.full(n, np.nan, np.float32)
    tape = chain_tape(jx, 1.1, 0.9)
    ia = (C.c_void_p * 1)(x.ctypes.data)
    oa = (C.c_void_p * 1)(y.ctypes.data)
    jx.call("jx_tape_run_host", tape.handle, ia, oa, n, block, dev.stream)
    dev.sync()
    assert _close(y, oracle.chain_fwd(x, np.float32(1.1), np.float32(0.9)))


@pytest.mark.parametrize("n,batch,block", [(4096, 37, 0), (1024, 100, 7), (8, 1000, 64)])
def test_fft_host_matches_oracle(jx, dev, oracle, n, batch, block):
    x = np.random.default_rng(n + batch).standard_normal((batch, n, 2)).astype(np.float32)
    y = np.full_like(x, np.nan)
    jx.call("jx_fft_c2c_f32_host", x.ctypes.data, y.ctypes.data, n, batch, 0, block, dev.stream)
    dev.sync()
    ref = oracle.fft_c2c(x)
    for b in (0, batch // 2, batch - 1):
        assert normwise_rel(y[b], ref[b]) <= 1e-5


def test_fft2_host_matches_device_call(jx, dev):
    import torch
    h, w, batch = 64, 128, 21
    x = np.random.default_rng(5).standard_normal((batch, h, w, 2)).astype(np.float32)
    y = np.full_like(x, np.nan)
    jx.call("jx_fft2_c2c_f32_host", x.ctypes.data, y.ctypes.data, h, w, batch, 1, 4, dev.stream)
    dev.sync()
    X = dev.put(x)
    Y = dev.full(x.shape, np.nan)
    jx.call("jx_fft2_c2c_f32", X.data_ptr(), Y.data_ptr(), h, w, batch, 1, dev.stream)
    assert np.array_equal(y, dev.get(Y))  # same kernels, same bits


def test_registered_host_memory(jx, dev, oracle):
    """A caller's own arrays page-locked with jx_host_register give the same
    results, and unregister cleanly afterwards."""
    from test_gpu_elementwise import chain_tape, _close
    n = 5_000_003
    x = np.random.default_rng(9).standard_normal(n).astype(np.float32)
    y = np.full(n, np.nan, np.float32)
    jx.call("jx_host_register", x.ctypes.data, x.nbytes)
    jx.call("jx_host_register", y.ctypes.data, y.nbytes)
    try:
        tape = chain_tape(jx, 1.1, 0.9)
        ia = (C.c_void_p * 1)(x.ctypes.data)
        oa = (C.c_void_p * 1)(y.ctypes.data)
        jx.call("jx_tape_run_host", tape.handle, ia, oa, n, 1 << 20, dev.stream)
        dev.sync()
    finally:
        jx.call("jx_host_unregister", x.ctypes.data)
        jx.call("jx_host_unregister", y.ctypes.data)
    assert _close(y, oracle.chain_fwd(x, np.float32(1.1), np.float32(0.9)))


@pytest.mark.parametrize("M,N,K,batch,block", [(64, 96, 40, 5, 2), (256, 256, 300, 3, 0), (33, 17, 9, 7, 3)])
def test_batched_gemm_host_matches_oracle(jx, dev, oracle, M, N, K, batch, block):
    rng = np.random.default_rng(M + batch)
    a = rng.uniform(-1, 1, (batch, M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (batch, K, N)).astype(np.float32)
    c = np.full((batch, M, N), np.nan, np.float32)
    jx.call("jx_gemm_batched_f32_host", a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K, batch, block,
            dev.stream)
    dev.sync()
    for i in range(batch):
        assert normwise_rel(c[i], oracle.matmul(a[i], b[i])) <= 1e-5


@pytest.mark.parametrize("is_max", [True, False])
def test_pool_host_matches_device_call(jx, dev, is_max):
    x = np.random.default_rng(4).standard_normal((7, 3, 21, 19)).astype(np.float32)
    geo = (7, 3, 21, 19, 3, 3, 2, 2, 1, 1)
    op = jx.POOL_MAX if is_max else jx.POOL_AVG
    y = np.full((7, 3, 11, 10), np.nan, np.float32)
    jx.call("jx_pool2d_f32_host", x.ctypes.data, y.ctypes.data, *geo, op, 2, dev.stream)
    dev.sync()
    X = dev.put(x)
    Y = dev.full(y.shape, np.nan)
    jx.call("jx_pool2d_f32", X.data_ptr(), Y.data_ptr(), *geo, op, dev.stream)
    assert np.array_equal(y, dev.get(Y))  # same kernel, same bits
