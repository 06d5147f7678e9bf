"""GEMM parity through the C ABI against the oracle (Array::matmul CPU loop,
src/ops/linalg.rs:215-232).  Tolerance: normwise relative error <= 1e-5 for
the tcgen05 3xTF32 path; bit-identical for JX_PREC_EXACT."""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _inputs(oracle, M, N, K, seed=1):
    """Seeded U(-1,1) operands from the reference PRNG (src/random.rs:161-181)."""
    ka, kb = oracle.key_from_seed(seed).split()
    a = oracle.uniform_range(ka, M * K, -1.0, 1.0).reshape(M, K)
    b = oracle.uniform_range(kb, K * N, -1.0, 1.0).reshape(K, N)
    return a, b


def _gemm(jx, dev, a, b, precision, transA=False, transB=False):
    M = a.shape[1] if transA else a.shape[0]
    K = a.shape[0] if transA else a.shape[1]
    N = b.shape[0] if transB else b.shape[1]
    A, B = dev.put(a), dev.put(b)
    C = dev.full((M, N), np.nan)
    jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, transA, transB, precision=precision,
            stream=dev.stream)
    return dev.get(C)


@pytest.mark.parametrize("prec", [0, 1], ids=["3xtf32", "exact"])
def test_known_answer_2x2(jx, dev, prec):
    c = _gemm(jx, dev, np.array([[1, 2], [3, 4]], np.float32), np.array([[5, 6], [7, 8]], np.float32), prec)
    np.testing.assert_allclose(c, [[19, 22], [43, 50]], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("prec", [0, 1], ids=["3xtf32", "exact"])
def test_identity(jx, dev, prec):
    a = np.arange(1, 10, dtype=np.float32).reshape(3, 3)
    np.testing.assert_array_equal(_gemm(jx, dev, a, np.eye(3, dtype=np.float32), prec), a)
    np.testing.assert_array_equal(_gemm(jx, dev, np.eye(3, dtype=np.float32), a, prec), a)


SHAPES = [(1, 1, 1), (2, 3, 4), (17, 33, 65), (128, 256, 32), (129, 257, 33), (300, 520, 1000),
          (1024, 1024, 1024), (640, 384, 2048), (255, 1000, 784), (256, 256, 32768), (128, 512, 100003)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_3xtf32_vs_oracle(jx, dev, oracle, M, N, K):
    a, b = _inputs(oracle, M, N, K)
    c = _gemm(jx, dev, a, b, jx.PREC_3XTF32)
    ref = oracle.matmul(a, b, nthreads=8)
    ref64 = oracle.matmul_f64(a, b) if M * N * K <= 2 ** 28 else a.astype(np.float64) @ b.astype(np.float64)
    assert normwise_rel(c, ref) <= TOL
    assert normwise_rel(c, ref64) <= TOL
    assert np.isfinite(c).all()


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (17, 33, 65), (129, 257, 33), (128, 784, 256)])
def test_exact_is_bit_identical(jx, dev, oracle, M, N, K):
    a, b = _inputs(oracle, M, N, K, seed=3)
    c = _gemm(jx, dev, a, b, jx.PREC_EXACT)
    assert np.array_equal(c, oracle.matmul(a, b, nthreads=8))


@pytest.mark.parametrize("prec", [0, 1], ids=["3xtf32", "exact"])
@pytest.mark.parametrize("tA,tB", [(False, True), (True, False), (True, True)])
def test_transposes(jx, dev, oracle, prec, tA, tB):
    M, N, K = 130, 270, 97
    a, b = _inputs(oracle, M, N, K, seed=5)
    at = np.ascontiguousarray(a.T) if tA else a
    bt = np.ascontiguousarray(b.T) if tB else b
    c = _gemm(jx, dev, at, bt, prec, tA, tB)
    ref = oracle.matmul(a, b)
    if prec == 1:
        assert np.array_equal(c, ref)
    else:
        assert normwise_rel(c, ref) <= TOL


@pytest.mark.parametrize("prec", [0, 1], ids=["3xtf32", "exact"])
def test_batched_matches_einsum_loop(jx, dev, oracle, prec):
    """einsum("bij,bjk->bik") loop (src/ops/einsum.rs:505-519)."""
    bt, M, N, K = 5, 96, 300, 130
    ka, kb = oracle.key_from_seed(9).split()
    a = oracle.uniform_range(ka, bt * M * K, -1, 1).reshape(bt, M, K)
    b = oracle.uniform_range(kb, bt * K * N, -1, 1).reshape(bt, K, N)
    A, B = dev.put(a), dev.put(b)
    C = dev.full((bt, M, N), np.nan)
    jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, batch=bt, strideA=M * K, strideB=K * N,
            strideC=M * N, precision=prec, stream=dev.stream)
    c = dev.get(C)
    ref = oracle.bmm(a, b, nthreads=8)
    if prec == 1:
        assert np.array_equal(c, ref)
    else:
        for i in range(bt):
            assert normwise_rel(c[i], ref[i]) <= TOL


def test_leading_dimensions(jx, dev, oracle):
    """Sub-matrix views: lda/ldb/ldc larger than the logical width."""
    M, N, K = 70, 90, 50
    a, b = _inputs(oracle, M, N, K, seed=11)
    abig = np.zeros((M, K + 12), np.float32); abig[:, :K] = a
    bbig = np.zeros((K, N + 4), np.float32); bbig[:, :N] = b
    A, B = dev.put(abig), dev.put(bbig)
    C = dev.full((M, N + 8), -7.0)
    jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, lda=K + 12, ldb=N + 4, ldc=N + 8,
            stream=dev.stream)
    c = dev.get(C)
    assert normwise_rel(c[:, :N], oracle.matmul(a, b)) <= TOL
    assert np.all(c[:, N:] == -7.0)  # untouched padding


FUSED_SHAPES = [
    # (batch, M, N, K, lda_pad, ldb_pad) through JX_PREC_3XTF32_FUSED: the
    # split inside the kernel (raw f32 tiles by TMA, B MN-major); ragged M, N
    # and K exercise TMA's zero fill
    (1, 1, 4, 4, 0, 0), (1, 5, 36, 8, 0, 0), (1, 129, 260, 36, 0, 0), (1, 200, 516, 1028, 0, 0),
    (1, 300, 4, 100, 0, 0), (3, 96, 300, 132, 0, 0), (2, 130, 264, 68, 4, 8), (1, 1024, 1024, 1024, 0, 0),
]


@pytest.mark.parametrize("bt,M,N,K,pa,pb", FUSED_SHAPES)
def test_fused_split_path(jx, dev, oracle, bt, M, N, K, pa, pb):
    ka, kb = oracle.key_from_seed(13 + M).split()
    a = oracle.uniform_range(ka, bt * M * K, -1, 1).reshape(bt, M, K)
    b = oracle.uniform_range(kb, bt * K * N, -1, 1).reshape(bt, K, N)
    abig = np.zeros((bt, M, K + pa), np.float32); abig[:, :, :K] = a
    bbig = np.zeros((bt, K, N + pb), np.float32); bbig[:, :, :N] = b
    A, B = dev.put(abig), dev.put(bbig)
    C = dev.full((bt, M, N), np.nan)
    jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, lda=K + pa, ldb=N + pb, batch=bt,
            strideA=M * (K + pa), strideB=K * (N + pb), strideC=M * N, precision=jx.PREC_3XTF32_FUSED,
            stream=dev.stream)
    c = dev.get(C)
    ref = oracle.bmm(a, b, nthreads=8)
    for i in range(bt):
        assert normwise_rel(c[i], ref[i]) <= TOL
        ref64 = a[i].astype(np.float64) @ b[i].astype(np.float64)
        assert normwise_rel(c[i], ref64) <= TOL


def test_fused_precision_rejects_transposed_operands(jx, dev):
    A, B, C = dev.full((8, 8), 1.0), dev.full((8, 8), 1.0), dev.full((8, 8), 0.0)
    with pytest.raises(jx.JaxRsError) as e:
        jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), 8, 8, 8, transA=True, precision=jx.PREC_3XTF32_FUSED,
                stream=dev.stream)
    assert "JX_PREC_3XTF32_FUSED" in e.value.message


def test_8192_cubed_sampled_rows(jx, dev, oracle):
    """Full-size headline shape: every output is computed on the device, and
    16 sampled rows are checked against the oracle's own loop."""
    M = N = K = 8192
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    c = _gemm(jx, dev, a, b, jx.PREC_3XTF32)
    rows = np.sort(rng.choice(M, 16, replace=False))
    for r in rows:
        ref = oracle.matmul_rows(a, b, int(r), int(r) + 1, nthreads=8)
        assert normwise_rel(c[r:r + 1], ref) <= TOL
    # checksum of checksums: sum over rows of C equals (1^T A) B
    colsum = a.astype(np.float64).sum(0) @ b.astype(np.float64)
    assert normwise_rel(c.astype(np.float64).sum(0), colsum) <= 1e-5


def test_many_small_products_default_precision(jx, dev, oracle):
    """160 products of 256^3 under JX_PREC_3XTF32: one 256 x 256 tile each,
    160 in all, enough for every SM pair, so the dispatcher takes the SM-pair
    kernel on its own (batch index as a TMA coordinate)."""
    bt, n = 160, 256
    rng = np.random.default_rng(17)
    a = rng.uniform(-1, 1, (bt, n, n)).astype(np.float32)
    b = rng.uniform(-1, 1, (bt, n, n)).astype(np.float32)
    A, B = dev.put(a), dev.put(b)
    C = dev.full((bt, n, n), np.nan)
    jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), n, n, n, batch=bt, strideA=n * n, strideB=n * n,
            strideC=n * n, stream=dev.stream)
    c = dev.get(C)
    for i in (0, 77, bt - 1):
        assert normwise_rel(c[i], oracle.matmul(a[i], b[i], nthreads=8)) <= TOL
    assert normwise_rel(c.astype(np.float64).sum(axis=1), np.einsum("bij,bjk->bk", a.astype(np.float64),
                                                                    b.astype(np.float64))) <= TOL


@pytest.mark.parametrize("M,N,K", [(300, 520, 1000), (2304, 2304, 512)], ids=["split_path", "pair_kernel"])
def test_non_finite_operands_mark_the_same_outputs(jx, dev, oracle, M, N, K):
    """An infinite or NaN operand element: the 3xTF32 product is non-finite
    exactly where the reference's loop (src/ops/linalg.rs:220-228) is, and
    every other output keeps the normwise tolerance.  (Where the reference
    gives +-inf the 3xTF32 value can be NaN: the infinite hi part meets the
    other operand's lo part, which may be zero or of the other sign.)"""
    rng = np.random.default_rng(M)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    a[7, 3] = np.inf
    a[M - 2, K - 1] = np.nan
    b[5, N // 2] = -np.inf
    c = _gemm(jx, dev, a, b, jx.PREC_3XTF32)
    with np.errstate(invalid="ignore", over="ignore"):
        ref = a.astype(np.float64) @ b.astype(np.float64)
    bad = ~np.isfinite(ref)
    assert np.array_equal(~np.isfinite(c), bad)
    assert normwise_rel(c[~bad], ref[~bad]) <= TOL
