"""The SM-pair 3xTF32 GEMM (JX_PREC_3XTF32_PAIR: tcgen05 cta_group::2, split
in shared memory) against the oracle's Array::matmul loop
(src/ops/linalg.rs:215-232) and f64, every transposition, ragged edges,
padded leading dimensions and batches.  Tolerance: normwise relative error
<= 1e-5, as for every 3xTF32 path.  Shapes have at least one 256 x 256 tile
per SM pair (74 pairs on a B200)."""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _run(jx, dev, a, b, M, N, K, tA=False, tB=False, lda=None, ldb=None, batch=1, sA=0, sB=0):
    A, B = dev.put(a), dev.put(b)
    C = dev.full((batch, M, N), np.nan)
    jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, tA, tB, lda=lda, ldb=ldb, batch=batch, strideA=sA,
            strideB=sB, strideC=M * N, precision=jx.PREC_3XTF32_PAIR, stream=dev.stream)
    return dev.get(C)


def _check_rows(oracle, a, b, c, rows):
    for r in rows:
        ref = oracle.matmul_rows(a, b, int(r), int(r) + 1, nthreads=8)
        assert normwise_rel(c[r:r + 1], ref) <= TOL


@pytest.mark.parametrize("tA,tB", [(False, False), (True, False), (False, True), (True, True)],
                         ids=["nn", "tn", "nt", "tt"])
@pytest.mark.parametrize("M,N,K", [(2304, 2304, 1000), (2200, 2332, 76), (2048, 2560, 4096)])
def test_pair_transposes_vs_oracle(jx, dev, oracle, tA, tB, M, N, K):
    rng = np.random.default_rng(M + 3 * N + K + 2 * tA + tB)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    a_in = np.ascontiguousarray(a.T) if tA else a
    b_in = np.ascontiguousarray(b.T) if tB else b
    c = _run(jx, dev, a_in, b_in, M, N, K, tA, tB)[0]
    assert np.isfinite(c).all()
    assert normwise_rel(c, a.astype(np.float64) @ b.astype(np.float64)) <= TOL
    _check_rows(oracle, a, b, c, [0, 1, 127, 128, 255, 256, M // 2, M - 1])


def test_pair_batched_with_padded_rows(jx, dev, oracle):
    """[8, 800, 520] x [8, 520, 808] with lda = 524 and ldb = 812: the batch
    index is a TMA coordinate, padding columns are never read."""
    bt, M, K, N, pa, pb = 8, 800, 520, 808, 4, 4
    rng = np.random.default_rng(31)
    a = rng.uniform(-1, 1, (bt, M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (bt, K, N)).astype(np.float32)
    abig = np.full((bt, M, K + pa), 7.0, np.float32)
    abig[:, :, :K] = a
    bbig = np.full((bt, K, N + pb), -3.0, np.float32)
    bbig[:, :, :N] = b
    c = _run(jx, dev, abig, bbig, M, N, K, lda=K + pa, ldb=N + pb, batch=bt, sA=M * (K + pa), sB=K * (N + pb))
    ref = oracle.bmm(a, b, nthreads=8)
    for i in range(bt):
        assert normwise_rel(c[i], ref[i]) <= TOL
        assert normwise_rel(c[i], a[i].astype(np.float64) @ b[i].astype(np.float64)) <= TOL


def test_pair_8192_cubed_sampled_rows(jx, dev, oracle):
    """The headline shape on the pair kernel: 16 sampled rows against the
    oracle, all rows by the column-sum identity 1^T(AB) = (1^T A)B."""
    M = N = K = 8192
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    c = _run(jx, dev, a, b, M, N, K)[0]
    _check_rows(oracle, a, b, c, np.sort(rng.choice(M, 16, replace=False)))
    colsum = a.astype(np.float64).sum(0) @ b.astype(np.float64)
    assert normwise_rel(c.astype(np.float64).sum(0), colsum) <= TOL


def test_pair_twice_in_a_row_same_result(jx, dev):
    """Deterministic: the same call twice gives the same bits (fixed
    accumulation order per output)."""
    M = N = 2304
    K = 640
    rng = np.random.default_rng(4)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    c1 = _run(jx, dev, a, b, M, N, K)
    c2 = _run(jx, dev, a, b, M, N, K)
    assert np.array_equal(c1, c2)


def test_pair_precision_rejects_too_few_tiles(jx, dev):
    A, B, C = dev.full((256, 256), 1.0), dev.full((256, 256), 1.0), dev.full((256, 256), 0.0)
    with pytest.raises(jx.JaxRsError) as e:
        jx.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), 256, 256, 256, precision=jx.PREC_3XTF32_PAIR,
                stream=dev.stream)
    assert e.value.status == jx.JX_EINVAL and "SM pair" in e.value.message


def test_pair_padded_output_rows_and_batch_stride(jx, dev, oracle):
    """C with ldc > N and a batch stride beyond M*ldc: the pair kernel writes
    only the product's columns, the padding keeps its sentinel."""
    bt, M, N, K = 4, 1024, 1536, 200  # 4 x 4 x 6 = 96 pair tiles
    ldc, sC = N + 12, (1024 + 3) * (N + 12)
    rng = np.random.default_rng(41)
    a = rng.uniform(-1, 1, (bt, M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (bt, K, N)).astype(np.float32)
    A, B = dev.put(a), dev.put(b)
    Cbuf = dev.full((bt * sC,), -5.0)
    jx.gemm(A.data_ptr(), B.data_ptr(), Cbuf.data_ptr(), M, N, K, ldc=ldc, batch=bt, strideA=M * K,
            strideB=K * N, strideC=sC, precision=jx.PREC_3XTF32_PAIR, stream=dev.stream)
    c = dev.get(Cbuf)
    for i in range(bt):
        blk = c[i * sC:i * sC + M * ldc].reshape(M, ldc)
        assert normwise_rel(blk[:, :N], a[i].astype(np.float64) @ b[i].astype(np.float64)) <= TOL
        assert (blk[:, N:] == -5.0).all()
        assert (c[i * sC + M * ldc:(i + 1) * sC] == -5.0).all()
