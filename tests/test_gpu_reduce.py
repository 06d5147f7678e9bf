"""Reductions against the oracle (src/ops/reduce.rs).  max/min/argmax/argmin
are bit-exact; sums are tree-ordered and match normwise <= 1e-5 (and against
an f64 restatement)."""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (7, 33), (1000, 4096), (513, 1001), (4096, 4096),
                                       (2, 100000)])
@pytest.mark.parametrize("op", ["sum", "max", "min"])
def test_reduce_last_axis(jx, dev, oracle, rows, cols, op):
    rng = np.random.default_rng(rows * 31 + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    X, Y = dev.put(x), dev.full((rows,), np.nan)
    jx.reduce_axis(X.data_ptr(), Y.data_ptr(), rows, cols, 1, op, dev.stream)
    y = dev.get(Y)
    o = oracle.reduce_axis(x, 1, op, nthreads=8)
    if op == "sum":
        assert normwise_rel(y, o) <= 1e-5
        assert normwise_rel(y, oracle.sum_rows_f64(x)) <= 1e-5
    else:
        assert np.array_equal(y, o)


@pytest.mark.parametrize("shape,axis", [((2, 3), 0), ((4, 5, 6), 1), ((3, 4, 5), 0), ((64, 3, 130), 1)])
@pytest.mark.parametrize("op", ["sum", "max", "min", "prod"])
def test_reduce_other_axes(jx, dev, oracle, shape, axis, op):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal(shape) * 0.5 + (1.0 if op == "prod" else 0.0)).astype(np.float32)
    outer = int(np.prod(shape[:axis])); inner = int(np.prod(shape[axis + 1:]))
    X, Y = dev.put(x), dev.full((outer * inner,), np.nan)
    jx.reduce_axis(X.data_ptr(), Y.data_ptr(), outer, shape[axis], inner, op, dev.stream)
    y = dev.get(Y).reshape(shape[:axis] + shape[axis + 1:])
    o = oracle.reduce_axis(x, axis, op)
    # strided reductions fold sequentially per output: bit-exact for every op
    assert np.array_equal(y, o)


@pytest.mark.parametrize("n", [1, 5, 1000, 65537, 1 << 24, (1 << 24) + 3])
@pytest.mark.parametrize("op", ["sum", "max", "min"])
def test_reduce_all(jx, dev, oracle, n, op):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    X, Y = dev.put(x), dev.full((1,), np.nan)
    jx.reduce_all(X.data_ptr(), Y.data_ptr(), n, op, dev.stream)
    y = float(dev.get(Y)[0])
    if op == "sum":
        ref = oracle.sum_all_f64(x)
        assert abs(y - ref) <= 1e-5 * max(1.0, np.abs(x).sum() * 1e-3)
    else:
        assert y == oracle.reduce_all(x, op)


def test_sum_1_to_1000(jx, dev):
    """tests/gpu_tests.rs:208-222 (the reference's two-pass GPU sum)."""
    x = np.arange(1, 1001, dtype=np.float32)
    X, Y = dev.put(x), dev.full((1,), np.nan)
    jx.reduce_all(X.data_ptr(), Y.data_ptr(), 1000, "sum", dev.stream)
    assert abs(float(dev.get(Y)[0]) - 500500.0) < 1e-3


@pytest.mark.parametrize("is_max", [True, False])
def test_argreduce_ties_bit_exact(jx, dev, oracle, is_max):
    rows, cols = 4096, 777
    rng = np.random.default_rng(8)
    x = rng.integers(-3, 4, (rows, cols)).astype(np.float32)  # many ties
    x[5] = -np.inf
    x[6] = np.inf
    X = dev.put(x)
    I = dev.empty((rows,), dtype=dev.torch.int32)
    V = dev.full((rows,), np.nan)
    jx.argreduce_rows(X.data_ptr(), I.data_ptr(), V.data_ptr(), rows, cols, is_max, dev.stream)
    idx, val = dev.get(I), dev.get(V)
    o = oracle.arg_rows(x, is_max)
    assert np.array_equal(idx, o)
    assert np.array_equal(val, x[np.arange(rows), o])
    assert jx.device_status() == 0


def test_argmax_doc_and_nan_flag(jx, dev):
    X = dev.put(np.array([[3, 1, 4, 2]], np.float32))
    I = dev.empty((1,), dtype=dev.torch.int32)
    jx.argreduce_rows(X.data_ptr(), I.data_ptr(), None, 1, 4, True, dev.stream)
    assert dev.get(I).tolist() == [2]
    jx.argreduce_rows(X.data_ptr(), I.data_ptr(), None, 1, 4, False, dev.stream)
    assert dev.get(I).tolist() == [1]
    assert jx.device_status() == 0
    Xn = dev.put(np.array([[1, np.nan, 0]], np.float32))
    jx.argreduce_rows(Xn.data_ptr(), I.data_ptr(), None, 1, 3, True, dev.stream)
    assert jx.device_status() & jx.DEVERR_NAN


def test_argmax_full_config_rows(jx, dev, oracle):
    """[65536, 4096] last-axis argmax, bit-exact against the oracle."""
    rows, cols = 65536, 4096
    rng = np.random.default_rng(12)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    X = dev.put(x)
    I = dev.empty((rows,), dtype=dev.torch.int32)
    jx.argreduce_rows(X.data_ptr(), I.data_ptr(), None, rows, cols, True, dev.stream)
    assert np.array_equal(dev.get(I), oracle.arg_rows(x, True, nthreads=8))


def test_sum_and_max_vjp(jx, dev, oracle):
    rows, cols = 300, 129
    rng = np.random.default_rng(13)
    x = rng.integers(-2, 3, (rows, cols)).astype(np.float32)
    ct = rng.standard_normal(rows).astype(np.float32)
    X, CT = dev.put(x), dev.put(ct)
    DX = dev.full((rows, cols), np.nan)
    jx.sum_rows_vjp(CT.data_ptr(), DX.data_ptr(), rows, cols, dev.stream)
    assert np.array_equal(dev.get(DX), oracle.sum_rows_vjp(ct, cols))
    jx.max_rows_vjp(X.data_ptr(), CT.data_ptr(), DX.data_ptr(), rows, cols, dev.stream)
    assert np.array_equal(dev.get(DX), oracle.max_rows_vjp(x, ct))


@pytest.mark.parametrize("rows,cols", [(37, 4), (300, 128), (64, 1024), (64, 1028), (40, 2048), (33, 4096),
                                       (17, 8192), (9, 8196)])
def test_max_vjp_widths(jx, dev, oracle, rows, cols):
    """Every width class of the register-resident kernel and the fallback:
    ties (small integers), a row of -inf and a NaN, bit-identical."""
    rng = np.random.default_rng(rows + cols)
    x = rng.integers(-3, 4, (rows, cols)).astype(np.float32)
    x[0, :] = -np.inf
    x[1, 2] = np.nan
    ct = rng.standard_normal(rows).astype(np.float32)
    X, CT = dev.put(x), dev.put(ct)
    DX = dev.full((rows, cols), np.nan)
    jx.max_rows_vjp(X.data_ptr(), CT.data_ptr(), DX.data_ptr(), rows, cols, dev.stream)
    assert np.array_equal(dev.get(DX), oracle.max_rows_vjp(x, ct))
