"""nn/optim kernels and the native MLP trainer against the oracle.

Tolerances: Adam, bias add, relu, relu backward and column sums are
bit-identical (the reference's op order, no FMA); softmax / cross-entropy use
the device exp/log (a few ulp from glibc): |d - o| <= 1e-5*|o| + 1e-7.  MLP
training (784-256-128-10, batch 128, Adam, 100 steps): per-step loss within
1e-4 and final weights within 1e-5 of the oracle's restatement.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _close(d, o, rtol=1e-5, atol=1e-7):
    d = np.asarray(d, np.float64)
    o = np.asarray(o, np.float64)
    return np.all(np.abs(d - o) <= rtol * np.abs(o) + atol)


@pytest.mark.parametrize("rows,cols", [(1, 3), (128, 10), (77, 1000), (4, 4097)])
def test_softmax_rows(jx, dev, oracle, rows, cols):
    x = np.random.default_rng(rows).standard_normal((rows, cols)).astype(np.float32) * 3
    X, Y = dev.put(x), dev.full((rows, cols), np.nan)
    jx.call("jx_softmax_rows_f32", X.data_ptr(), Y.data_ptr(), rows, cols, dev.stream)
    y = dev.get(Y)
    assert _close(y, oracle.softmax_rows(x))
    np.testing.assert_allclose(y.sum(1), 1.0, atol=1e-5)


@pytest.mark.parametrize("rows,cols", [(128, 10), (33, 1000), (5, 7)])
def test_softmax_xent_fwd_bwd(jx, dev, oracle, rows, cols):
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32) * 2
    y = rng.integers(0, cols, rows).astype(np.float32)
    y[0] = cols + 3  # out of range: one_hot marks nothing
    X, Yl = dev.put(x), dev.put(y)
    P, D, Lo = dev.full((rows, cols), np.nan), dev.full((rows, cols), np.nan), dev.full((1,), np.nan)
    jx.call("jx_softmax_xent_f32", X.data_ptr(), Yl.data_ptr(), P.data_ptr(), D.data_ptr(), Lo.data_ptr(), rows,
            cols, rows * cols, dev.stream)
    p_ref = oracle.softmax_rows(x)
    t = oracle.one_hot(y, cols)
    assert _close(dev.get(P), p_ref)
    assert abs(float(dev.get(Lo)[0]) - oracle.cross_entropy(p_ref, t)) <= 1e-5 * abs(oracle.cross_entropy(p_ref, t))
    assert _close(dev.get(D), oracle.softmax_xent_bwd(p_ref, t), rtol=1e-5, atol=1e-10)


@pytest.mark.parametrize("act", [0, 1, 2])
def test_bias_act_and_backward(jx, dev, oracle, act):
    rows, cols = 64, 256
    rng = np.random.default_rng(act)
    z = rng.standard_normal((rows, cols)).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    Z, Bb, Pre = dev.put(z), dev.put(b), dev.full((rows, cols), np.nan)
    jx.call("jx_bias_act_f32", Z.data_ptr(), Bb.data_ptr(), Pre.data_ptr(), rows, cols, act, dev.stream)
    pre_ref = oracle.binary("add", z, b)
    assert np.array_equal(dev.get(Pre), pre_ref)
    y = dev.get(Z)
    if act == 0:
        assert np.array_equal(y, pre_ref)
    elif act == 1:
        assert np.array_equal(y, oracle.unary("relu", pre_ref))
    else:
        assert _close(y, oracle.unary("gelu", pre_ref), atol=1e-6)
    dy = rng.standard_normal((rows, cols)).astype(np.float32)
    DY, DZ, DB = dev.put(dy), dev.full((rows, cols), np.nan), dev.full((cols,), np.nan)
    jx.call("jx_act_bwd_f32", DY.data_ptr(), Pre.data_ptr(), DZ.data_ptr(), DB.data_ptr(), rows, cols, act,
            dev.stream)
    dz = dev.get(DZ)
    if act == 1:
        assert np.array_equal(dz, (dy * (pre_ref > 0).astype(np.float32)).astype(np.float32))
    if act != 2:
        assert np.array_equal(dev.get(DB), oracle.col_sum(dz))


def test_col_sum_many_rows(jx, dev, oracle):
    rows, cols = 5000, 300
    dy = np.random.default_rng(5).standard_normal((rows, cols)).astype(np.float32)
    DY, DB = dev.put(dy), dev.full((cols,), np.nan)
    jx.call("jx_col_sum_f32", DY.data_ptr(), DB.data_ptr(), rows, cols, dev.stream)
    ref = dy.astype(np.float64).sum(0)
    assert np.abs(dev.get(DB) - ref).max() <= 1e-5 * np.abs(dy).sum(0).max()


def test_adam_bit_exact_over_steps(jx, dev, oracle):
    """optim::adam_update: several steps, several tensors, bit-identical."""
    import ctypes as C
    rng = np.random.default_rng(9)
    sizes = [1, 37, 4096]
    ps = [rng.standard_normal(n).astype(np.float32) for n in sizes]
    P = [dev.put(p) for p in ps]
    M = [dev.full((n,), 0.0) for n in sizes]
    V = [dev.full((n,), 0.0) for n in sizes]
    om = [np.zeros(n, np.float32) for n in sizes]
    ov = [np.zeros(n, np.float32) for n in sizes]
    op = [p.copy() for p in ps]
    vp = C.c_void_p
    for step in range(1, 6):
        gs = [rng.standard_normal(n).astype(np.float32) for n in sizes]
        G = [dev.put(g) for g in gs]
        arr = lambda ts: (vp * len(ts))(*[t.data_ptr() for t in ts])
        jx.call("jx_adam_step_f32", arr(P), arr(G), arr(M), arr(V), (C.c_int64 * 3)(*sizes), 3, 1e-3, 0.9, 0.999,
                1e-8, step, dev.stream)
        for i in range(3):
            op[i], om[i], ov[i] = oracle.adam_update(op[i], gs[i], om[i], ov[i], 1e-3, 0.9, 0.999, 1e-8, step,
                                                     step == 1)
        dev.sync()
    for i in range(3):
        assert np.array_equal(dev.get(P[i]), op[i])
        assert np.array_equal(dev.get(M[i]), om[i])
        assert np.array_equal(dev.get(V[i]), ov[i])


def _train_device(jx, dev, Ws, bs, data, widths, precision):
    net = jx.MLP(widths, ["relu"] * (len(widths) - 2), data[0][0].shape[0], precision)
    net.set_params(net.pack(Ws, bs))
    net.set_adam(1e-3, 0.9, 0.999, 1e-8)
    losses = []
    Lo = dev.full((1,), np.nan)
    for x, y in data:
        X, Y = dev.put(x), dev.put(y)
        net.step(X.data_ptr(), Y.data_ptr(), Lo.data_ptr(), dev.stream)
        losses.append(float(dev.get(Lo)[0]))
    return losses, net.unpack(net.get_params())


@pytest.mark.parametrize("steps", [3])
def test_small_mlp_few_steps(jx, dev, oracle, steps):
    import oracle.mlp as OM
    widths = [784, 256, 128, 10]
    Ws, bs = OM.xavier_params(widths, seed=1)
    data = OM.batches(steps, 128, 784, 10, seed=0)
    ol, oW, ob = OM.train(Ws, bs, data)
    dl, (dW, db) = _train_device(jx, dev, Ws, bs, data, widths, jx.PREC_EXACT)
    np.testing.assert_allclose(dl, ol, atol=1e-6, rtol=1e-6)
    for a, b in zip(dW + db, oW + ob):
        assert np.abs(a - b).max() <= 1e-5


def test_small_mlp_100_steps_matches_oracle(jx, dev, oracle):
    """The configured run: 784-256-128-10 ReLU, batch 128, Adam 1e-3, 100 steps."""
    import oracle.mlp as OM
    widths = [784, 256, 128, 10]
    Ws, bs = OM.xavier_params(widths, seed=1)
    data = OM.batches(100, 128, 784, 10, seed=0)
    ol, oW, ob = OM.train(Ws, bs, data)
    dl, (dW, db) = _train_device(jx, dev, Ws, bs, data, widths, jx.PREC_EXACT)
    assert max(abs(a - b) for a, b in zip(dl, ol)) <= 1e-4
    assert ol[-1] < ol[0]  # it learns
    worst = max(float(np.abs(a - b).max()) for a, b in zip(dW + db, oW + ob))
    assert worst <= 1e-5, worst


def test_mlp_3xtf32_tracks_oracle(jx, dev, oracle):
    """Tensor-core GEMMs (3xTF32) in the trainer: losses within 1e-4 over 20 steps."""
    import oracle.mlp as OM
    widths = [784, 256, 128, 10]
    Ws, bs = OM.xavier_params(widths, seed=1)
    data = OM.batches(20, 128, 784, 10, seed=0)
    ol, _, _ = OM.train(Ws, bs, data)
    dl, _ = _train_device(jx, dev, Ws, bs, data, widths, jx.PREC_3XTF32)
    assert max(abs(a - b) for a, b in zip(dl, ol)) <= 1e-4


def _train_mode(jx, dev, Ws, bs, data, widths, acts, fused):
    net = jx.MLP(widths, acts, data[0][0].shape[0], jx.PREC_EXACT)
    jx.call("jx_mlp_set_fused", net.handle, 1 if fused else 0)
    net.set_params(net.pack(Ws, bs))
    net.set_adam(1e-3, 0.9, 0.999, 1e-8)
    losses = []
    Lo = dev.full((1,), np.nan)
    for x, y in data:
        X, Y = dev.put(x), dev.put(y)
        net.step(X.data_ptr(), Y.data_ptr(), Lo.data_ptr(), dev.stream)
        losses.append(dev.get(Lo)[0])
    return np.array(losses), net.get_params()


@pytest.mark.parametrize("widths,acts,batch", [([784, 256, 128, 10], ["relu", "relu"], 128),
                                               ([33, 70, 5], ["gelu"], 300),
                                               ([20, 17, 9, 13, 3], ["relu", "none", "gelu"], 37),
                                               ([64, 10], [], 16)])
def test_fused_step_bit_identical_to_graph(jx, dev, oracle, widths, acts, batch):
    """One cooperative kernel per step gives the captured graph's bits:
    losses and every parameter after 12 Adam steps."""
    import oracle.mlp as OM
    Ws, bs = OM.xavier_params(widths, seed=3)
    data = OM.batches(12, batch, widths[0], widths[-1], seed=4)
    lf, pf = _train_mode(jx, dev, Ws, bs, data, widths, acts, True)
    lg, pg = _train_mode(jx, dev, Ws, bs, data, widths, acts, False)
    assert np.array_equal(lf, lg)
    assert np.array_equal(pf, pg)
    assert jx.device_status() == 0


def test_bounded_barrier_wait_reports_timeout(jx, dev, oracle):
    """A grid barrier that can never complete gives up after its limit,
    reports JX_DEVERR_TIMEOUT, and the device keeps working."""
    import ctypes as C
    jx.device_status()  # clear the error word
    flag = C.c_int(0)
    jx.call("jx_selftest_barrier_timeout", 200, C.byref(flag))
    assert flag.value == 1
    assert jx.device_status() & 0x2
    assert jx.device_status() == 0  # read and cleared
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    A, B = dev.put(a), dev.put(np.eye(3, dtype=np.float32))
    Cm = dev.full((2, 3), np.nan)
    jx.gemm(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), 2, 3, 3, precision=jx.PREC_EXACT, stream=dev.stream)
    assert np.array_equal(dev.get(Cm), a)
