"""The wide-MLP training path at reduced width, against the oracle.

The wide data-parallel workload is Dense 8192 -> 4 x 8192 (GELU) -> 1000 with
softmax cross-entropy, He-normal init and Adam, every GEMM on the tensor cores
in 3xTF32.  These tests keep that structure (four GELU layers, a wider softmax
head, He-normal weights, 3xTF32, the same jx_mlp_train_step path) at widths the
oracle's restatement (oracle/mlp.py with gelu activations: Array::matmul
src/ops/linalg.rs:215-232, nn::gelu src/nn.rs:111-122, cross_entropy_loss
:300-318, optim::adam_update src/optim.rs:138-189) trains in seconds.

Tolerances: per-step losses within 1e-4 of the oracle's (the training-loss
bound for this path); parameters after the run normwise within 1e-4 (Adam
divides each update by the gradient's own running RMS, so a parameter whose
gradient is near zero can take a different full-size step on rounding noise).
"""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


def he_params(widths, seed):
    """He-normal weights (N(0,1) * sqrt(2 / fan_in)), zero biases."""
    rng = np.random.default_rng(seed)
    Ws = [(rng.standard_normal((widths[l], widths[l + 1])) * np.sqrt(2.0 / widths[l])).astype(np.float32)
          for l in range(len(widths) - 1)]
    bs = [np.zeros(widths[l + 1], np.float32) for l in range(len(widths) - 1)]
    return Ws, bs


def train_device(jx, dev, Ws, bs, data, widths, acts, precision=None):
    precision = jx.PREC_3XTF32 if precision is None else precision
    net = jx.MLP(widths, acts, data[0][0].shape[0], precision)
    net.set_params(net.pack(Ws, bs))
    net.set_adam(1e-3, 0.9, 0.999, 1e-8)
    losses = []
    Lo = dev.full((1,), np.nan)
    for x, y in data:
        X, Y = dev.put(x), dev.put(y)
        net.step(X.data_ptr(), Y.data_ptr(), Lo.data_ptr(), dev.stream)
        losses.append(float(dev.get(Lo)[0]))
    return losses, net.unpack(net.get_params())


@pytest.mark.parametrize("width,classes,batch,steps", [(512, 100, 256, 25), (256, 40, 384, 20)])
def test_wide_mlp_gelu_3xtf32_tracks_oracle(jx, dev, oracle, width, classes, batch, steps):
    import oracle.mlp as OM
    widths = [width] * 5 + [classes]
    acts = ["gelu"] * 4
    Ws, bs = he_params(widths, seed=11)
    data = OM.batches(steps, batch, width, classes, seed=5)
    ol, oW, ob = OM.train(Ws, bs, data, acts=acts, nthreads=8)
    dl, (dW, db) = train_device(jx, dev, Ws, bs, data, widths, acts)
    assert np.isfinite(dl).all()
    assert ol[-1] < ol[0]  # it learns
    worst = max(abs(a - b) for a, b in zip(dl, ol))
    assert worst <= 1e-4, worst
    got = np.concatenate([a.ravel() for a in dW + db])
    want = np.concatenate([a.ravel() for a in oW + ob])
    assert normwise_rel(got, want) <= 1e-4


def test_wide_mlp_first_step_gradient_direction(jx, dev, oracle):
    """One step from the same start: the parameter change (= Adam's first
    update, -lr * sign-like m/sqrt(v)) agrees with the oracle's for all but a
    vanishing fraction of parameters."""
    import oracle.mlp as OM
    widths = [384] * 5 + [64]
    acts = ["gelu"] * 4
    Ws, bs = he_params(widths, seed=12)
    data = OM.batches(1, 200, 384, 64, seed=6)
    _, oW, ob = OM.train(Ws, bs, data, acts=acts, nthreads=8)
    _, (dW, db) = train_device(jx, dev, Ws, bs, data, widths, acts)
    d_dev = np.concatenate([(a - w).ravel() for a, w in zip(dW + db, Ws + bs)])
    d_ora = np.concatenate([(a - w).ravel() for a, w in zip(oW + ob, Ws + bs)])
    agree = np.mean(np.abs(d_dev - d_ora) <= 1e-6)
    assert agree >= 0.999, agree
