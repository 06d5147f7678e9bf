"""Batched FFT against the oracle's restatement of fft_recursive
(src/ops/fft.rs:40-70) and a float64 FFT.  Tolerance: normwise relative error
<= 1e-5 (the reference uses f32 twiddles from f32 angles; both are compared)."""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


def _cplx(rng, shape):
    return rng.standard_normal(shape + (2,)).astype(np.float32)


def _run(jx, dev, x, n, batch, inverse=False, inplace=False):
    X = dev.put(x)
    Y = X if inplace else dev.full(x.shape, np.nan)
    jx.fft_c2c(X.data_ptr(), Y.data_ptr(), n, batch, inverse, dev.stream)
    return dev.get(Y)


def _f64(x, inverse=False):
    z = x[..., 0].astype(np.float64) + 1j * x[..., 1].astype(np.float64)
    r = np.fft.ifft(z, axis=-1) if inverse else np.fft.fft(z, axis=-1)
    return np.stack([r.real, r.imag], -1)


def test_known_answers(jx, dev):
    """fft([1,2,3,4]) DC = 10 (src/ops/fft.rs:635-647); ifft(fft(x)) = x (:649-664)."""
    x = np.array([[1, 0], [2, 0], [3, 0], [4, 0]], np.float32)
    y = _run(jx, dev, x, 4, 1)
    assert abs(y[0, 0] - 10) < 1e-5 and abs(y[0, 1]) < 1e-5
    back = _run(jx, dev, y, 4, 1, inverse=True)
    np.testing.assert_allclose(back[:, 0], [1, 2, 3, 4], atol=1e-5)


@pytest.mark.parametrize("logn", list(range(0, 14)))
@pytest.mark.parametrize("inverse", [False, True])
def test_sizes_vs_oracle(jx, dev, oracle, logn, inverse):
    n = 1 << logn
    batch = max(1, min(64, (1 << 16) // n)) + 1  # odd batch: partial CTAs
    x = _cplx(np.random.default_rng(logn), (batch, n))
    y = _run(jx, dev, x, n, batch, inverse)
    assert normwise_rel(y, oracle.fft_c2c(x, inverse=inverse)) <= 1e-5
    assert normwise_rel(y, _f64(x, inverse)) <= 1e-5


def test_in_place(jx, dev, oracle):
    x = _cplx(np.random.default_rng(5), (33, 4096))
    y = _run(jx, dev, x, 4096, 33, inplace=True)
    assert normwise_rel(y, _f64(x)) <= 1e-5


@pytest.mark.parametrize("h,w,batch", [(4, 4, 1), (8, 32, 3), (32, 8, 2), (64, 64, 5), (16, 1024, 1),
                                       (1024, 16, 1), (2, 2, 7), (1, 8, 2)])
@pytest.mark.parametrize("inverse", [False, True])
def test_fft2_vs_oracle(jx, dev, oracle, h, w, batch, inverse):
    x = _cplx(np.random.default_rng(h * w), (batch, h, w))
    X, Y = dev.put(x), dev.full(x.shape, np.nan)
    jx.fft2_c2c(X.data_ptr(), Y.data_ptr(), h, w, batch, inverse, dev.stream)
    y = dev.get(Y)
    assert normwise_rel(y, oracle.fft2_c2c(x, inverse=inverse)) <= 1e-5
    z = x[..., 0].astype(np.float64) + 1j * x[..., 1]
    r = np.fft.ifft2(z) if inverse else np.fft.fft2(z)
    assert normwise_rel(y, np.stack([r.real, r.imag], -1)) <= 1e-5


def test_ifft2_roundtrip_4x4(jx, dev):
    """src/ops/fft.rs:690-715: ifft2(fft2(x)) == x (real input)."""
    x = np.zeros((4, 4, 2), np.float32)
    x[..., 0] = np.arange(1, 17, dtype=np.float32).reshape(4, 4)
    X, Y, Z = dev.put(x), dev.full(x.shape, np.nan), dev.full(x.shape, np.nan)
    jx.fft2_c2c(X.data_ptr(), Y.data_ptr(), 4, 4, 1, False, dev.stream)
    jx.fft2_c2c(Y.data_ptr(), Z.data_ptr(), 4, 4, 1, True, dev.stream)
    np.testing.assert_allclose(dev.get(Z)[..., 0], x[..., 0], atol=1e-4)


def test_fft2_1024_square(jx, dev, oracle):
    x = _cplx(np.random.default_rng(11), (2, 1024, 1024))
    X, Y = dev.put(x), dev.full(x.shape, np.nan)
    jx.fft2_c2c(X.data_ptr(), Y.data_ptr(), 1024, 1024, 2, False, dev.stream)
    y = dev.get(Y)
    z = x[..., 0].astype(np.float64) + 1j * x[..., 1]
    r = np.fft.fft2(z)
    assert normwise_rel(y, np.stack([r.real, r.imag], -1)) <= 1e-5


def test_full_config_1d_properties(jx, dev, oracle):
    """n = 4096 x 65536 (the configured 2 GiB batch): round trip, Parseval,
    and sampled rows against the oracle."""
    n, batch = 4096, 65536
    rng = np.random.default_rng(3)
    x = rng.standard_normal((batch, n, 2), dtype=np.float32)
    X = dev.put(x)
    Y = dev.full(x.shape, np.nan)
    jx.fft_c2c(X.data_ptr(), Y.data_ptr(), n, batch, False, dev.stream)
    rows = rng.choice(batch, 8, replace=False)
    y_rows = dev.get(Y[rows])
    assert normwise_rel(y_rows, oracle.fft_c2c(x[rows])) <= 1e-5
    # Parseval per transform: sum |X|^2 = n * sum |x|^2 (computed on the device by torch, float64)
    ex = (X.double() ** 2).sum(dim=(1, 2))
    ey = (Y.double() ** 2).sum(dim=(1, 2))
    assert float(((ey / (n * ex)) - 1).abs().max()) <= 1e-5
    jx.fft_c2c(Y.data_ptr(), Y.data_ptr(), n, batch, True, dev.stream)
    err = float(((Y - X).double() ** 2).sum().sqrt() / (X.double() ** 2).sum().sqrt())
    assert err <= 1e-5
