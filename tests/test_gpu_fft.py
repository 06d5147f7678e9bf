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
                                       (1024, 16, 1), (2, 2, 7), (1, 8, 2), (1024, 8, 3), (1024, 32, 3),
                                       (1024, 4, 2)])
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


def test_fft2_1024_in_place_batch5(jx, dev):
    """5 x 1024 x 1024 in place (640 column tiles of the TMA column pass, more
    than the SMs hold at once) against a float64 FFT; the inverse brings x
    back."""
    x = _cplx(np.random.default_rng(12), (5, 1024, 1024))
    X = dev.put(x)
    jx.fft2_c2c(X.data_ptr(), X.data_ptr(), 1024, 1024, 5, False, dev.stream)
    y = dev.get(X)
    z = x[..., 0].astype(np.float64) + 1j * x[..., 1]
    r = np.fft.fft2(z)
    assert normwise_rel(y, np.stack([r.real, r.imag], -1)) <= 1e-5
    jx.fft2_c2c(X.data_ptr(), X.data_ptr(), 1024, 1024, 5, True, dev.stream)
    assert normwise_rel(dev.get(X), x) <= 1e-5


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


# ---- real input / real output (fft, rfft, irfft, rfftn, irfftn) --------------
@pytest.mark.parametrize("n,batch", [(2, 3), (4, 1), (8, 5), (16, 7), (64, 3), (1024, 9), (2048, 5), (4096, 4), (16384, 2)])
@pytest.mark.parametrize("full", [True, False])
def test_real_input_fft_vs_oracle(jx, dev, oracle, n, batch, full):
    rng = np.random.default_rng(n + batch)
    x = rng.standard_normal((batch, n)).astype(np.float32)
    bins = n if full else n // 2 + 1
    X, Y = dev.put(x), dev.full((batch, bins, 2), np.nan)
    jx.call("jx_fft_r2c_f32", X.data_ptr(), Y.data_ptr(), n, batch, 1 if full else 0, dev.stream)
    y = dev.get(Y)
    ref = oracle.fft_real(x, full=full)
    for b in range(batch):
        assert normwise_rel(y[b], ref[b]) <= 1e-5
    y64 = np.fft.fft(x.astype(np.float64), axis=1)[:, :bins]
    assert normwise_rel(y, np.stack([y64.real, y64.imag], axis=-1)) <= 1e-5


@pytest.mark.parametrize("n,batch", [(2, 3), (4, 2), (8, 5), (64, 3), (1024, 9), (2048, 5), (4096, 4), (16384, 2)])
def test_irfft_vs_oracle_and_round_trip(jx, dev, oracle, n, batch):
    rng = np.random.default_rng(7 * n + batch)
    x = rng.standard_normal((batch, n)).astype(np.float32)
    spec = oracle.fft_real(x, full=False)
    spec[:, 0, 1] = 0.37    # imaginary parts of DC and Nyquist do not reach the output
    spec[:, -1, 1] = -1.25
    S, Y = dev.put(spec), dev.full((batch, n), np.nan)
    jx.call("jx_fft_c2r_f32", S.data_ptr(), Y.data_ptr(), n, batch, dev.stream)
    y = dev.get(Y)
    ref = oracle.irfft(spec, n)
    for b in range(batch):
        assert normwise_rel(y[b], ref[b]) <= 1e-5
        assert normwise_rel(y[b], x[b]) <= 1e-5


@pytest.mark.parametrize("h,w,batch", [(1, 2, 2), (4, 4, 1), (8, 16, 3), (64, 128, 2), (256, 512, 2)])
def test_rfftn_irfftn_2d_vs_oracle(jx, dev, oracle, h, w, batch):
    rng = np.random.default_rng(h * w + batch)
    x = rng.standard_normal((batch, h, w)).astype(np.float32)
    m = w // 2 + 1
    X, S = dev.put(x), dev.full((batch, h, m, 2), np.nan)
    jx.call("jx_rfft2_f32", X.data_ptr(), S.data_ptr(), h, w, batch, dev.stream)
    s = dev.get(S)
    ref = oracle.rfftn2(x)
    for b in range(batch):
        assert normwise_rel(s[b], ref[b]) <= 1e-5
    Y = dev.full((batch, h, w), np.nan)
    jx.call("jx_irfft2_f32", S.data_ptr(), Y.data_ptr(), h, w, batch, dev.stream)
    y = dev.get(Y)
    yref = oracle.irfftn2(ref, w)
    for b in range(batch):
        assert normwise_rel(y[b], yref[b]) <= 1e-5
        assert normwise_rel(y[b], x[b]) <= 1e-5


def test_real_fft_rejects_bad_sizes(jx, dev):
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_fft_r2c_f32", None, None, 12, 1, 1, dev.stream)
    assert "power of 2" in e.value.message
