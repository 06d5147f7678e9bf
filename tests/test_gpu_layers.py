"""conv1d, pooling, global pooling and normalisation on the device against
the oracle's restatements of the reference loops.

Tolerances: conv1d, pooling and global max pooling are bit-identical to the
oracle (same loop order, unfused f32).  Global average pooling: |d - o| <=
2e-6 |o| + 1e-6 (tree sum against a sequential one).  Normalisation:
normwise <= 1e-6 against an f64 evaluation of the same formula and <= 2e-5
against the reference-order oracle (whose sequential f32 statistics carry
their own rounding); statistics within 1e-6 relative of f64."""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


def _same(a, b):
    return np.array_equal(a, b, equal_nan=True)


# ---- conv1d -----------------------------------------------------------------
CONV1D = [  # B, C, L, O, K, stride, pad
    (1, 1, 5, 1, 3, 1, 0),       # nn::conv1d's own case
    (2, 3, 100, 5, 3, 1, 1),
    (3, 16, 1000, 70, 5, 2, 2),  # two output-channel tiles, ragged
    (1, 40, 300, 8, 7, 3, 0),
    (2, 1, 17, 3, 17, 1, 0),     # kernel as long as the input
    (1, 2, 10, 3, 4, 1, 5),      # outputs entirely in the padding
    (1, 3, 1000, 4, 200, 1, 0),  # long filter, one input channel per chunk
    (2, 33, 4096, 64, 3, 1, 1),
    (1, 5, 64, 2, 9, 5, 4),
]


@pytest.mark.parametrize("B,C,L,O,K,S,P", CONV1D)
def test_conv1d_bit_identical(jx, dev, oracle, B, C, L, O, K, S, P):
    rng = np.random.default_rng(B * 1000 + C * 10 + K)
    x = rng.standard_normal((B, C, L)).astype(np.float32)
    w = rng.standard_normal((O, C, K)).astype(np.float32)
    ref = oracle.conv1d(x, w, S, P, nthreads=8)
    X, Wt = dev.put(x), dev.put(w)
    Y = dev.full(ref.shape, np.nan)
    jx.call("jx_conv1d_f32", X.data_ptr(), Wt.data_ptr(), Y.data_ptr(), B, C, O, L, K, S, P, dev.stream)
    assert _same(dev.get(Y), ref)


def test_conv1d_skips_padded_taps(jx, dev, oracle):
    """A non-finite filter tap that only ever meets padding must not turn the
    output into NaN (the reference skips padded taps, it does not multiply by
    zero)."""
    B, C, L, O, K, S, P = 1, 2, 50, 3, 5, 1, 2
    rng = np.random.default_rng(7)
    x = rng.standard_normal((B, C, L)).astype(np.float32)
    w = rng.standard_normal((O, C, K)).astype(np.float32)
    w[:, :, 0] = np.inf
    ref = oracle.conv1d(x, w, S, P)
    X, Wt = dev.put(x), dev.put(w)
    Y = dev.full(ref.shape, 0.0)
    jx.call("jx_conv1d_f32", X.data_ptr(), Wt.data_ptr(), Y.data_ptr(), B, C, O, L, K, S, P, dev.stream)
    got = dev.get(Y)
    assert _same(got, ref)
    assert np.isfinite(got[..., :2]).all()  # the inf tap only meets padding there


# ---- pooling ----------------------------------------------------------------
POOL = [  # N-planes as (batch, channels), H, W, kh, kw, sh, sw, ph, pw
    ((1, 1), 4, 4, 2, 2, 2, 2, 0, 0),
    ((2, 3), 2, 5, 2, 2, 1, 2, 0, 0),
    ((4, 8), 56, 56, 3, 3, 2, 2, 1, 1),     # ResNet stem pooling
    ((2, 16), 112, 112, 2, 2, 2, 2, 0, 0),
    ((1, 5), 7, 9, 3, 2, 3, 1, 1, 0),
    ((3, 2), 1, 100, 1, 4, 1, 3, 0, 0),     # 1-D pooling
    ((1, 1), 5, 5, 5, 5, 1, 1, 2, 2),       # windows mostly in the padding
    ((2, 2), 13, 11, 4, 3, 4, 3, 0, 0),
]


@pytest.mark.parametrize("dims,H,W,kh,kw,sh,sw,ph,pw", POOL)
@pytest.mark.parametrize("is_max", [True, False])
def test_pool2d_bit_identical(jx, dev, oracle, dims, H, W, kh, kw, sh, sw, ph, pw, is_max):
    B, C = dims
    rng = np.random.default_rng(H * W + kh)
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    ref = oracle.pool2d(x, (kh, kw), (sh, sw), (ph, pw), is_max=is_max)
    X = dev.put(x)
    Y = dev.full(ref.shape, np.nan)
    jx.call("jx_pool2d_f32", X.data_ptr(), Y.data_ptr(), B, C, H, W, kh, kw, sh, sw, ph, pw,
            jx.POOL_MAX if is_max else jx.POOL_AVG, dev.stream)
    assert _same(dev.get(Y), ref)


def test_maxpool_nan_and_avgpool_wrappers(jx, dev, oracle):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 4, 9, 9)).astype(np.float32)
    x[0, 0, 1, 1] = np.nan  # f32::max ignores a NaN operand
    x[1, 2, :3, :3] = -np.inf
    for name, is_max in (("jx_maxpool2d_f32", True), ("jx_avgpool2d_f32", False)):
        ref = oracle.pool2d(x, (3, 3), (2, 2), (1, 1), is_max=is_max)
        X = dev.put(x)
        Y = dev.full(ref.shape, 0.0)
        jx.call(name, X.data_ptr(), Y.data_ptr(), 2, 4, 9, 9, 3, 3, 2, 1, dev.stream)
        assert _same(dev.get(Y), ref), name


@pytest.mark.parametrize("B,C,H,W", [(1, 1, 2, 2), (8, 64, 56, 56), (3, 5, 7, 7), (2, 3, 1, 1), (1, 2, 33, 31)])
def test_global_pool(jx, dev, oracle, B, C, H, W):
    x = np.random.default_rng(B + C + H).standard_normal((B, C, H, W)).astype(np.float32)
    X = dev.put(x)
    for is_max in (True, False):
        ref = oracle.global_pool(x, is_max=is_max)
        Y = dev.full((B, C), np.nan)
        jx.call("jx_global_pool2d_f32", X.data_ptr(), Y.data_ptr(), B, C, H, W,
                jx.POOL_MAX if is_max else jx.POOL_AVG, dev.stream)
        got = dev.get(Y)
        if is_max:
            assert _same(got, ref)
        else:
            assert np.all(np.abs(got - ref) <= 2e-6 * np.abs(ref) + 1e-6)


# ---- normalisation ----------------------------------------------------------
NORM = [  # outer (batch), channels, inner (spatial), affine
    (2, 3, 1, False),         # nn::batch_norm's own case
    (8, 16, 3136, True),      # NCHW feature map, wide rows
    (1000, 37, 1, False),     # batch_norm [batch, features], narrow
    (4, 5, 7, True),          # odd spatial size
    (1, 1, 100003, False),    # layer_norm over a whole array
    (3, 2, 130, True),        # wide, not a multiple of 4
    (64, 256, 49, True),      # 7x7 maps
]


def _norm_f64(x, outer, C, inner, eps, g, b):
    x3 = x.reshape(outer, C, inner).astype(np.float64)
    m = x3.mean(axis=(0, 2))
    v = ((x3 - m[None, :, None]) ** 2).mean(axis=(0, 2))
    y = (x3 - m[None, :, None]) / np.sqrt(v + eps)[None, :, None]
    if g is not None:
        y = y * g[None, :, None] + b[None, :, None]
    return y.reshape(x.shape), m, v


@pytest.mark.parametrize("outer,C,inner,affine", NORM)
@pytest.mark.parametrize("offset", [0.0, 1000.0])
def test_batchnorm(jx, dev, oracle, outer, C, inner, affine, offset):
    rng = np.random.default_rng(outer + C + inner)
    x = (offset + rng.standard_normal(outer * C * inner) * rng.uniform(0.5, 2.0)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, C).astype(np.float32) if affine else None
    b = rng.standard_normal(C).astype(np.float32) if affine else None
    eps = 1e-5
    X = dev.put(x)
    Y = dev.full(x.shape, np.nan)
    M, V = dev.full((C,), np.nan), dev.full((C,), np.nan)
    G = dev.put(g) if affine else None
    Bt = dev.put(b) if affine else None
    jx.call("jx_batchnorm_f32", X.data_ptr(), G.data_ptr() if affine else None, Bt.data_ptr() if affine else None,
            Y.data_ptr(), outer, C, inner, eps, M.data_ptr(), V.data_ptr(), dev.stream)
    y, m, v = dev.get(Y), dev.get(M), dev.get(V)
    y64, m64, v64 = _norm_f64(x, outer, C, inner, eps, g, b)
    assert np.all(np.abs(m - m64) <= 1e-6 * np.abs(m64) + 1e-7)
    assert np.all(np.abs(v - v64) <= 1e-6 * v64 + 1e-12)
    assert normwise_rel(y, y64) <= 1e-6
    if offset == 0.0:
        ref, _, _ = oracle.batchnorm(x, outer, C, inner, eps, g, b)
        assert normwise_rel(y, ref) <= 2e-5


def test_batchnorm_zero_variance_is_zero(jx, dev):
    """Constant channels (the reference's zero-variance test) normalise to exactly 0."""
    x = np.tile(np.array([5.0, 3.0, 7.0], np.float32), (64, 1))
    X = dev.put(x)
    Y = dev.full(x.shape, np.nan)
    jx.call("jx_batchnorm_f32", X.data_ptr(), None, None, Y.data_ptr(), 64, 3, 1, 1e-5, None, None, dev.stream)
    assert np.all(dev.get(Y) == 0.0)


def test_batchnorm_large_feature_map_properties(jx, dev):
    """[64, 256, 56, 56]: every channel of the output has mean 0 and variance
    var/(var+eps) to f64 accuracy (size-independent check at full size)."""
    import torch
    B, C, HW = 64, 256, 56 * 56
    gen = torch.Generator(device="cuda").manual_seed(11)
    X = torch.randn(B, C, HW, device="cuda", generator=gen) * 3.0 + 0.5
    Y = torch.empty_like(X)
    V = dev.full((C,), np.nan)
    jx.call("jx_batchnorm_f32", X.data_ptr(), None, None, Y.data_ptr(), B, C, HW, 1e-5, None, V.data_ptr(),
            dev.stream)
    dev.sync()
    y64 = Y.double()
    mean = y64.mean(dim=(0, 2))
    var = y64.var(dim=(0, 2), unbiased=False)
    v = V.double()
    assert float(mean.abs().max()) < 1e-6
    assert float((var - v / (v + 1e-5)).abs().max()) < 1e-5
