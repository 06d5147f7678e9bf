"""conv2d forward / input gradient / weight gradient against the oracle's
restatement of conv2d_batched's loop (src/nn.rs:2097-2138) and its adjoints.
Tolerance: normwise relative error <= 1e-5."""
import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["one_cta", "pair"])
def kernel(jx, request):
    """Runs the test on each implicit kernel (one-CTA 128x256 tiles, SM-pair
    256x256 tiles); the automatic choice takes the pair kernel only once a
    pass's tiles fill 90% of the SM pairs, which these shapes mostly do not."""
    jx.call("jx_conv_set_kernel", jx.CONV_ONE_CTA if request.param == "one_cta" else jx.CONV_PAIR)
    yield request.param
    jx.call("jx_conv_set_kernel", jx.CONV_AUTO)


def _conv(jx, dev, name, a, b, out_shape, geo):
    A, Bt = dev.put(a), dev.put(b)
    Y = dev.full(out_shape, np.nan)
    jx.call(name, A.data_ptr(), Bt.data_ptr(), Y.data_ptr(), *geo, dev.stream)
    return dev.get(Y)


def test_doc_example(jx, dev):
    """conv2d_batched doc-test (src/nn.rs:2039-2047): ones [1,3,8,8] * 0.1 [16,3,3,3] -> [1,16,6,6] of 2.7."""
    x = np.ones((1, 3, 8, 8), np.float32)
    w = np.full((16, 3, 3, 3), 0.1, np.float32)
    y = _conv(jx, dev, "jx_conv2d_fwd_f32", x, w, (1, 16, 6, 6), (1, 3, 8, 8, 16, 3, 3, 1, 0))
    np.testing.assert_allclose(y, 2.7, rtol=1e-6, atol=1e-5)


CASES = [
    # B, C, H, W, O, KH, KW, stride, pad
    (1, 1, 5, 5, 1, 3, 3, 1, 0),
    (2, 3, 7, 6, 4, 3, 3, 1, 1),
    (3, 5, 9, 11, 7, 3, 3, 2, 1),
    (2, 4, 8, 8, 6, 1, 1, 1, 0),
    (1, 6, 10, 7, 5, 5, 3, 2, 2),
    (2, 16, 14, 14, 32, 3, 3, 1, 1),
    (1, 3, 6, 6, 2, 6, 6, 1, 0),
    (4, 64, 12, 12, 48, 3, 3, 1, 1),
    # O above one 128-row tile; odd stride and kernel extents
    (2, 8, 9, 9, 130, 3, 3, 1, 1),
    (3, 3, 17, 13, 5, 4, 2, 3, 1),
    # C*KH*KW = 4608 exceeds the implicit kernel's gather table: forward and
    # weight gradient take the explicit im2col path, the input gradient
    # (O*KH*KW = 36) the implicit one
    (1, 512, 5, 5, 4, 3, 3, 1, 1),
]


@pytest.mark.parametrize("case", CASES)
def test_fwd_dx_dw_vs_oracle(jx, dev, oracle, kernel, case):
    B, C, H, W, O, KH, KW, S, P = case
    rng = np.random.default_rng(sum(case))
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = rng.standard_normal((O, C, KH, KW)).astype(np.float32)
    y_ref = oracle.conv2d_fwd(x, w, S, P)
    y = _conv(jx, dev, "jx_conv2d_fwd_f32", x, w, y_ref.shape, case)
    assert normwise_rel(y, y_ref) <= 1e-5
    g = rng.standard_normal(y_ref.shape).astype(np.float32)
    dx_ref = oracle.conv2d_bwd_data(g, w, x.shape, S, P)
    dx = _conv(jx, dev, "jx_conv2d_bwd_data_f32", g, w, x.shape, case)
    assert normwise_rel(dx, dx_ref) <= 1e-5
    dw_ref = oracle.conv2d_bwd_filter(x, g, w.shape, S, P)
    dw = _conv(jx, dev, "jx_conv2d_bwd_filter_f32", x, g, w.shape, case)
    assert normwise_rel(dw, dw_ref) <= 1e-5


# Larger "same" convolutions: a partial second 128-row output-channel tile
# for the forward, 5x5 taps, 1x1 taps and 64-pixel rows.
PAIR_CASES = [
    (20, 64, 16, 16, 96, 3, 3, 1, 1),
    (8, 32, 40, 24, 288, 5, 5, 1, 2),
    (10, 32, 32, 64, 64, 1, 1, 1, 0),
]


@pytest.mark.parametrize("case", PAIR_CASES)
def test_same_padding_shapes_vs_oracle(jx, dev, oracle, kernel, case):
    B, C, H, W, O, KH, KW, S, P = case
    rng = np.random.default_rng(7 + sum(case))
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = rng.standard_normal((O, C, KH, KW)).astype(np.float32)
    y_ref = oracle.conv2d_fwd(x, w, S, P, nthreads=8)
    y = _conv(jx, dev, "jx_conv2d_fwd_f32", x, w, y_ref.shape, case)
    assert np.isfinite(y).all()
    assert normwise_rel(y, y_ref) <= 1e-5
    g = rng.standard_normal(y_ref.shape).astype(np.float32)
    dx_ref = oracle.conv2d_bwd_data(g, w, x.shape, S, P, nthreads=8)
    dx = _conv(jx, dev, "jx_conv2d_bwd_data_f32", g, w, x.shape, case)
    assert np.isfinite(dx).all()
    assert normwise_rel(dx, dx_ref) <= 1e-5
    dw_ref = oracle.conv2d_bwd_filter(x, g, w.shape, S, P, nthreads=8)
    dw = _conv(jx, dev, "jx_conv2d_bwd_filter_f32", x, g, w.shape, case)
    assert np.isfinite(dw).all()
    assert normwise_rel(dw, dw_ref) <= 1e-5


def test_set_kernel_rejects_unknown(jx):
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_conv_set_kernel", 7)
    assert e.value.status == jx.JX_EINVAL


def test_rejects_bad_shapes(jx, dev):
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_conv2d_fwd_f32", 1, 1, 1, 1, 3, 4, 4, 8, 7, 7, 1, 0, None)
    assert "Kernel height too large" in e.value.message
    with pytest.raises(jx.JaxRsError):
        jx.call("jx_conv2d_fwd_f32", 1, 1, 1, 1, 3, 4, 4, 8, 3, 3, 0, 0, None)


def test_pair_and_one_cta_kernels_agree(jx, dev):
    """Both implicit kernels split the operands the same way and promote the
    same 128-long partial sums, on a shape large enough for the automatic
    choice to take the pair kernel (batch 16 of 256 x 28 x 28, 3x3)."""
    import torch
    B, C, H, W, O, K = 16, 256, 28, 28, 256, 3
    geo = (B, C, H, W, O, K, K, 1, 1)
    g_ = torch.Generator(device="cuda")
    g_.manual_seed(9)
    X = torch.randn((B, C, H, W), device="cuda", generator=g_)
    Wt = torch.randn((O, C, K, K), device="cuda", generator=g_)
    G = torch.randn((B, O, H, W), device="cuda", generator=g_)
    outs = {}
    try:
        for which in (jx.CONV_ONE_CTA, jx.CONV_PAIR):
            jx.call("jx_conv_set_kernel", which)
            Y, DX, DW = torch.empty_like(G), torch.empty_like(X), torch.empty_like(Wt)
            jx.call("jx_conv2d_fwd_f32", X.data_ptr(), Wt.data_ptr(), Y.data_ptr(), *geo, dev.stream)
            jx.call("jx_conv2d_bwd_data_f32", G.data_ptr(), Wt.data_ptr(), DX.data_ptr(), *geo, dev.stream)
            jx.call("jx_conv2d_bwd_filter_f32", X.data_ptr(), G.data_ptr(), DW.data_ptr(), *geo, dev.stream)
            dev.sync()
            outs[which] = [t.cpu().numpy() for t in (Y, DX, DW)]
    finally:
        jx.call("jx_conv_set_kernel", jx.CONV_AUTO)
    for a, b in zip(outs[jx.CONV_ONE_CTA], outs[jx.CONV_PAIR]):
        assert np.isfinite(b).all()
        assert normwise_rel(b, a) <= 1e-6


def test_full_config_sampled_image_and_adjoint_identity(jx, dev, oracle):
    """[64,256,56,56] x [256,256,3,3], stride 1, pad 1: image 0 of the forward
    against the oracle, and <conv(x,w), g> = <x, dX(g)> = <w, dW(x, g)> in f64."""
    import torch
    B, C, H, W, O, K = 64, 256, 56, 56, 256, 3
    geo = (B, C, H, W, O, K, K, 1, 1)
    g_ = torch.Generator(device="cuda")
    g_.manual_seed(3)
    X = torch.randn((B, C, H, W), device="cuda", generator=g_)
    Wt = torch.randn((O, C, K, K), device="cuda", generator=g_) * float(np.sqrt(2.0 / (C * K * K)))
    G = torch.randn((B, O, H, W), device="cuda", generator=g_)
    Y = torch.empty((B, O, H, W), device="cuda")
    DX = torch.empty_like(X)
    DW = torch.empty_like(Wt)
    s = dev.stream
    jx.call("jx_conv2d_fwd_f32", X.data_ptr(), Wt.data_ptr(), Y.data_ptr(), *geo, s)
    jx.call("jx_conv2d_bwd_data_f32", G.data_ptr(), Wt.data_ptr(), DX.data_ptr(), *geo, s)
    jx.call("jx_conv2d_bwd_filter_f32", X.data_ptr(), G.data_ptr(), DW.data_ptr(), *geo, s)
    dev.sync()
    x0 = X[:1].cpu().numpy()
    y0_ref = oracle.conv2d_fwd(x0, Wt.cpu().numpy(), 1, 1, nthreads=8)
    assert normwise_rel(Y[:1].cpu().numpy(), y0_ref) <= 1e-5
    lhs = float((Y.double() * G.double()).sum())
    mid = float((X.double() * DX.double()).sum())
    rhs = float((Wt.double() * DW.double()).sum())
    scale = float((Y.double().abs() * G.double().abs()).sum())
    assert abs(lhs - mid) <= 1e-5 * scale
    assert abs(lhs - rhs) <= 1e-5 * scale
