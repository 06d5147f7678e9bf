"""The oracle (C restatement of the reference CPU paths) against the
reference's own known answers and an independent PRNG restatement."""
import json
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _cases():
    with open(os.path.join(GOLD, "known_answers.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_known_answer(oracle, case):
    O = oracle
    op = case["op"]
    if op == "matmul":
        got = O.matmul(np.array(case["a"], np.float32), np.array(case["b"], np.float32))
        np.testing.assert_allclose(got, case["expected"], rtol=case["rtol"], atol=case["atol"])
    elif op == "reduce_all":
        got = O.reduce_all(np.array(case["x"], np.float32), case["red"])
        assert abs(got - case["expected"]) <= case["atol"] + case["rtol"] * abs(case["expected"])
    elif op == "reduce_axis":
        got = O.reduce_axis(np.array(case["x"], np.float32), case["axis"], case["red"])
        np.testing.assert_allclose(got, case["expected"], rtol=case["rtol"], atol=case["atol"])
    elif op in ("argmax", "argmin"):
        got = O.arg_rows(np.array(case["x"], np.float32), is_max=(op == "argmax"))
        assert got.tolist() == case["expected"]
    elif op == "binary":
        got = O.binary(case["bin"], np.array(case["a"], np.float32), np.array(case["b"], np.float32))
        np.testing.assert_allclose(got, case["expected"], rtol=case["rtol"], atol=case["atol"])
    elif op == "unary":
        got = O.unary(case["un"], np.array(case["x"], np.float32))
        np.testing.assert_allclose(got, case["expected"], rtol=case["rtol"], atol=case["atol"])
    elif op == "fft":
        x = np.array(case["x"], np.float32)
        z = np.stack([x, np.zeros_like(x)], -1)
        got = O.fft_c2c(z)
        np.testing.assert_allclose(got[0], case["expected_dc"], atol=case["atol"])
    elif op == "fft_roundtrip":
        x = np.array(case["x"], np.float32)
        z = np.stack([x, np.zeros_like(x)], -1)
        back = O.fft_c2c(O.fft_c2c(z), inverse=True)
        np.testing.assert_allclose(back[:, 0], x, atol=case["atol"])
    elif op == "fft2_roundtrip":
        x = np.array(case["x"], np.float32)
        z = np.stack([x, np.zeros_like(x)], -1)
        back = O.fft2_c2c(O.fft2_c2c(z), inverse=True)
        np.testing.assert_allclose(back[..., 0], x, atol=case["atol"])
    elif op == "conv2d_const":
        x = np.full(case["x_shape"], case["x_value"], np.float32)
        w = np.full(case["w_shape"], case["w_value"], np.float32)
        y = O.conv2d_fwd(x, w, case["stride"], case["pad"])
        assert list(y.shape) == case["expected_shape"]
        np.testing.assert_allclose(y, case["expected_value"], rtol=case["rtol"], atol=case["atol"])
    elif op == "softmax":
        y = O.softmax_rows(np.array(case["x"], np.float32))
        assert abs(y.sum() - case["row_sum"]) < case["atol"]
        assert np.all(np.diff(y[0]) > 0)
    elif op == "normal_seed":
        got = O.normal(O.key_from_seed(case["seed"]), case["n"])
        np.testing.assert_allclose(got, case["expected"], rtol=case["rtol"], atol=case["atol"])
    elif op == "conv1d":
        y = O.conv1d(np.array(case["x"], np.float32), np.array(case["w"], np.float32), case["stride"], case["pad"])
        if "expected_shape" in case:
            assert list(y.shape) == case["expected_shape"]
        else:
            np.testing.assert_allclose(y, case["expected"], rtol=case["rtol"], atol=case["atol"])
    elif op == "pool2d":
        y = O.pool2d(np.array(case["x"], np.float32), tuple(case["kernel"]), tuple(case["stride"]),
                     tuple(case["pad"]), is_max=case["max"])
        assert y.tolist() == case["expected"]
    elif op == "global_pool":
        y = O.global_pool(np.array(case["x"], np.float32), is_max=case["max"])
        assert y.tolist() == case["expected"]
    elif op == "batchnorm":
        x = np.array(case["x"], np.float32)
        g = np.array(case["gamma"], np.float32) if "gamma" in case else None
        b = np.array(case["beta"], np.float32) if "beta" in case else None
        y, _, _ = O.batchnorm(x, case["outer"], case["channels"], case["inner"], case["eps"], g, b)
        flat = y.reshape(-1)
        if "check" in case:
            for i, v in case["check"].items():
                assert abs(flat[int(i)] - v) < case["atol"]
        if "all_within" in case:
            assert np.all(np.abs(flat) < case["all_within"])
        if "mean_within" in case:
            assert abs(float(np.sum(flat, dtype=np.float32)) / flat.size) < case["mean_within"]
        if "expected_shape" in case:
            assert list(y.shape) == case["expected_shape"]
    else:
        pytest.fail("unknown case " + op)


def test_prng_matches_python_restatement(oracle):
    O = oracle
    with open(os.path.join(GOLD, "prng_vectors.json")) as f:
        cases = json.load(f)["cases"]
    for c in cases:
        k = O.key_from_seed(c["seed"])
        assert [hex(k.s0), hex(k.s1)] == c["key"]
        a, b = k.split()
        assert [hex(a.s0), hex(a.s1)] == c["split0"]
        assert [hex(b.s0), hex(b.s1)] == c["split1"]
        ka = O.Key(a.s0, a.s1)
        assert [hex(O.next_u64(ka)) for _ in range(8)] == c["u64_from_split0"]
        u = O.uniform(O.Key(b.s0, b.s1), 8)
        assert (u * np.float32(1 << 24)).astype(np.int64).tolist() == c["f32_numerators_from_split1"]
        r = O.randint(O.Key(b.s0, b.s1), 8, 0, 10)
        assert r.astype(np.int64).tolist() == c["randint_0_10_from_split1"]


def test_split_n_chain(oracle):
    O = oracle
    k = O.key_from_seed(7)
    keys = k.split_n(3)
    cur = k
    for i in range(3):
        a, b = cur.split()
        assert (keys[i].s0, keys[i].s1) == (a.s0, a.s1)
        cur = b


def test_oracle_matmul_vs_f64(oracle):
    O = oracle
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (33, 70)).astype(np.float32)
    b = rng.uniform(-1, 1, (70, 21)).astype(np.float32)
    c = O.matmul(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.abs(c - ref).max() < 1e-5
    np.testing.assert_allclose(O.matmul_f64(a, b), ref, rtol=1e-12, atol=1e-12)
    # the row-parallel path computes the same bits
    assert np.array_equal(O.matmul(a, b, nthreads=4), c)


def test_oracle_fft_vs_dft(oracle):
    O = oracle
    rng = np.random.default_rng(1)
    z = rng.standard_normal((64, 2)).astype(np.float32)
    got = O.fft_c2c(z)
    ref = O.dft_f64(z)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6
    np.testing.assert_allclose(ref[:, 0] + 1j * ref[:, 1], np.fft.fft(z[:, 0] + 1j * z[:, 1]), atol=1e-9)


def test_oracle_chain_vjp_matches_finite_difference(oracle):
    O = oracle
    x = np.linspace(-3, 3, 61).astype(np.float32)
    a, b = 1.2, 0.7
    _, dx = O.chain_vjp(x, a, b)
    y64, dx64 = O.chain_f64(x, a, b)
    np.testing.assert_allclose(dx, dx64, rtol=1e-5, atol=1e-6)
    h = 1e-6
    xp = x.astype(np.float64)
    fd = (O.chain_f64((xp + h).astype(np.float32), a, b)[0] - O.chain_f64((xp - h).astype(np.float32), a, b)[0])
    # central difference on the f64 twin, step limited by f32 input rounding
    step = (xp + h).astype(np.float32).astype(np.float64) - (xp - h).astype(np.float32).astype(np.float64)
    ok = step > 0
    np.testing.assert_allclose(fd[ok] / step[ok], dx64[ok], rtol=2e-2, atol=2e-2)


def test_oracle_conv_adjoints(oracle):
    """<conv(x,w), g> == <x, dX(g)> == <w, dW(x,g)> in f64 (adjoint identity)."""
    O = oracle
    rng = np.random.default_rng(2)
    x = rng.standard_normal((2, 3, 7, 6)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 3)).astype(np.float32)
    for stride, pad in ((1, 1), (2, 0), (2, 1)):
        y = O.conv2d_fwd(x, w, stride, pad)
        g = rng.standard_normal(y.shape).astype(np.float32)
        dx = O.conv2d_bwd_data(g, w, x.shape, stride, pad)
        dw = O.conv2d_bwd_filter(x, g, w.shape, stride, pad)
        lhs = float((y.astype(np.float64) * g).sum())
        assert abs(lhs - float((x.astype(np.float64) * dx).sum())) < 1e-3 * max(1, abs(lhs))
        assert abs(lhs - float((w.astype(np.float64) * dw).sum())) < 1e-3 * max(1, abs(lhs))


def test_oracle_argmax_ties_and_nan(oracle):
    O = oracle
    x = np.array([[1, 5, 5, 2], [7, 7, 7, 7], [-np.inf] * 4], np.float32)
    assert O.arg_rows(x, True).tolist() == [2, 3, 3]
    assert O.arg_rows(x, False).tolist() == [0, 0, 0]
    with pytest.raises(ValueError):
        O.arg_rows(np.array([[1, np.nan]], np.float32))


def test_oracle_adam_first_steps(oracle):
    """optim::adam_update doc example (src/optim.rs:116-135): moves params against the gradient."""
    O = oracle
    p = np.array([1.0, 2.0, 3.0], np.float32)
    g = np.array([0.1, 0.2, 0.3], np.float32)
    z = np.zeros(3, np.float32)
    p1, m1, v1 = O.adam_update(p, g, z, z, 0.001, 0.9, 0.999, 1e-8, 1, True)
    assert np.all(p1 < p)
    np.testing.assert_allclose(p - p1, 0.001, rtol=1e-3)  # first step magnitude ~= lr
    np.testing.assert_allclose(m1, np.float32(0.1) * g, rtol=1e-6)


def test_real_fft_known_answers(oracle):
    """src/ops/fft.rs:666-676 test_rfft (3 bins, DC 10), :721-737
    test_irfft_reconstruction (|irfft(rfft(x)) - x| < 1e-4), :740-750 rfftn of
    a 1-D array equals rfft, and fft of real input (:635-646, DC 10, imag 0)."""
    x = np.array([1, 2, 3, 4], np.float32)
    r = oracle.fft_real(x, full=False)
    assert r.size == 6 and abs(r[0, 0] - 10.0) < 1e-5
    f = oracle.fft_real(x)
    assert f.size == 8 and abs(f[0, 0] - 10.0) < 1e-5 and abs(f[0, 1]) < 1e-5
    x8 = np.arange(1, 9, dtype=np.float32)
    assert np.max(np.abs(oracle.irfft(oracle.fft_real(x8, full=False), 8) - x8)) < 1e-4
    img = np.arange(1, 17, dtype=np.float32).reshape(4, 4)
    s = oracle.rfftn2(img)
    assert s.shape == (4, 3, 2)
    assert np.max(np.abs(oracle.irfftn2(s, 4) - img)) < 1e-4
