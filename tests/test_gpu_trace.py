"""Traced programs on the device: jit / value_and_grad / vjp of elementwise
functions against the oracle's chain and its VJP, and random expression DAGs
against a float64 evaluation and float64 central differences (the
reference's gradient tests use central differences too,
tests/gradient_correctness.rs:13-39).  Tolerances: forward values as the
elementwise ops (|d - o| <= 1e-5 |o| + 1e-6); gradients of random DAGs
normwise <= 2e-3 against central differences (the differences' own error)."""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tr(jx):
    return importlib.import_module("jax-rs_b200.trace")


def _close(d, o, rel=1e-5, ab=1e-6):
    d, o = np.asarray(d, np.float64), np.asarray(o, np.float64)
    return np.all(np.abs(d - o) <= rel * np.abs(o) + ab)


def _run(dev, prog, ins, n_out):
    n = ins[0].size
    X = [dev.put(x) for x in ins]
    Y = [dev.full((n,), np.nan) for _ in range(n_out)]
    prog.run([x.data_ptr() for x in X], [y.data_ptr() for y in Y], n, dev.stream)
    return [dev.get(y) for y in Y]


def chain(t):
    return lambda x, a, b: t.gelu(x * a + b) * t.sigmoid(x) - t.tanh(x) / 2


def test_jit_chain_matches_oracle(tr, dev, oracle):
    n = 100003
    x = oracle.normal(oracle.key_from_seed(2), n)
    a, b = np.float32(1.1), np.float32(0.9)
    (y,) = _run(dev, tr.jit(chain(tr), 3), [x, np.full(n, a, np.float32), np.full(n, b, np.float32)], 1)
    assert _close(y, oracle.chain_fwd(x, a, b))


def test_value_and_grad_chain_matches_oracle_vjp(tr, dev, oracle):
    n = 65537
    x = oracle.normal(oracle.key_from_seed(4), n)
    a, b = np.float32(0.8), np.float32(1.3)
    prog = tr.value_and_grad(chain(tr), 3, argnums=(0,))
    assert prog.info()["tapes"] == 1 and prog.info()["scratch"] == 0
    y, dx = _run(dev, prog, [x, np.full(n, a, np.float32), np.full(n, b, np.float32)], 2)
    y_ref, dx_ref = oracle.chain_vjp(x, a, b)
    assert _close(y, y_ref)
    assert _close(dx, dx_ref)


def test_vjp_with_cotangent_input(tr, dev, oracle):
    n = 4099
    x = oracle.normal(oracle.key_from_seed(5), n)
    ct = oracle.normal(oracle.key_from_seed(6), n)
    a, b = np.float32(1.1), np.float32(0.9)
    prog = tr.vjp(chain(tr), 3, argnums=(0,))
    y, dx = _run(dev, prog, [x, np.full(n, a, np.float32), np.full(n, b, np.float32), ct], 2)
    y_ref, dx_ref = oracle.chain_vjp(x, a, b, ct)
    assert _close(y, y_ref)
    assert _close(dx, dx_ref)


# ---- random expression DAGs -------------------------------------------------
UNARY = {  # name -> (f64 forward, argument domain transform)
    "tanh": np.tanh, "exp": lambda v: np.exp(np.clip(v, -20, 20)), "sin": np.sin, "cos": np.cos,
    "sigmoid": lambda v: 1.0 / (1.0 + np.exp(-v)), "square": np.square, "neg": np.negative,
    "gelu": lambda v: 0.5 * v * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (v + 0.044715 * v ** 3))),
}


def _random_program(tr, rng, n_inputs, depth):
    """A random DAG as (traced builder, f64 evaluator)."""
    ops = []
    for _ in range(depth):
        kind = rng.integers(0, 3)
        if kind == 0:
            ops.append(("un", rng.choice(list(UNARY))))
        elif kind == 1:
            ops.append(("bin", rng.choice(["add", "sub", "mul"])))
        else:
            ops.append(("scale", float(rng.uniform(0.3, 1.5))))
    picks = [(int(rng.integers(0, 10 ** 6)), int(rng.integers(0, 10 ** 6))) for _ in range(depth)]

    def build(vals, lib):
        vals = list(vals)
        for (kind, arg), (i, j) in zip(ops, picks):
            x, y = vals[i % len(vals)], vals[j % len(vals)]
            if kind == "un":
                if lib is np:
                    v = UNARY[arg](x)
                else:
                    v = {"tanh": tr.tanh, "exp": lambda u: tr.exp(tr.minimum(tr.maximum(u, -20.0), 20.0)),
                         "sin": tr.sin, "cos": tr.cos, "sigmoid": tr.sigmoid, "square": tr.square,
                         "neg": lambda u: -u, "gelu": tr.gelu}[arg](x)
            elif kind == "bin":
                v = {"add": lambda p, q: p + q, "sub": lambda p, q: p - q, "mul": lambda p, q: p * q}[arg](x, y)
            else:
                v = x * arg
            vals.append(v)
        return vals[-1]
    return build


@pytest.mark.parametrize("seed", range(6))
def test_random_dags_value_and_grad(tr, dev, seed):
    rng = np.random.default_rng(100 + seed)
    n_in = int(rng.integers(1, 4))
    build = _random_program(tr, rng, n_in, depth=int(rng.integers(6, 30)))
    prog = tr.value_and_grad(lambda *xs: build(xs, tr), n_in, argnums=tuple(range(n_in)))
    n = 4096
    xs = [rng.uniform(-1.5, 1.5, n).astype(np.float32) for _ in range(n_in)]
    outs = _run(dev, prog, xs, 1 + n_in)
    x64 = [x.astype(np.float64) for x in xs]
    y64 = build(x64, np)
    assert np.linalg.norm(outs[0] - y64) <= 1e-5 * np.linalg.norm(y64) + 1e-5 * np.sqrt(n)
    h = 1e-4
    for k in range(n_in):
        xp = [v.copy() for v in x64]
        xm = [v.copy() for v in x64]
        xp[k] += h
        xm[k] -= h
        fd = (build(xp, np) - build(xm, np)) / (2 * h)
        err = np.linalg.norm(outs[1 + k] - fd)
        assert err <= 2e-3 * np.linalg.norm(fd) + 1e-4 * np.sqrt(n), (seed, k, err, np.linalg.norm(fd))


def test_multi_tape_program_through_scratch(tr, dev):
    """150 chained tanh steps exceed one tape; the split program goes through
    scratch buffers and must equal the step-by-step f64 result."""
    def f(x):
        y = x
        for i in range(150):
            y = tr.tanh(y * (1.0 + i * 1e-3))
        return y
    prog = tr.jit(f, 1)
    assert prog.info()["tapes"] >= 3 and prog.info()["scratch"] >= 1
    x = np.random.default_rng(1).uniform(-2, 2, 10007).astype(np.float32)
    (y,) = _run(dev, prog, [x], 1)
    ref = x.astype(np.float64)
    for i in range(150):
        ref = np.tanh(ref * np.float32(1.0 + i * 1e-3))
    assert np.max(np.abs(y - ref)) <= 2e-5


def test_wide_sum_and_repeated_outputs(tr, dev):
    g = tr.Graph()
    xs = [g.input() for _ in range(6)]
    s = xs[0]
    for v in xs[1:]:
        s = s + v
    prog = g.compile([s, xs[2], g.const(2.5), s])
    n = 1000
    data = [np.random.default_rng(k).standard_normal(n).astype(np.float32) for k in range(6)]
    outs = _run(dev, prog, data, 4)
    ref = data[0]
    for d in data[1:]:
        ref = (ref + d).astype(np.float32)
    assert np.array_equal(outs[0], ref)  # same left-to-right f32 additions
    assert np.array_equal(outs[1], data[2])
    assert np.all(outs[2] == 2.5)
    assert np.array_equal(outs[3], ref)


@pytest.mark.parametrize("op,lo,hi", [("tan", -1.2, 1.2), ("sinh", -3, 3), ("cosh", -3, 3), ("asin", -0.9, 0.9),
                                      ("acos", -0.9, 0.9), ("atan", -3, 3), ("asinh", -3, 3), ("acosh", 1.1, 4),
                                      ("atanh", -0.9, 0.9), ("expm1", -3, 3), ("log1p", -0.9, 3),
                                      ("cbrt", 0.2, 8), ("log2", 0.1, 8), ("floor", -3, 3)])
def test_unary_method_gradients_vs_central_differences(tr, dev, op, lo, hi):
    g = tr.Graph()
    x = g.input()
    y = g.unary(op, x)
    (dx,) = g.vjp([y], [g.const(1.0)], [x])
    prog = g.compile([y, dx])
    xs = np.random.default_rng(3).uniform(lo, hi, 4096).astype(np.float32)
    yv, dxv = _run(dev, prog, [xs], 2)
    f = {"tan": np.tan, "sinh": np.sinh, "cosh": np.cosh, "asin": np.arcsin, "acos": np.arccos,
         "atan": np.arctan, "asinh": np.arcsinh, "acosh": np.arccosh, "atanh": np.arctanh, "expm1": np.expm1,
         "log1p": np.log1p, "cbrt": np.cbrt, "log2": np.log2, "floor": np.floor}[op]
    x64 = xs.astype(np.float64)
    h = 1e-5
    fd = (f(x64 + h) - f(x64 - h)) / (2 * h)
    if op == "floor":
        fd = np.zeros_like(x64)  # zero almost everywhere, as the reference's rule
    assert np.linalg.norm(dxv - fd) <= 1e-4 * np.linalg.norm(fd) + 1e-4 * np.sqrt(xs.size), op
