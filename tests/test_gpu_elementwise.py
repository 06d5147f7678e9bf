"""Elementwise kernels and the jit op-tape against the oracle.  Ops without a
transcendental are bit-identical (same f32 op order, no FMA); chains with
tanhf/expf match within |d - o| <= 1e-5*|o| + 1e-6 (CUDA vs glibc ulps)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def chain_tape(jx, a, b):
    """y = gelu(x*a + b) * sigmoid(x) - tanh(x)/2, as the tracer lowers it."""
    U, B = jx.OP_UNARY, jx.OP_BINARY
    code = [
        (jx.OP_CONST, 1, 0, 0), (jx.OP_CONST, 2, 1, 0), (jx.OP_CONST, 3, 2, 0),
        (B + jx.BIN["mul"], 4, 0, 1), (B + jx.BIN["add"], 4, 4, 2), (U + jx.UN["gelu"], 4, 4, 0),
        (U + jx.UN["sigmoid"], 5, 0, 0), (B + jx.BIN["mul"], 4, 4, 5),
        (U + jx.UN["tanh"], 5, 0, 0), (B + jx.BIN["div"], 5, 5, 3), (B + jx.BIN["sub"], 4, 4, 5),
        (jx.OP_STORE, 0, 4, 0),
    ]
    return jx.Tape(code, [a, b, 2.0], 1, 1)


def chain_vjp_tape(jx, a, b):
    """Forward plus dx (ones cotangent), in the oracle's op order."""
    U, B = jx.OP_UNARY, jx.OP_BINARY
    code = [
        (jx.OP_CONST, 1, 0, 0), (jx.OP_CONST, 2, 1, 0), (jx.OP_CONST, 3, 2, 0), (jx.OP_CONST, 4, 3, 0),
        (B + jx.BIN["mul"], 5, 0, 1), (B + jx.BIN["add"], 5, 5, 2),
        (U + jx.UN["gelu"], 6, 5, 0), (U + jx.UN["gelu_grad"], 7, 5, 0),
        (U + jx.UN["sigmoid"], 8, 0, 0), (U + jx.UN["tanh"], 9, 0, 0),
        (B + jx.BIN["mul"], 10, 6, 8), (B + jx.BIN["div"], 11, 9, 4), (B + jx.BIN["sub"], 10, 10, 11),
        (jx.OP_STORE, 0, 10, 0),
        (B + jx.BIN["mul"], 10, 7, 1), (B + jx.BIN["mul"], 10, 10, 8),
        (B + jx.BIN["sub"], 11, 3, 8), (B + jx.BIN["mul"], 11, 8, 11), (B + jx.BIN["mul"], 11, 6, 11),
        (B + jx.BIN["add"], 10, 10, 11),
        (B + jx.BIN["mul"], 11, 9, 9), (B + jx.BIN["sub"], 11, 3, 11), (B + jx.BIN["div"], 11, 11, 4),
        (B + jx.BIN["sub"], 10, 10, 11),
        (jx.OP_STORE, 1, 10, 0),
    ]
    return jx.Tape(code, [a, b, 1.0, 2.0], 1, 2)


def _close(d, o):
    d = np.asarray(d, np.float64)
    o = np.asarray(o, np.float64)
    return np.all(np.abs(d - o) <= 1e-5 * np.abs(o) + 1e-6)


@pytest.mark.parametrize("n", [1, 3, 4, 5, 1023, 4096 + 7, 1 << 20])
def test_chain_tape_vs_oracle(jx, dev, oracle, n):
    k = oracle.key_from_seed(2).split_n(2)
    x = oracle.normal(k[0], n)
    ab = oracle.uniform_range(k[1], 2, 0.5, 1.5)
    a, b = float(ab[0]), float(ab[1])
    X = dev.put(x)
    Y = dev.full((n,), np.nan)
    chain_tape(jx, a, b).run([X.data_ptr()], [Y.data_ptr()], n, dev.stream)
    y = dev.get(Y)
    assert _close(y, oracle.chain_fwd(x, np.float32(a), np.float32(b)))
    y64, _ = oracle.chain_f64(x, a, b)
    assert np.linalg.norm(y - y64) / np.linalg.norm(y64) <= 1e-5


@pytest.mark.parametrize("n", [7, 1 << 16])
def test_chain_vjp_tape_vs_oracle(jx, dev, oracle, n):
    x = oracle.normal(oracle.key_from_seed(5).split()[0], n) * 2
    a, b = 0.8, 1.1
    X = dev.put(x)
    Y, DX = dev.full((n,), np.nan), dev.full((n,), np.nan)
    chain_vjp_tape(jx, a, b).run([X.data_ptr()], [Y.data_ptr(), DX.data_ptr()], n, dev.stream)
    y, dx = dev.get(Y), dev.get(DX)
    oy, odx = oracle.chain_vjp(x, np.float32(a), np.float32(b))
    assert _close(y, oy)
    assert _close(dx, odx)


def test_tape_unaligned_pointers(jx, dev, oracle):
    n = 1001
    x = oracle.normal(oracle.key_from_seed(4).split()[0], n + 1)
    X = dev.put(x)
    Y = dev.full((n + 1,), np.nan)
    chain_tape(jx, 1.0, 1.0).run([X.data_ptr() + 4], [Y.data_ptr() + 4], n, dev.stream)
    y = dev.get(Y)
    assert np.isnan(y[0])
    assert _close(y[1:], oracle.chain_fwd(x[1:], np.float32(1.0), np.float32(1.0)))


EXACT_UNARY = ["neg", "abs", "sqrt", "recip", "square", "relu"]


@pytest.mark.parametrize("op", EXACT_UNARY + ["tanh", "exp", "log", "sin", "cos", "gelu", "sigmoid"])
def test_unary_vs_oracle(jx, dev, oracle, op):
    n = 10001
    x = oracle.normal(oracle.key_from_seed(6).split()[1], n) * 3
    if op in ("sqrt", "log"):
        x = np.abs(x) + 1e-3
    X, Y = dev.put(x), dev.full((n,), np.nan)
    jx.unary(op, X.data_ptr(), Y.data_ptr(), n, dev.stream)
    y = dev.get(Y)
    o = oracle.unary(op, x)
    if op in EXACT_UNARY:
        assert np.array_equal(y, o)
    else:
        assert _close(y, o)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "min", "max"])
@pytest.mark.parametrize("sa,sb", [((1000,), (1000,)), ((2, 1), (1, 3)), ((64, 33), (33,)), ((4, 1, 5), (3, 1)),
                                   ((7,), ())])
def test_binary_broadcast_bit_exact(jx, dev, oracle, op, sa, sb):
    rng = np.random.default_rng(3)
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32) + 3.0
    out_shape = np.broadcast_shapes(sa, sb)
    A, B = dev.put(a), dev.put(b)
    O = dev.full(out_shape, np.nan)
    jx.binary(op, A.data_ptr(), sa, B.data_ptr(), sb, O.data_ptr(), dev.stream)
    got = dev.get(O)
    assert np.array_equal(got, oracle.binary(op, a, b))
