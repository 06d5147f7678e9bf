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


def test_chain_full_size_sampled_blocks(jx, dev, oracle):
    """The configured 2^28-element chain, forward and value-and-gradient
    tapes, checked in 66 blocks of 4096 elements (the first, the last and 64
    at seeded random offsets) against the oracle's restatement of the same
    blocks; every output finite."""
    import torch
    n, blk = 1 << 28, 4096
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    X = torch.randn(n, device="cuda", generator=g)
    a, b = 1.1, 0.9
    Y = dev.full((n,), np.nan)
    DY, DX = dev.full((n,), np.nan), dev.full((n,), np.nan)
    chain_tape(jx, a, b).run([X.data_ptr()], [Y.data_ptr()], n, dev.stream)
    chain_vjp_tape(jx, a, b).run([X.data_ptr()], [DY.data_ptr(), DX.data_ptr()], n, dev.stream)
    dev.sync()
    assert bool(torch.isfinite(Y).all()) and bool(torch.isfinite(DX).all())
    rng = np.random.default_rng(9)
    starts = [0, n - blk] + list(rng.integers(0, n // blk, 64) * blk)
    for s0 in starts:
        x = X[s0:s0 + blk].cpu().numpy()
        assert _close(Y[s0:s0 + blk].cpu().numpy(), oracle.chain_fwd(x, np.float32(a), np.float32(b)))
        oy, odx = oracle.chain_vjp(x, np.float32(a), np.float32(b))
        assert _close(DY[s0:s0 + blk].cpu().numpy(), oy)
        assert _close(DX[s0:s0 + blk].cpu().numpy(), odx)


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


SAFE_UN = ["neg", "abs", "tanh", "sigmoid", "relu", "square", "gelu"]
SAFE_BIN = ["add", "sub", "mul", "min", "max"]


def _emulate(oracle, code, consts, inputs, n_out):
    """Runs a register-form tape with the oracle's per-op functions (f32)."""
    regs = {i: x for i, x in enumerate(inputs)}
    outs = [None] * n_out
    for op, dst, s0, s1 in code:
        if op == 1:
            regs[dst] = np.full_like(inputs[0], consts[s0])
        elif op == 2:
            outs[dst] = regs[s0].copy()
        elif op == 64:
            regs[dst] = np.where(regs[s0] > 0, regs[s1], np.float32(0)).astype(np.float32)
        elif op >= 48:
            name = [k for k, v in oracle.BINOPS.items() if v == op - 48][0]
            regs[dst] = oracle.binary(name, regs[s0], regs[s1])
        else:
            name = [k for k, v in oracle.UNOPS.items() if v == op - 16][0]
            regs[dst] = oracle.unary(name, regs[s0])
    return outs


@pytest.mark.parametrize("seed", range(12))
def test_random_tapes_vs_oracle(jx, dev, oracle, seed):
    """Random straight-line tapes: value reuse, x op x, both operand orders,
    constants, several inputs/outputs -- exercises the accumulator lowering."""
    rng = np.random.default_rng(seed)
    n_in = int(rng.integers(1, 5))
    n_out = int(rng.integers(1, 4))
    consts = [float(c) for c in rng.uniform(-2, 2, 4).astype(np.float32)]
    defined = list(range(n_in))
    code = []
    for _ in range(int(rng.integers(4, 24))):
        kind = rng.random()
        dst = int(rng.integers(0, 12))
        if kind < 0.1:
            code.append((jx.OP_CONST, dst, int(rng.integers(0, 4)), 0))
        elif kind < 0.45:
            code.append((jx.OP_UNARY + jx.UN[SAFE_UN[rng.integers(len(SAFE_UN))]], dst,
                         int(rng.choice(defined)), 0))
        elif kind < 0.55:
            code.append((jx.OP_SELECT_GT, dst, int(rng.choice(defined)), int(rng.choice(defined))))
        else:
            a = int(rng.choice(defined))
            b = a if rng.random() < 0.2 else int(rng.choice(defined))
            code.append((jx.OP_BINARY + jx.BIN[SAFE_BIN[rng.integers(len(SAFE_BIN))]], dst, a, b))
        if dst not in defined:
            defined.append(dst)
    for j in range(n_out):
        code.append((jx.OP_STORE, j, int(rng.choice(defined)), 0))
    n = 4099
    xs = [rng.standard_normal(n).astype(np.float32) for _ in range(n_in)]
    try:
        tape = jx.Tape(code, consts, n_in, n_out)
    except jx.JaxRsError as e:
        assert "live at once" in e.message  # legitimately too many live values
        return
    X = [dev.put(x) for x in xs]
    Y = [dev.full((n,), np.nan) for _ in range(n_out)]
    tape.run([t.data_ptr() for t in X], [t.data_ptr() for t in Y], n, dev.stream)
    want = _emulate(oracle, code, consts, xs, n_out)
    for j in range(n_out):
        got = dev.get(Y[j])
        assert _close(got, want[j]), (seed, j, code)


def _ulp_grid():
    xs = np.concatenate([np.linspace(-30, 30, 1 << 20, dtype=np.float32),
                         np.logspace(-30, 1.4, 4096).astype(np.float32),
                         -np.logspace(-30, 1.4, 4096).astype(np.float32),
                         np.array([0.0, -0.0, 0.25, -0.25, 0.2499999, 88.0, -87.0, 1e-38], np.float32)])
    return xs


@pytest.mark.parametrize("op,rel,absol", [("exp", 1.5e-6, 0.0), ("tanh", 5e-6, 3e-7), ("sigmoid", 1.5e-6, 1e-30),
                                          ("gelu", 5e-6, 3e-7)])
def test_transcendental_error_bounds(jx, dev, oracle, op, rel, absol):
    """exp/tanh/sigmoid/gelu on the multi-function unit against glibc (the
    reference's libm): per element |d - o| <= rel*|o| + absol."""
    x = _ulp_grid()
    if op == "exp":
        x = x[(x > -87.0) & (x < 88.0)]  # normal-range results (below 2^-126 flushes to zero)
    X, Y = dev.put(x), dev.full(x.shape, np.nan)
    jx.unary(op, X.data_ptr(), Y.data_ptr(), x.size, dev.stream)
    y = dev.get(Y).astype(np.float64)
    o = oracle.unary(op, x).astype(np.float64)
    err = np.abs(y - o)
    bound = rel * np.abs(o) + absol
    worst = int(np.argmax(err - bound))
    assert np.all(err <= bound), (op, float(x[worst]), y[worst], o[worst])


@pytest.mark.parametrize("op,rel,absol", [("exp", 1.5e-6, 0.0), ("tanh", 5e-6, 3e-7), ("sigmoid", 1.5e-6, 1e-30),
                                          ("gelu", 5e-6, 3e-7)])
def test_transcendental_overflow_and_special_values(jx, dev, oracle, op, rel, absol):
    """Arguments where exp overflows or underflows (|x| up to 1e30), infinities
    and NaN: same infinities and NaNs as the reference, finite values within
    the bound (results below 2^-126 flush to zero)."""
    big = np.concatenate([np.linspace(-200, 200, 8001), np.logspace(1, 30, 200), -np.logspace(1, 30, 200)])
    x = np.concatenate([big, [np.inf, -np.inf, np.nan, 88.7, 88.8, -88.7, -103.9, -104.0]]).astype(np.float32)
    X, Y = dev.put(x), dev.full(x.shape, 7.0)
    jx.unary(op, X.data_ptr(), Y.data_ptr(), x.size, dev.stream)
    y = dev.get(Y).astype(np.float64)
    o = oracle.unary(op, x).astype(np.float64)
    assert np.array_equal(np.isnan(y), np.isnan(o)), (op, x[np.isnan(y) != np.isnan(o)])
    inf = np.isinf(o)
    assert np.array_equal(y[inf], o[inf])
    fin = np.isfinite(o) & (np.abs(o) >= 2.0 ** -126)
    err = np.abs(y[fin] - o[fin])
    assert np.all(err <= rel * np.abs(o[fin]) + absol), (op, x[fin][np.argmax(err - rel * np.abs(o[fin]))])
    tiny = np.isfinite(o) & (np.abs(o) < 2.0 ** -126)
    assert np.all(np.abs(y[tiny]) <= 2.0 ** -126 + absol)


def test_tanh_small_arguments_keep_relative_accuracy(jx, dev):
    """Below |x| = 0.05 tanh uses its odd series: relative accuracy holds down
    to the smallest inputs; above it the absolute error stays below 3e-7."""
    x = np.array([1e-30, -1e-20, 1e-10, 3e-5, -0.01, 0.049, 0.1, -0.3, 2.0], np.float32)
    X, Y = dev.put(x), dev.full(x.shape, np.nan)
    jx.unary("tanh", X.data_ptr(), Y.data_ptr(), x.size, dev.stream)
    y = dev.get(Y).astype(np.float64)
    ref = np.tanh(x.astype(np.float64))
    small = np.abs(x) < 0.05
    np.testing.assert_allclose(y[small], ref[small], rtol=2e-7)
    assert np.all(np.abs(y[~small] - ref[~small]) <= 3e-7)


def test_div_by_power_of_two_constant_is_exact(jx, dev, oracle):
    """x / 2 lowered to x * 0.5 must give the bits of the IEEE division."""
    code = [(jx.OP_CONST, 1, 0, 0), (jx.OP_BINARY + jx.BIN["div"], 2, 0, 1), (jx.OP_STORE, 0, 2, 0)]
    for c in (2.0, 0.25, -8.0, 3.0):
        tape = jx.Tape(code, [c], 1, 1)
        x = np.random.default_rng(1).standard_normal(1001).astype(np.float32) * 1e3
        X, Y = dev.put(x), dev.full(x.shape, np.nan)
        tape.run([X.data_ptr()], [Y.data_ptr()], x.size, dev.stream)
        assert np.array_equal(dev.get(Y), (x / np.float32(c)).astype(np.float32))


def test_folded_constants_give_the_device_bits(jx, dev):
    """A constant subexpression folded on the host (-(1/3)) gives the bits the
    device's own IEEE ops give; a NaN constant result stays on the device."""
    from test_abi import _folding_tape
    tape = _folding_tape(jx)
    x = np.random.default_rng(2).standard_normal(4099).astype(np.float32) * 100
    X, Y0, Y1 = dev.put(x), dev.full(x.shape, 7.0), dev.full(x.shape, 7.0)
    tape.run([X.data_ptr()], [Y0.data_ptr(), Y1.data_ptr()], x.size, dev.stream)
    assert np.array_equal(dev.get(Y0), x * -(np.float32(1) / np.float32(3)))
    assert np.isnan(dev.get(Y1)).all()


MORE_UNARY = {  # op -> (domain lo, hi, exact)
    "sign": (-3, 3, True), "ceil": (-50, 50, True), "floor": (-50, 50, True), "round": (-50, 50, True),
    "trunc": (-50, 50, True), "tan": (-1.4, 1.4, False), "sinh": (-20, 20, False), "cosh": (-20, 20, False),
    "asin": (-0.999, 0.999, False), "acos": (-0.999, 0.999, False), "atan": (-50, 50, False),
    "asinh": (-50, 50, False), "acosh": (1.0, 50, False), "atanh": (-0.99, 0.99, False),
    "expm1": (-10, 10, False), "log1p": (-0.99, 50, False), "cbrt": (-100, 100, False), "log2": (1e-3, 1e3, False),
}


@pytest.mark.parametrize("op", sorted(MORE_UNARY))
def test_remaining_unary_methods_vs_oracle(jx, dev, oracle, op):
    """Array::tan .. log2 (src/ops/unary.rs:82-541) against the oracle's
    restatement (glibc, and Rust std's own asinh/acosh/atanh formulas):
    the rounding family and sign bit-identical, the rest within
    |d - o| <= 1e-5 |o| + 1e-6."""
    lo, hi, exact = MORE_UNARY[op]
    rng = np.random.default_rng(len(op))
    x = rng.uniform(lo, hi, 100003).astype(np.float32)
    x[:6] = np.array([lo, hi, 0.5 * (lo + hi), 2.5, -2.5, 0.0], np.float32).clip(lo, hi)
    if op == "sign":
        x[6:9] = [np.nan, -0.0, np.inf]
    X, Y = dev.put(x), dev.full(x.shape, 7.0)
    jx.unary(op, X.data_ptr(), Y.data_ptr(), x.size, dev.stream)
    y, o = dev.get(Y), oracle.unary(op, x)
    if exact:
        assert np.array_equal(y, o, equal_nan=True)
    else:
        assert _close(y, o)
