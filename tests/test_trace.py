"""The native tracer (jx_graph_* / jx_program_*) without a GPU: graph
recording, structural sharing, reverse-mode node construction, fusion into
op-tapes under the tape limits, and NVRTC compilation of every tape."""
import importlib

import pytest


@pytest.fixture(scope="module")
def tr():
    return importlib.import_module("jax-rs_b200.trace")


def chain(t):
    return lambda x, a, b: t.gelu(x * a + b) * t.sigmoid(x) - t.tanh(x) / 2


def test_identical_nodes_are_shared(tr):
    g = tr.Graph()
    x = g.input()
    a, b = tr.tanh(x), tr.tanh(x)
    assert a.id == b.id
    assert g.const(2.0).id == g.const(2.0).id
    assert g.const(2.0).id != g.const(-2.0).id
    assert g.size() == (4, 1)  # x, tanh, 2, -2


def test_chain_fuses_into_one_tape(tr):
    p = tr.jit(chain(tr), 3)
    info = p.info()
    assert info == {"tapes": 1, "inputs": 3, "outputs": 1, "scratch": 0}
    p.check()


def test_value_and_grad_of_chain_is_one_tape(tr):
    p = tr.value_and_grad(chain(tr), 3, argnums=(0, 1, 2))
    info = p.info()
    assert info["outputs"] == 4 and info["scratch"] == 0
    assert info["tapes"] >= 1
    p.check()


def test_wide_sum_splits_on_the_input_limit(tr):
    # six program inputs cannot feed one tape (4 inputs at most)
    p = tr.jit(lambda a, b, c, d, e, f: a + b + c + d + e + f, 6)
    info = p.info()
    assert info["tapes"] >= 2
    p.check()


def test_long_chain_splits_on_the_instruction_limit(tr):
    def f(x):
        y = x
        for i in range(150):
            y = tr.tanh(y * (1.0 + i * 1e-3))
        return y
    p = tr.jit(f, 1)
    info = p.info()
    assert info["tapes"] >= 3 and info["scratch"] >= 1
    p.check()


def test_register_pressure_splits(tr):
    # twenty values all alive until a final reduction tree
    def f(x):
        vs = [tr.sin(x * float(k + 1)) for k in range(20)]
        while len(vs) > 1:
            vs = [vs[i] + vs[i + 1] if i + 1 < len(vs) else vs[i] for i in range(0, len(vs), 2)]
        return vs[0]
    p = tr.jit(f, 1)
    assert p.info()["tapes"] >= 1
    p.check()


def test_outputs_may_be_inputs_or_constants(tr):
    g = tr.Graph()
    x = g.input()
    p = g.compile([x, g.const(3.5), tr.exp(x), x])
    assert p.info()["outputs"] == 4
    p.check()


def test_vjp_of_unused_input_is_zero_constant(tr):
    g = tr.Graph()
    x, y = g.input(), g.input()
    (gy,) = g.vjp([tr.exp(x)], [g.const(1.0)], [y])
    assert gy.id == g.const(0.0).id


def test_every_op_has_a_derivative_or_a_clear_error(tr):
    jx = importlib.import_module("jax-rs_b200")
    g = tr.Graph()
    x, y = g.input(), g.input()
    outs = [x + y, x - y, x * y, x / y, x ** y, tr.maximum(x, y), tr.minimum(x, y), tr.where_positive(x, y)]
    outs += [f(x) for f in (tr.tanh, tr.exp, tr.log, tr.sin, tr.cos, tr.sqrt, tr.square, tr.reciprocal,
                            tr.relu, tr.gelu, tr.sigmoid)] + [-x, abs(x)]
    grads = g.vjp(outs, [g.const(1.0)] * len(outs), [x, y])
    g.compile(grads).check()
    with pytest.raises(jx.JaxRsError) as e:
        g.vjp([g.unary("gelu_grad", x)], [g.const(1.0)], [x])
    assert "no derivative" in e.value.message


def test_bad_operands_are_rejected(tr):
    jx = importlib.import_module("jax-rs_b200")
    g = tr.Graph()
    with pytest.raises(jx.JaxRsError):
        jx.call("jx_graph_unary", g.handle, 4, 99, jx.C.byref(jx.C.c_int()))
    with pytest.raises(jx.JaxRsError):
        jx.call("jx_graph_binary", g.handle, 42, 0, 0, jx.C.byref(jx.C.c_int()))
