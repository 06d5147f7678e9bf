"""Tracing front end over the native graph API (jx_graph_* / jx_program_*).

Mirrors the reference's user-facing transformations: ``jit``
(src/trace/jit.rs:44-107), ``vjp``, ``grad`` and ``value_and_grad``
(src/trace/grad.rs:450-837).  A function of ``Var`` arguments is traced once
(operators and the functions below record nodes in a native graph), the
native side differentiates the recorded graph in reverse mode and fuses it
into op-tapes, and the resulting ``Program`` runs on device buffers of any
length.  Everything is elementwise over equal-length f32 vectors; Python
scalars become constants.

    prog = value_and_grad(lambda x, a, b: gelu(x * a + b) * sigmoid(x) - tanh(x) / 2, 3, argnums=(0,))
    prog.run([x_ptr, a_ptr, b_ptr], [y_ptr, dx_ptr], n, stream)
"""
from __future__ import annotations

import ctypes as C
import importlib

_jx = importlib.import_module(__name__.rsplit(".", 1)[0])
_call, _BIN, _UN = _jx.call, _jx.BIN, _jx.UN


def _node(fn, *args) -> int:
    out = C.c_int(0)
    _call(fn, *args, C.byref(out))
    return out.value


class Graph:
    """A native jx_graph: nodes over equal-length f32 vectors."""

    def __init__(self):
        h = C.c_void_p()
        _call("jx_graph_create", C.byref(h))
        self.handle = h

    def input(self) -> "Var":
        return Var(self, _node("jx_graph_input", self.handle))

    def const(self, value: float) -> "Var":
        return Var(self, _node("jx_graph_const", self.handle, C.c_float(value)))

    def lift(self, v) -> "Var":
        if isinstance(v, Var):
            if v.graph is not self:
                raise ValueError("values from different traces cannot be combined")
            return v
        return self.const(float(v))

    def unary(self, op: str, x) -> "Var":
        return Var(self, _node("jx_graph_unary", self.handle, _UN[op], self.lift(x).id))

    def binary(self, op: str, x, y) -> "Var":
        return Var(self, _node("jx_graph_binary", self.handle, _BIN[op], self.lift(x).id, self.lift(y).id))

    def select_gt(self, x, y) -> "Var":
        return Var(self, _node("jx_graph_select_gt", self.handle, self.lift(x).id, self.lift(y).id))

    def size(self):
        n, i = C.c_int(0), C.c_int(0)
        _call("jx_graph_size", self.handle, C.byref(n), C.byref(i))
        return n.value, i.value

    def vjp(self, outs, cts, wrt):
        """Reverse-mode gradient nodes of sum_i <outs[i], cts[i]> with respect to wrt."""
        ids = lambda vs: (C.c_int * len(vs))(*[self.lift(v).id for v in vs])
        grads = (C.c_int * len(wrt))()
        _call("jx_graph_vjp", self.handle, len(outs), ids(outs), ids(cts), len(wrt), ids(wrt), grads)
        return [Var(self, g) for g in grads]

    def compile(self, outs) -> "Program":
        arr = (C.c_int * len(outs))(*[self.lift(v).id for v in outs])
        h = C.c_void_p()
        _call("jx_graph_compile", self.handle, len(outs), arr, C.byref(h))
        return Program(h, self)

    def __del__(self):
        try:
            if self.handle:
                _jx.lib().jx_graph_destroy(self.handle)
        except Exception:
            pass


class Var:
    """A traced value (a node of a Graph)."""
    __slots__ = ("graph", "id")

    def __init__(self, graph: Graph, node: int):
        self.graph, self.id = graph, node

    def __add__(self, o): return self.graph.binary("add", self, o)
    def __radd__(self, o): return self.graph.binary("add", o, self)
    def __sub__(self, o): return self.graph.binary("sub", self, o)
    def __rsub__(self, o): return self.graph.binary("sub", o, self)
    def __mul__(self, o): return self.graph.binary("mul", self, o)
    def __rmul__(self, o): return self.graph.binary("mul", o, self)
    def __truediv__(self, o): return self.graph.binary("div", self, o)
    def __rtruediv__(self, o): return self.graph.binary("div", o, self)
    def __pow__(self, o): return self.graph.binary("pow", self, o)
    def __rpow__(self, o): return self.graph.binary("pow", o, self)
    def __neg__(self): return self.graph.unary("neg", self)
    def __abs__(self): return self.graph.unary("abs", self)


def _un(op):
    def f(x: Var) -> Var:
        return x.graph.unary(op, x)
    f.__name__ = op
    return f


tanh, exp, log, sin, cos, sqrt = _un("tanh"), _un("exp"), _un("log"), _un("sin"), _un("cos"), _un("sqrt")
square, reciprocal, relu, gelu, sigmoid = _un("square"), _un("recip"), _un("relu"), _un("gelu"), _un("sigmoid")


def maximum(x, y):
    g = x.graph if isinstance(x, Var) else y.graph
    return g.binary("max", x, y)


def minimum(x, y):
    g = x.graph if isinstance(x, Var) else y.graph
    return g.binary("min", x, y)


def where_positive(x: Var, y):
    """x > 0 ? y : 0."""
    return x.graph.select_gt(x, y)


class Program:
    """Fused op-tapes for a set of outputs (jx_program)."""

    def __init__(self, handle, graph: Graph):
        self.handle, self._graph = handle, graph

    def info(self):
        v = [C.c_int(0) for _ in range(4)]
        _call("jx_program_info", self.handle, *[C.byref(x) for x in v])
        return dict(zip(("tapes", "inputs", "outputs", "scratch"), (x.value for x in v)))

    def tape_source(self, i: int) -> str:
        t = C.c_void_p()
        _call("jx_program_tape", self.handle, i, C.byref(t))
        need = C.c_size_t(0)
        _call("jx_tape_source", t, None, 0, C.byref(need))
        buf = C.create_string_buffer(need.value)
        _call("jx_tape_source", t, buf, need.value, C.byref(need))
        return buf.value.decode()

    def check(self):
        """NVRTC-compiles every tape's kernel without a GPU (raises on failure)."""
        for i in range(self.info()["tapes"]):
            t = C.c_void_p()
            _call("jx_program_tape", self.handle, i, C.byref(t))
            _call("jx_tape_check", t)

    def run(self, ins, outs, n, stream=None):
        ia = (C.c_void_p * max(len(ins), 1))(*ins)
        oa = (C.c_void_p * max(len(outs), 1))(*outs)
        _call("jx_program_run", self.handle, ia, oa, n, stream)

    def __del__(self):
        try:
            if self.handle:
                _jx.lib().jx_program_destroy(self.handle)
        except Exception:
            pass


def _trace(fn, n_inputs):
    g = Graph()
    xs = [g.input() for _ in range(n_inputs)]
    out = fn(*xs)
    outs = list(out) if isinstance(out, (tuple, list)) else [out]
    return g, xs, [g.lift(o) for o in outs]


def jit(fn, n_inputs: int) -> Program:
    """Trace fn once; the program computes its output(s)."""
    g, _, outs = _trace(fn, n_inputs)
    return g.compile(outs)


def vjp(fn, n_inputs: int, argnums=(0,)) -> Program:
    """Program over n_inputs + (one cotangent per output) inputs computing the
    outputs followed by the cotangent-weighted gradients for argnums."""
    g, xs, outs = _trace(fn, n_inputs)
    cts = [g.input() for _ in outs]
    grads = g.vjp(outs, cts, [xs[i] for i in argnums])
    return g.compile(outs + grads)


def value_and_grad(fn, n_inputs: int, argnums=(0,)) -> Program:
    """Outputs: fn's (single) output, then d output / d x for x in argnums with
    a ones cotangent (elementwise derivatives)."""
    g, xs, outs = _trace(fn, n_inputs)
    if len(outs) != 1:
        raise ValueError("value_and_grad needs a single output")
    grads = g.vjp(outs, [g.const(1.0)], [xs[i] for i in argnums])
    return g.compile(outs + grads)


def grad(fn, n_inputs: int, argnums=(0,)) -> Program:
    """Like value_and_grad without the value output."""
    g, xs, outs = _trace(fn, n_inputs)
    if len(outs) != 1:
        raise ValueError("grad needs a single output")
    return g.compile(g.vjp(outs, [g.const(1.0)], [xs[i] for i in argnums]))
