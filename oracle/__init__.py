"""CPU oracle for the jax-rs CUDA backend -- TEST INFRASTRUCTURE ONLY.

This package wraps ``libjaxrs_oracle.so`` (built from ``jaxrs_oracle.c`` by the
Makefile beside it), a C restatement of the jax-rs 0.5.1 CPU code paths
(``src/random.rs``, ``src/ops/linalg.rs``, ``src/ops/reduce.rs``, ``src/nn.rs``,
``src/ops/fft.rs``, ``src/optim.rs``).  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline legs may import it; the product library never
calls into it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libjaxrs_oracle.so")
_lib = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
i64 = C.c_int64


class Key(C.Structure):
    """``PRNGKey { state: [u64; 2] }`` (src/random.rs:15-18)."""

    _fields_ = [("s0", C.c_uint64), ("s1", C.c_uint64)]

    def __repr__(self):
        return f"Key(0x{self.s0:016x}, 0x{self.s1:016x})"

    def split(self):
        a, b = Key(), Key()
        lib().jxo_key_split(C.byref(self), C.byref(a), C.byref(b))
        return a, b

    def split_n(self, n):
        arr = (Key * n)()
        lib().jxo_key_split_n(C.byref(self), n, arr)
        return [Key(k.s0, k.s1) for k in arr]


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    src = os.path.join(_HERE, "jaxrs_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        kp = C.POINTER(Key)
        L.jxo_key_from_seed.argtypes = [C.c_uint64, kp]
        L.jxo_key_split.argtypes = [kp, kp, kp]
        L.jxo_key_split_n.argtypes = [kp, i64, kp]
        L.jxo_next_u64.argtypes = [kp]
        L.jxo_next_u64.restype = C.c_uint64
        L.jxo_uniform.argtypes = [Key, f32p, i64]
        L.jxo_uniform_range.argtypes = [Key, f32p, i64, C.c_float, C.c_float]
        L.jxo_randint.argtypes = [Key, f32p, i64, C.c_int32, C.c_int32]
        L.jxo_normal.argtypes = [Key, f32p, i64]
        L.jxo_matmul.argtypes = [f32p, f32p, f32p, i64, i64, i64, C.c_int]
        L.jxo_matmul_rows.argtypes = [f32p, f32p, f32p, i64, i64, i64, i64, i64, C.c_int]
        L.jxo_matmul_f64.argtypes = [f32p, f32p, f64p, i64, i64, i64]
        L.jxo_bmm.argtypes = [f32p, f32p, f32p, i64, i64, i64, i64, C.c_int]
        L.jxo_transpose.argtypes = [f32p, f32p, i64, i64]
        for nm in ("jxo_gelu", "jxo_gelu_grad", "jxo_sigmoid", "jxo_relu", "jxo_tanh", "jxo_exp"):
            getattr(L, nm).argtypes = [f32p, f32p, i64]
        L.jxo_unary.argtypes = [C.c_int, f32p, f32p, i64]
        L.jxo_binary_broadcast.argtypes = [C.c_int, f32p, C.POINTER(C.c_int64), C.c_int, f32p,
                                           C.POINTER(C.c_int64), C.c_int, f32p,
                                           C.POINTER(C.c_int64), C.POINTER(C.c_int)]
        L.jxo_chain_fwd.argtypes = [f32p, f32p, i64, C.c_float, C.c_float]
        L.jxo_chain_fwd_eager.argtypes = [f32p, f32p, i64, C.c_float, C.c_float]
        L.jxo_chain_vjp.argtypes = [f32p, C.c_void_p, C.c_void_p, f32p, i64, C.c_float, C.c_float]
        L.jxo_chain_f64.argtypes = [f32p, C.c_void_p, C.c_void_p, i64, C.c_float, C.c_float]
        L.jxo_reduce_all.argtypes = [f32p, i64, C.c_int]
        L.jxo_reduce_all.restype = C.c_float
        L.jxo_sum_all_f64.argtypes = [f32p, i64]
        L.jxo_sum_all_f64.restype = C.c_double
        L.jxo_reduce_axis.argtypes = [f32p, f32p, i64, i64, i64, C.c_int, C.c_int]
        L.jxo_sum_rows_f64.argtypes = [f32p, f64p, i64, i64]
        L.jxo_arg_rows.argtypes = [f32p, i32p, i64, i64, C.c_int, C.c_int]
        L.jxo_sum_rows_vjp.argtypes = [f32p, f32p, i64, i64]
        L.jxo_max_rows_vjp.argtypes = [f32p, f32p, f32p, i64, i64]
        L.jxo_fft_c2c.argtypes = [f32p, f32p, i64, i64, C.c_int, C.c_int]
        L.jxo_fft2_c2c.argtypes = [f32p, f32p, i64, i64, i64, C.c_int, C.c_int]
        L.jxo_fft_real.argtypes = [f32p, f32p, i64, i64, C.c_int]
        L.jxo_irfft.argtypes = [f32p, f32p, i64, i64]
        L.jxo_rfftn2.argtypes = [f32p, f32p, i64, i64, i64]
        L.jxo_irfftn2.argtypes = [f32p, f32p, i64, i64, i64]
        L.jxo_dft_f64.argtypes = [f32p, f64p, i64, C.c_int]
        conv = [i64] * 9 + [C.c_int]
        L.jxo_conv2d_fwd.argtypes = [f32p, f32p, f32p] + conv
        L.jxo_conv2d_bwd_data.argtypes = [f32p, f32p, f32p] + conv
        L.jxo_conv2d_bwd_filter.argtypes = [f32p, f32p, f32p] + conv
        L.jxo_softmax_rows.argtypes = [f32p, f32p, i64, i64]
        L.jxo_log_softmax_rows.argtypes = [f32p, f32p, i64, i64]
        L.jxo_one_hot.argtypes = [f32p, f32p, i64, i64]
        L.jxo_cross_entropy.argtypes = [f32p, f32p, i64]
        L.jxo_cross_entropy.restype = C.c_float
        L.jxo_adam_update.argtypes = [f32p, f32p, f32p, f32p, i64, C.c_float, C.c_float, C.c_float,
                                      C.c_float, i64, C.c_int]
        L.jxo_dense_fwd.argtypes = [f32p, f32p, f32p, f32p, i64, i64, i64, C.c_int]
        L.jxo_softmax_xent_bwd.argtypes = [f32p, f32p, f32p, i64, i64]
        L.jxo_col_sum.argtypes = [f32p, f32p, i64, i64]
        L.jxo_conv1d.argtypes = [f32p, f32p, f32p] + [i64] * 7 + [C.c_int]
        L.jxo_pool2d.argtypes = [f32p, f32p] + [i64] * 9 + [C.c_int]
        L.jxo_global_pool.argtypes = [f32p, f32p, i64, i64, C.c_int]
        L.jxo_batchnorm.argtypes = [f32p, C.c_void_p, C.c_void_p, f32p, i64, i64, i64, C.c_float,
                                    C.c_void_p, C.c_void_p]
        L.jxo_channel_stats_f64.argtypes = [f32p, i64, i64, i64, f64p, f64p]
        L.jxo_version.restype = C.c_char_p
        _lib = L
    return _lib


# --------------------------------------------------------------------------
# numpy-facing helpers
# --------------------------------------------------------------------------
def _c(x, dt=np.float32):
    return np.ascontiguousarray(x, dtype=dt)


def key_from_seed(seed: int) -> Key:
    k = Key()
    lib().jxo_key_from_seed(seed, C.byref(k))
    return k


def next_u64(key: Key) -> int:
    return lib().jxo_next_u64(C.byref(key))


def uniform(key: Key, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().jxo_uniform(key, out, n)
    return out


def uniform_range(key: Key, n: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().jxo_uniform_range(key, out, n, lo, hi)
    return out


def randint(key: Key, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().jxo_randint(key, out, n, lo, hi)
    return out


def normal(key: Key, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().jxo_normal(key, out, n)
    return out


def matmul(a, b, nthreads=1):
    a, b = _c(a), _c(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), np.float32)
    lib().jxo_matmul(a, b, c, m, n, k, nthreads)
    return c


def matmul_rows(a, b, r0, r1, nthreads=1):
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((r1 - r0, n), np.float32)
    lib().jxo_matmul_rows(a, b, c, m, n, k, r0, r1, nthreads)
    return c


def matmul_f64(a, b):
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float64)
    lib().jxo_matmul_f64(a, b, c, m, n, k)
    return c


def bmm(a, b, nthreads=1):
    a, b = _c(a), _c(b)
    bt, m, k = a.shape
    n = b.shape[2]
    c = np.empty((bt, m, n), np.float32)
    lib().jxo_bmm(a, b, c, bt, m, n, k, nthreads)
    return c


UNOPS = {"neg": 0, "abs": 1, "sin": 2, "cos": 3, "tanh": 4, "exp": 5, "log": 6, "sqrt": 7, "recip": 8,
         "square": 9, "relu": 10, "gelu": 11, "sigmoid": 12, "tan": 14, "sign": 15, "sinh": 16, "cosh": 17,
         "asin": 18, "acos": 19, "atan": 20, "asinh": 21, "acosh": 22, "atanh": 23, "ceil": 24, "floor": 25,
         "round": 26, "trunc": 27, "expm1": 28, "log1p": 29, "cbrt": 30, "log2": 31}


def unary(name, x):
    x = _c(x)
    y = np.empty_like(x)
    lib().jxo_unary(UNOPS[name], x, y, x.size)
    return y


def gelu_grad(x):
    """Derivative of nn::gelu's tanh form (src/nn.rs:111-122), elementwise."""
    x = _c(x)
    y = np.empty_like(x)
    lib().jxo_gelu_grad(x, y, x.size)
    return y


BINOPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "min": 5, "max": 6}


def binary(op, a, b):
    a, b = _c(a), _c(b)
    ad = (C.c_int64 * max(a.ndim, 1))(*(a.shape or (1,)))
    bd = (C.c_int64 * max(b.ndim, 1))(*(b.shape or (1,)))
    nd = max(a.ndim, b.ndim, 1)
    shape = np.broadcast_shapes(a.shape, b.shape)
    out = np.empty(shape, np.float32)
    od = (C.c_int64 * 16)()
    on = C.c_int()
    rc = lib().jxo_binary_broadcast(BINOPS[op], a, ad, max(a.ndim, 1), b, bd, max(b.ndim, 1), out, od, C.byref(on))
    if rc != 0:
        raise ValueError("shapes not broadcastable")
    assert on.value == nd or a.ndim == 0 or b.ndim == 0
    return out


def chain_fwd(x, a, b):
    x = _c(x)
    y = np.empty_like(x)
    lib().jxo_chain_fwd(x, y, x.size, a, b)
    return y


def chain_fwd_eager(x, a, b):
    x = _c(x)
    y = np.empty_like(x)
    lib().jxo_chain_fwd_eager(x, y, x.size, a, b)
    return y


def chain_vjp(x, a, b, ct=None):
    x = _c(x)
    y = np.empty_like(x)
    dx = np.empty_like(x)
    ctk = None if ct is None else _c(ct)
    lib().jxo_chain_vjp(x, None if ctk is None else ctk.ctypes.data, y.ctypes.data, dx, x.size, a, b)
    return y, dx


def chain_f64(x, a, b):
    x = _c(x)
    y = np.empty(x.shape, np.float64)
    dx = np.empty(x.shape, np.float64)
    lib().jxo_chain_f64(x, y.ctypes.data, dx.ctypes.data, x.size, a, b)
    return y, dx


RED = {"sum": 0, "max": 1, "min": 2, "prod": 3}


def reduce_all(x, op):
    x = _c(x).reshape(-1)
    return lib().jxo_reduce_all(x, x.size, RED[op])


def sum_all_f64(x):
    x = _c(x).reshape(-1)
    return lib().jxo_sum_all_f64(x, x.size)


def reduce_axis(x, axis, op, nthreads=1):
    x = _c(x)
    shape = x.shape
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    ln = shape[axis]
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    y = np.empty(shape[:axis] + shape[axis + 1:], np.float32)
    lib().jxo_reduce_axis(x, y.reshape(-1) if y.ndim else y.reshape(1), outer, ln, inner, RED[op], nthreads)
    return y


def sum_rows_f64(x):
    x = _c(x)
    r, c = x.shape
    y = np.empty(r, np.float64)
    lib().jxo_sum_rows_f64(x, y, r, c)
    return y


def arg_rows(x, is_max=True, nthreads=1):
    x = _c(x)
    r, c = x.shape
    idx = np.empty(r, np.int32)
    rc = lib().jxo_arg_rows(x, idx, r, c, 1 if is_max else 0, nthreads)
    if rc != 0:
        raise ValueError("NaN in arg reduction input")
    return idx


def sum_rows_vjp(ct, cols):
    ct = _c(ct)
    dx = np.empty((ct.size, cols), np.float32)
    lib().jxo_sum_rows_vjp(ct, dx, ct.size, cols)
    return dx


def max_rows_vjp(x, ct):
    x, ct = _c(x), _c(ct)
    dx = np.empty_like(x)
    lib().jxo_max_rows_vjp(x, ct, dx, x.shape[0], x.shape[1])
    return dx


def fft_c2c(x, inverse=False, nthreads=1):
    """x: float32 [..., n, 2] interleaved complex; transforms the last complex axis."""
    x = _c(x)
    n = x.shape[-2]
    batch = x.size // (2 * n)
    y = np.empty_like(x)
    if lib().jxo_fft_c2c(x, y, n, batch, 1 if inverse else 0, nthreads) != 0:
        raise ValueError("FFT size must be a power of 2")
    return y


def fft2_c2c(x, inverse=False, nthreads=1):
    """x: float32 [..., h, w, 2]."""
    x = _c(x)
    h, w = x.shape[-3], x.shape[-2]
    batch = x.size // (2 * h * w)
    y = np.empty_like(x)
    if lib().jxo_fft2_c2c(x, y, h, w, batch, 1 if inverse else 0, nthreads) != 0:
        raise ValueError("FFT size must be a power of 2")
    return y


def fft_real(x, full=True):
    """fft of real rows (src/ops/fft.rs:91-126; rfft :212-234 when not full):
    x float32 [..., n] -> [..., bins, 2], bins = n or n/2+1."""
    x = _c(x)
    n = x.shape[-1]
    batch = x.size // n
    bins = n if full else n // 2 + 1
    y = np.empty(x.shape[:-1] + (bins, 2), np.float32)
    if lib().jxo_fft_real(x, y, n, batch, 1 if full else 0) != 0:
        raise ValueError("FFT size must be a power of 2")
    return y


def irfft(x, n):
    """irfft (src/ops/fft.rs:417-462): x float32 [..., n/2+1, 2] -> [..., n]."""
    x = _c(x)
    batch = x.size // (2 * (n // 2 + 1))
    y = np.empty(x.shape[:-2] + (n,), np.float32)
    if lib().jxo_irfft(x, y, n, batch) != 0:
        raise ValueError("FFT size must be a power of 2")
    return y


def rfftn2(x):
    """rfftn of 2-D images (src/ops/fft.rs:474-553): [..., h, w] -> [..., h, w/2+1, 2]."""
    x = _c(x)
    h, w = x.shape[-2], x.shape[-1]
    batch = x.size // (h * w)
    y = np.empty(x.shape[:-1] + (w // 2 + 1, 2), np.float32)
    if lib().jxo_rfftn2(x, y, h, w, batch) != 0:
        raise ValueError("FFT size must be a power of 2")
    return y


def irfftn2(x, w):
    """irfftn of 2-D spectra (src/ops/fft.rs:554-628): [..., h, w/2+1, 2] -> [..., h, w]."""
    x = _c(x)
    h = x.shape[-3]
    batch = x.size // (2 * h * (w // 2 + 1))
    y = np.empty(x.shape[:-3] + (h, w), np.float32)
    if lib().jxo_irfftn2(x, y, h, w, batch) != 0:
        raise ValueError("FFT size must be a power of 2")
    return y


def dft_f64(x, inverse=False):
    x = _c(x)
    n = x.shape[-2]
    out = np.empty(x.shape, np.float64)
    lib().jxo_dft_f64(x, out, n, 1 if inverse else 0)
    return out


def _conv_dims(B, C_, H, W, O, KH, KW, stride, pad):
    return (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1


def conv2d_fwd(x, w, stride, pad, nthreads=1):
    x, w = _c(x), _c(w)
    B, Ci, H, W = x.shape
    O, _, KH, KW = w.shape
    OH, OW = _conv_dims(B, Ci, H, W, O, KH, KW, stride, pad)
    y = np.empty((B, O, OH, OW), np.float32)
    lib().jxo_conv2d_fwd(x, w, y, B, Ci, H, W, O, KH, KW, stride, pad, nthreads)
    return y


def conv2d_bwd_data(dy, w, x_shape, stride, pad, nthreads=1):
    dy, w = _c(dy), _c(w)
    B, Ci, H, W = x_shape
    O, _, KH, KW = w.shape
    dx = np.empty(x_shape, np.float32)
    lib().jxo_conv2d_bwd_data(dy, w, dx, B, Ci, H, W, O, KH, KW, stride, pad, nthreads)
    return dx


def conv2d_bwd_filter(x, dy, w_shape, stride, pad, nthreads=1):
    x, dy = _c(x), _c(dy)
    B, Ci, H, W = x.shape
    O, _, KH, KW = w_shape
    dw = np.empty(w_shape, np.float32)
    lib().jxo_conv2d_bwd_filter(x, dy, dw, B, Ci, H, W, O, KH, KW, stride, pad, nthreads)
    return dw


def softmax_rows(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().jxo_softmax_rows(x, y, x.shape[0], x.shape[1])
    return y


def log_softmax_rows(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().jxo_log_softmax_rows(x, y, x.shape[0], x.shape[1])
    return y


def one_hot(idx, classes):
    idx = _c(idx).reshape(-1)
    out = np.empty((idx.size, classes), np.float32)
    lib().jxo_one_hot(idx, out, idx.size, classes)
    return out


def cross_entropy(p, t):
    p, t = _c(p), _c(t)
    return lib().jxo_cross_entropy(p.reshape(-1), t.reshape(-1), p.size)


def adam_update(p, g, m, v, lr, b1, b2, eps, step, first):
    """In-place on copies; returns (p, m, v)."""
    p, g, m, v = _c(p).copy(), _c(g), _c(m).copy(), _c(v).copy()
    lib().jxo_adam_update(p, g, m, v, p.size, lr, b1, b2, eps, step, 1 if first else 0)
    return p, m, v


def dense_fwd(x, w, b, nthreads=1):
    x, w, b = _c(x), _c(w), _c(b)
    B, K = x.shape
    N = w.shape[1]
    y = np.empty((B, N), np.float32)
    lib().jxo_dense_fwd(x, w, b, y, B, K, N, nthreads)
    return y


def softmax_xent_bwd(p, t):
    p, t = _c(p), _c(t)
    dz = np.empty_like(p)
    lib().jxo_softmax_xent_bwd(p, t, dz, p.shape[0], p.shape[1])
    return dz


def col_sum(dy):
    dy = _c(dy)
    db = np.empty(dy.shape[1], np.float32)
    lib().jxo_col_sum(dy, db, dy.shape[0], dy.shape[1])
    return db


def transpose(x):
    x = _c(x)
    y = np.empty((x.shape[1], x.shape[0]), np.float32)
    lib().jxo_transpose(x, y, x.shape[0], x.shape[1])
    return y


# --------------------------------------------------------------------------
# Layers: conv1d, pooling, normalisation
# --------------------------------------------------------------------------
def conv1d(x, w, stride=1, pad=0, nthreads=1):
    """x [B, C, L], w [O, C, K] -> y [B, O, (L + 2 pad - K) // stride + 1] (conv1d shader order)."""
    x, w = _c(x), _c(w)
    B, Ci, L = x.shape
    O, _, K = w.shape
    OL = (L + 2 * pad - K) // stride + 1
    y = np.empty((B, O, OL), np.float32)
    if lib().jxo_conv1d(x, w, y, B, Ci, L, O, K, stride, pad, nthreads) != 0:
        raise ValueError("Kernel size must be <= input size")
    return y


def pool2d(x, kernel, stride=None, pad=(0, 0), is_max=True):
    """x [..., H, W] -> [..., OH, OW]; kernel, stride, pad are (h, w) pairs."""
    x = _c(x)
    H, W = x.shape[-2:]
    kh, kw = kernel
    sh, sw = stride if stride is not None else kernel
    ph, pw = pad
    OH, OW = (H + 2 * ph - kh) // sh + 1, (W + 2 * pw - kw) // sw + 1
    N = x.size // (H * W) if x.size else 0
    y = np.empty(x.shape[:-2] + (OH, OW), np.float32)
    if lib().jxo_pool2d(x, y, N, H, W, kh, kw, sh, sw, ph, pw, 1 if is_max else 0) != 0:
        raise ValueError("invalid pooling geometry")
    return y


def global_pool(x, is_max=False):
    """x [B, C, H, W] -> [B, C] (global_avg_pool2d / global_max_pool2d)."""
    x = _c(x)
    B, C_, H, W = x.shape
    y = np.empty((B, C_), np.float32)
    lib().jxo_global_pool(x, y, B * C_, H * W, 1 if is_max else 0)
    return y


def batchnorm(x, outer, channels, inner, eps, gamma=None, beta=None):
    """Normalise x viewed as [outer, channels, inner] per channel; returns (y, mean, var)."""
    x = _c(x)
    y = np.empty_like(x)
    mean = np.empty(channels, np.float32)
    var = np.empty(channels, np.float32)
    g = _c(gamma) if gamma is not None else None
    b = _c(beta) if beta is not None else None
    lib().jxo_batchnorm(x, g.ctypes.data if g is not None else None, b.ctypes.data if b is not None else None,
                        y, outer, channels, inner, eps, mean.ctypes.data, var.ctypes.data)
    return y, mean, var


def channel_stats_f64(x, outer, channels, inner):
    x = _c(x)
    m = np.empty(channels, np.float64)
    v = np.empty(channels, np.float64)
    lib().jxo_channel_stats_f64(x, outer, channels, inner, m, v)
    return m, v
