"""jax-rs B200 backend: Python binding of the C ABI (include/jaxrs_cuda.h).

The compute lives in ``libjaxrs_cuda.so`` (hand-written sm_100a CUDA, built by
``build.py``).  This module only loads it with ctypes and turns status codes
into exceptions; there is no Python or CPU fallback.  If the library is
missing, every call raises.

Import it with ``importlib.import_module("jax-rs_b200")`` (the directory name
has a hyphen).
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjaxrs_cuda.so")

# status codes (include/jaxrs_cuda.h)
JX_OK, JX_EINVAL, JX_ENOMEM, JX_ECUDA, JX_ENCCL, JX_ETIMEOUT, JX_EUNSUPPORTED, JX_EDEVICE, JX_EINTERNAL = range(9)
STATUS_NAMES = {0: "JX_OK", 1: "JX_EINVAL", 2: "JX_ENOMEM", 3: "JX_ECUDA", 4: "JX_ENCCL", 5: "JX_ETIMEOUT",
                6: "JX_EUNSUPPORTED", 7: "JX_EDEVICE", 8: "JX_EINTERNAL"}
PREC_3XTF32, PREC_EXACT, PREC_3XTF32_FUSED, PREC_3XTF32_PAIR = 0, 1, 2, 3
CONV_AUTO, CONV_ONE_CTA, CONV_PAIR = 0, 1, 2  # jx_conv_set_kernel
POOL_MAX, POOL_AVG = 0, 1
BIN = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "min": 5, "max": 6}
UN = {"neg": 0, "abs": 1, "sin": 2, "cos": 3, "tanh": 4, "exp": 5, "log": 6, "sqrt": 7, "recip": 8,
      "square": 9, "relu": 10, "gelu": 11, "sigmoid": 12, "gelu_grad": 13, "tan": 14, "sign": 15, "sinh": 16,
      "cosh": 17, "asin": 18, "acos": 19, "atan": 20, "asinh": 21, "acosh": 22, "atanh": 23, "ceil": 24,
      "floor": 25, "round": 26, "trunc": 27, "expm1": 28, "log1p": 29, "cbrt": 30, "log2": 31}
RED = {"sum": 0, "max": 1, "min": 2, "prod": 3}
OP_CONST, OP_STORE, OP_UNARY, OP_BINARY, OP_SELECT_GT = 1, 2, 16, 48, 64
DEVERR_NAN, DEVERR_TIMEOUT = 1, 2


class JaxRsError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


_lib = None
vp = C.c_void_p
i64 = C.c_int64
ci = C.c_int
cf = C.c_float

# name -> argtypes (all return int status unless listed in _RESTYPE)
_SIGS = {
    "jx_last_error": [],
    "jx_version": [],
    "jx_init": [ci],
    "jx_device_count": [C.POINTER(ci)],
    "jx_set_device": [ci],
    "jx_get_device": [C.POINTER(ci)],
    "jx_device_status": [C.POINTER(C.c_uint)],
    "jx_malloc": [C.POINTER(vp), C.c_size_t, ci, vp],
    "jx_free": [vp, vp],
    "jx_check_guards": [C.POINTER(ci)],
    "jx_selftest_fail_alloc": [ci],
    "jx_memcpy_h2d": [vp, vp, C.c_size_t, vp],
    "jx_memcpy_d2h": [vp, vp, C.c_size_t, vp],
    "jx_memcpy_d2d": [vp, vp, C.c_size_t, vp],
    "jx_stream_create": [C.POINTER(vp)],
    "jx_stream_destroy": [vp],
    "jx_stream_sync": [vp],
    "jx_host_register": [vp, C.c_size_t],
    "jx_host_unregister": [vp],
    "jx_conv1d_f32": [vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, vp],
    "jx_pool2d_f32": [vp, vp] + [i64] * 10 + [ci, vp],
    "jx_pool2d_f32_host": [vp, vp] + [i64] * 10 + [ci, i64, vp],
    "jx_gemm_batched_f32_host": [vp, vp, vp, i64, i64, i64, i64, i64, vp],
    "jx_maxpool2d_f32": [vp, vp] + [i64] * 8 + [vp],
    "jx_avgpool2d_f32": [vp, vp] + [i64] * 8 + [vp],
    "jx_global_pool2d_f32": [vp, vp, i64, i64, i64, i64, ci, vp],
    "jx_batchnorm_f32": [vp, vp, vp, vp, i64, i64, i64, cf, vp, vp, vp],
    "jx_gemm_f32": [vp, vp, vp, i64, i64, i64, ci, ci, i64, i64, i64, i64, i64, i64, i64, ci, vp],
    "jx_gemm_workspace_size": [i64, i64, i64, i64, C.POINTER(C.c_size_t)],
    "jx_gemm_kpad": [i64, C.POINTER(i64)],
    "jx_gemm_f32_noalloc": [vp, vp, vp, i64, i64, i64, ci, ci, i64, i64, i64, i64, i64, i64, i64, vp],
    "jx_gemm_split_f32": [vp, vp, vp, i64, i64, i64, ci, i64, i64, vp],
    "jx_gemm_presplit_f32": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, vp],
    "jx_binary_f32": [ci, vp, C.POINTER(i64), ci, vp, C.POINTER(i64), ci, vp, vp],
    "jx_unary_f32": [ci, vp, vp, i64, vp],
    "jx_tape_create": [C.POINTER(C.c_int32), ci, C.POINTER(cf), ci, ci, ci, C.POINTER(vp)],
    "jx_tape_destroy": [vp],
    "jx_tape_compile": [vp],
    "jx_tape_source": [vp, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)],
    "jx_tape_check": [vp],
    "jx_tape_run": [vp, C.POINTER(vp), C.POINTER(vp), i64, vp],
    "jx_tape_info": [vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "jx_tape_run_host": [vp, C.POINTER(vp), C.POINTER(vp), i64, i64, vp],
    "jx_gemm_f32_host": [vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, vp],
    "jx_fft_r2c_f32": [vp, vp, i64, i64, C.c_int, vp],
    "jx_fft_c2c_f32_host": [vp, vp, i64, i64, C.c_int, i64, vp],
    "jx_fft2_c2c_f32_host": [vp, vp, i64, i64, i64, C.c_int, i64, vp],
    "jx_fft_c2r_f32": [vp, vp, i64, i64, vp],
    "jx_rfft2_f32": [vp, vp, i64, i64, i64, vp],
    "jx_irfft2_f32": [vp, vp, i64, i64, i64, vp],
    "jx_random_uniform_f32": [C.c_uint64, C.c_uint64, vp, i64, cf, cf, vp],
    "jx_random_randint_f32": [C.c_uint64, C.c_uint64, vp, i64, C.c_int32, C.c_int32, vp],
    "jx_random_normal_f32": [C.c_uint64, C.c_uint64, vp, i64, vp],
    "jx_random_jump": [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.c_uint64],
    "jx_random_key_from_seed": [C.c_uint64, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)],
    "jx_random_key_split": [C.c_uint64, C.c_uint64] + [C.POINTER(C.c_uint64)] * 4,
    "jx_graph_create": [C.POINTER(vp)],
    "jx_graph_destroy": [vp],
    "jx_graph_input": [vp, C.POINTER(C.c_int)],
    "jx_graph_const": [vp, cf, C.POINTER(C.c_int)],
    "jx_graph_unary": [vp, C.c_int, C.c_int, C.POINTER(C.c_int)],
    "jx_graph_binary": [vp, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)],
    "jx_graph_select_gt": [vp, C.c_int, C.c_int, C.POINTER(C.c_int)],
    "jx_graph_size": [vp, C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "jx_graph_vjp": [vp, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int, C.POINTER(C.c_int),
                     C.POINTER(C.c_int)],
    "jx_graph_compile": [vp, C.c_int, C.POINTER(C.c_int), C.POINTER(vp)],
    "jx_program_info": [vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "jx_program_tape": [vp, C.c_int, C.POINTER(vp)],
    "jx_program_run": [vp, C.POINTER(vp), C.POINTER(vp), i64, vp],
    "jx_program_destroy": [vp],
    "jx_reduce_all_f32": [vp, vp, i64, ci, vp],
    "jx_reduce_axis_f32": [vp, vp, i64, i64, i64, ci, vp],
    "jx_argreduce_rows_f32": [vp, vp, vp, i64, i64, ci, vp],
    "jx_sum_rows_vjp_f32": [vp, vp, i64, i64, vp],
    "jx_max_rows_vjp_f32": [vp, vp, vp, i64, i64, vp],
    "jx_fft_c2c_f32": [vp, vp, i64, i64, ci, vp],
    "jx_fft2_c2c_f32": [vp, vp, i64, i64, i64, ci, vp],
    "jx_conv_set_kernel": [ci],
    "jx_conv2d_fwd_f32": [vp, vp, vp] + [i64] * 9 + [vp],
    "jx_conv2d_bwd_data_f32": [vp, vp, vp] + [i64] * 9 + [vp],
    "jx_conv2d_bwd_filter_f32": [vp, vp, vp] + [i64] * 9 + [vp],
    "jx_softmax_rows_f32": [vp, vp, i64, i64, vp],
    "jx_softmax_xent_f32": [vp, vp, vp, vp, vp, i64, i64, i64, vp],
    "jx_bias_act_f32": [vp, vp, vp, i64, i64, ci, vp],
    "jx_act_bwd_f32": [vp, vp, vp, vp, i64, i64, ci, vp],
    "jx_col_sum_f32": [vp, vp, i64, i64, vp],
    "jx_adam_step_f32": [C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(i64), ci,
                         cf, cf, cf, cf, i64, vp],
    "jx_mlp_create": [C.POINTER(i64), ci, C.POINTER(ci), i64, ci, C.POINTER(vp)],
    "jx_mlp_param_count": [vp, C.POINTER(i64)],
    "jx_mlp_param_offsets": [vp, C.POINTER(i64), C.POINTER(i64)],
    "jx_mlp_set_params": [vp, vp, i64],
    "jx_mlp_get_params": [vp, vp, i64],
    "jx_mlp_set_adam": [vp, cf, cf, cf, cf],
    "jx_mlp_attach_comm": [vp, vp, ci, i64],
    "jx_mlp_train_step": [vp, vp, vp, vp, vp],
    "jx_mlp_set_fused": [vp, ci],
    "jx_mlp_set_timing": [vp, ci],
    "jx_mlp_set_dp_sharded": [vp, ci],
    "jx_mlp_step_times": [vp, C.POINTER(cf)],
    "jx_selftest_barrier_timeout": [ci, C.POINTER(ci)],
    "jx_selftest_noalloc_flag": [C.c_uint],
    "jx_mlp_destroy": [vp],
    "jx_nccl_unique_id_size": [],
    "jx_nccl_get_unique_id": [vp],
    "jx_nccl_init": [vp, ci, ci, ci, C.POINTER(vp)],
    "jx_nccl_allreduce_sum_f32": [vp, vp, i64, vp],
    "jx_nccl_wait": [vp, vp, ci],
    "jx_nccl_destroy": [vp],
}
_RESTYPE = {"jx_last_error": C.c_char_p}


def header_symbols():
    """Names of every function include/jaxrs_cuda.h declares (parsed from the header)."""
    import re
    hdr = os.path.join(HERE, "..", "include", "jaxrs_cuda.h")
    with open(hdr) as f:
        txt = f.read()
    return sorted(set(re.findall(r"^JX_API\s+[\w\s\*]+?\b(jx_\w+)\s*\(", txt, flags=re.M)))


def lib():
    """Load libjaxrs_cuda.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise JaxRsError(JX_EUNSUPPORTED, f"{LIB_PATH} is missing: build it with jax-rs_b200/build.py "
                                              "(there is no fallback implementation)")
        L = C.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, C.c_int)
        _lib = L
    return _lib


def last_error() -> str:
    return lib().jx_last_error().decode(errors="replace")


def check(status: int, what: str = ""):
    if status != JX_OK:
        raise JaxRsError(status, f"{what}: {last_error()}" if what else last_error())
    return status


def call(name, *args):
    return check(getattr(lib(), name)(*args), name)


def init(device: int = 0):
    call("jx_init", device)


def device_status() -> int:
    flags = C.c_uint(0)
    call("jx_device_status", C.byref(flags))
    return flags.value


# --------------------------------------------------------------------------
# raw-pointer wrappers (device pointers as ints; streams as ints or None)
# --------------------------------------------------------------------------
def gemm(A, B, Cp, M, N, K, transA=False, transB=False, lda=None, ldb=None, ldc=None, batch=1,
         strideA=0, strideB=0, strideC=0, precision=PREC_3XTF32, stream=None):
    lda = lda if lda is not None else (M if transA else K)
    ldb = ldb if ldb is not None else (K if transB else N)
    ldc = ldc if ldc is not None else N
    call("jx_gemm_f32", A, B, Cp, M, N, K, int(transA), int(transB), lda, ldb, ldc, batch, strideA, strideB,
         strideC, precision, stream)


def gemm_kpad(K):
    kp = i64(0)
    call("jx_gemm_kpad", K, C.byref(kp))
    return kp.value


def gemm_split(src, hi, lo, rows, K, ld=None, trans=False, batch=1, stride=0, stream=None):
    ld = ld if ld is not None else (rows if trans else K)
    call("jx_gemm_split_f32", src, hi, lo, rows, K, ld, int(trans), batch, stride, stream)


def gemm_presplit(Ah, Al, Bh, Bl, Cp, M, N, Kp, ldc=None, batch=1, strideC=0, stream=None):
    call("jx_gemm_presplit_f32", Ah, Al, Bh, Bl, Cp, M, N, Kp, ldc if ldc is not None else N, batch, strideC,
         stream)


def _shape(shape):
    arr = (i64 * max(len(shape), 1))(*shape)
    return arr, len(shape)


def binary(op, a, a_shape, b, b_shape, out, stream=None):
    sa, na = _shape(a_shape)
    sb, nb = _shape(b_shape)
    call("jx_binary_f32", BIN[op], a, sa, na, b, sb, nb, out, stream)


def unary(op, x, y, n, stream=None):
    call("jx_unary_f32", UN[op], x, y, n, stream)


class Tape:
    """A validated op-tape (FusedGroup replacement) living in host memory until launch."""

    def __init__(self, code, consts, n_inputs, n_outputs):
        flat = [int(v) for ins in code for v in ins]
        carr = (C.c_int32 * max(len(flat), 1))(*flat)
        karr = (cf * max(len(consts), 1))(*consts)
        h = vp()
        call("jx_tape_create", carr, len(code), karr, len(consts), n_inputs, n_outputs, C.byref(h))
        self.handle = h
        self.n_inputs, self.n_outputs = n_inputs, n_outputs

    def source(self) -> str:
        need = C.c_size_t(0)
        call("jx_tape_source", self.handle, None, 0, C.byref(need))
        buf = C.create_string_buffer(need.value)
        call("jx_tape_source", self.handle, buf, need.value, C.byref(need))
        return buf.value.decode()

    def check(self):
        """NVRTC-compiles the tape's kernel without a GPU (raises on failure)."""
        call("jx_tape_check", self.handle)

    def run(self, ins, outs, n, stream=None):
        ia = (vp * max(len(ins), 1))(*ins)
        oa = (vp * max(len(outs), 1))(*outs)
        call("jx_tape_run", self.handle, ia, oa, n, stream)

    def __del__(self):
        try:
            if self.handle and _lib is not None:
                _lib.jx_tape_destroy(self.handle)
        except Exception:
            pass


def reduce_all(x, out, n, op, stream=None):
    call("jx_reduce_all_f32", x, out, n, RED[op], stream)


def reduce_axis(x, out, outer, length, inner, op, stream=None):
    call("jx_reduce_axis_f32", x, out, outer, length, inner, RED[op], stream)


def argreduce_rows(x, idx, val, rows, cols, is_max=True, stream=None):
    call("jx_argreduce_rows_f32", x, idx, val, rows, cols, int(is_max), stream)


def sum_rows_vjp(ct, dx, rows, cols, stream=None):
    call("jx_sum_rows_vjp_f32", ct, dx, rows, cols, stream)


def max_rows_vjp(x, ct, dx, rows, cols, stream=None):
    call("jx_max_rows_vjp_f32", x, ct, dx, rows, cols, stream)


def fft_c2c(x, y, n, batch, inverse=False, stream=None):
    call("jx_fft_c2c_f32", x, y, n, batch, int(inverse), stream)


def fft2_c2c(x, y, h, w, batch, inverse=False, stream=None):
    call("jx_fft2_c2c_f32", x, y, h, w, batch, int(inverse), stream)


class MLP:
    """Native Dense-stack trainer (jx_mlp_*): widths [d0, d1, ..., dL], hidden
    activations ('relu' | 'gelu' | 'none'), softmax cross-entropy, Adam."""

    ACTS = {"none": 0, "relu": 1, "gelu": 2}

    def __init__(self, widths, acts, batch, precision=PREC_3XTF32):
        w = (i64 * len(widths))(*widths)
        a = (ci * max(len(acts), 1))(*[self.ACTS[x] for x in acts] or [0])
        h = vp()
        call("jx_mlp_create", w, len(widths) - 1, a, batch, precision, C.byref(h))
        self.handle = h
        self.widths = list(widths)
        self.batch = batch
        n = i64(0)
        call("jx_mlp_param_count", h, C.byref(n))
        self.nparams = n.value
        L = len(widths) - 1
        wo, bo = (i64 * L)(), (i64 * L)()
        call("jx_mlp_param_offsets", h, wo, bo)
        self.w_off, self.b_off = list(wo), list(bo)

    def pack(self, weights, biases):
        """Flat parameter vector from per-layer W [in, out] and b [out] (numpy)."""
        import numpy as np
        flat = np.zeros(self.nparams, np.float32)
        for l, (W, b) in enumerate(zip(weights, biases)):
            flat[self.w_off[l]:self.w_off[l] + W.size] = np.asarray(W, np.float32).ravel()
            flat[self.b_off[l]:self.b_off[l] + b.size] = np.asarray(b, np.float32).ravel()
        return flat

    def unpack(self, flat):
        Ws, bs = [], []
        for l in range(len(self.widths) - 1):
            i, o = self.widths[l], self.widths[l + 1]
            Ws.append(flat[self.w_off[l]:self.w_off[l] + i * o].reshape(i, o))
            bs.append(flat[self.b_off[l]:self.b_off[l] + o])
        return Ws, bs

    def set_params(self, flat):
        import numpy as np
        flat = np.ascontiguousarray(flat, np.float32)
        call("jx_mlp_set_params", self.handle, flat.ctypes.data, flat.size)

    def get_params(self):
        import numpy as np
        out = np.empty(self.nparams, np.float32)
        call("jx_mlp_get_params", self.handle, out.ctypes.data, out.size)
        return out

    def set_adam(self, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8):
        call("jx_mlp_set_adam", self.handle, lr, b1, b2, eps)

    def attach_comm(self, comm, world, global_batch):
        call("jx_mlp_attach_comm", self.handle, comm, world, global_batch)

    def step(self, x, labels, loss_out=None, stream=None):
        call("jx_mlp_train_step", self.handle, x, labels, loss_out, stream)

    def set_timing(self, enable=True):
        call("jx_mlp_set_timing", self.handle, 1 if enable else 0)

    def step_times(self):
        """(forward, backward, tail) milliseconds of the last timed step."""
        ms = (cf * 3)()
        call("jx_mlp_step_times", self.handle, ms)
        return tuple(ms)

    def __del__(self):
        try:
            if self.handle and _lib is not None:
                _lib.jx_mlp_destroy(self.handle)
        except Exception:
            pass


def key_from_seed(seed):
    """PRNGKey::from_seed (src/random.rs:29-32) -> (s0, s1)."""
    a, b = C.c_uint64(), C.c_uint64()
    call("jx_random_key_from_seed", seed, C.byref(a), C.byref(b))
    return a.value, b.value


def key_split(key):
    """PRNGKey::split (src/random.rs:35-48) -> ((s0, s1), (s0, s1))."""
    v = [C.c_uint64() for _ in range(4)]
    call("jx_random_key_split", key[0], key[1], *[C.byref(x) for x in v])
    return (v[0].value, v[1].value), (v[2].value, v[3].value)
