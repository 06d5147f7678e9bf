"""C-ABI checks that need no GPU: the library loads, exports every function
include/jaxrs_cuda.h declares, and rejects bad arguments with JX_EINVAL before
touching the device (the reference panics on the same conditions)."""
import ctypes as C

import pytest


def test_library_exports_every_declared_symbol(jx):
    L = jx.lib()
    declared = jx.header_symbols()
    assert len(declared) >= 40
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing


def test_binding_covers_header(jx):
    assert set(jx.header_symbols()) <= set(jx._SIGS)


def test_gemm_rejects_bad_shapes(jx):
    with pytest.raises(jx.JaxRsError) as e:
        jx.gemm(0, 0, 0, -1, 2, 2)
    assert e.value.status == jx.JX_EINVAL
    with pytest.raises(jx.JaxRsError) as e:
        jx.gemm(1, 1, 1, 4, 4, 4, lda=2)
    assert "leading dimension" in e.value.message
    with pytest.raises(jx.JaxRsError):
        jx.gemm(1, 1, 1, 4, 4, 4, precision=7)


def test_gemm_empty_is_a_noop(jx):
    jx.gemm(0, 0, 0, 0, 5, 3)
    jx.gemm(0, 0, 0, 5, 0, 3)


def test_tape_validation(jx):
    U, B = jx.OP_UNARY, jx.OP_BINARY
    good = [(B + jx.BIN["mul"], 1, 0, 0), (jx.OP_STORE, 0, 1, 0)]
    t = jx.Tape(good, [], 1, 1)
    assert t.handle
    bad_cases = [
        ([(U + jx.UN["exp"], 1, 5, 0), (jx.OP_STORE, 0, 1, 0)], "undefined source"),
        ([(B + jx.BIN["add"], 1, 0, 0)], "output never stored"),
        ([(99, 1, 0, 0), (jx.OP_STORE, 0, 1, 0)], "unknown opcode"),
        ([(jx.OP_CONST, 1, 3, 0), (jx.OP_STORE, 0, 1, 0)], "constant index"),
        ([(U + jx.UN["exp"], 40, 0, 0), (jx.OP_STORE, 0, 40, 0)], "register range"),
    ]
    for code, why in bad_cases:
        with pytest.raises(jx.JaxRsError) as e:
            jx.Tape(code, [1.0], 1, 1)
        assert e.value.status == jx.JX_EINVAL, why
    with pytest.raises(jx.JaxRsError):
        jx.Tape(good * 100, [], 1, 1)  # longer than JX_TAPE_MAX_INSTR


def test_binary_broadcast_rejects_incompatible(jx):
    with pytest.raises(jx.JaxRsError) as e:
        jx.binary("add", 1, (2, 3), 1, (4,), 1)
    assert "broadcast" in e.value.message


def test_reduce_and_arg_argument_checks(jx):
    with pytest.raises(jx.JaxRsError):
        jx.call("jx_reduce_all_f32", 1, 1, 10, 9, None)
    with pytest.raises(jx.JaxRsError):
        jx.argreduce_rows(1, 1, None, 4, 0)


def test_last_error_is_thread_local(jx):
    import threading
    with pytest.raises(jx.JaxRsError):
        jx.gemm(0, 0, 0, -1, 1, 1)
    msg = jx.last_error()
    seen = []

    def other():
        seen.append(jx.last_error())

    th = threading.Thread(target=other)
    th.start()
    th.join()
    assert msg and seen == [""]


def _chain_code(jx):
    U, B = jx.OP_UNARY, jx.OP_BINARY
    return [(jx.OP_CONST, 1, 0, 0), (jx.OP_CONST, 2, 1, 0), (jx.OP_CONST, 3, 2, 0),
            (B + jx.BIN["mul"], 4, 0, 1), (B + jx.BIN["add"], 4, 4, 2), (U + jx.UN["gelu"], 4, 4, 0),
            (U + jx.UN["sigmoid"], 5, 0, 0), (B + jx.BIN["mul"], 4, 4, 5), (U + jx.UN["tanh"], 5, 0, 0),
            (B + jx.BIN["div"], 5, 5, 3), (B + jx.BIN["sub"], 4, 4, 5), (jx.OP_STORE, 0, 4, 0)]


def test_tape_kernel_compiles_without_gpu(jx):
    """The chain's generated kernel NVRTC-compiles for sm_100a (no GPU needed),
    and division by the constant 2 became a multiplication by 0.5."""
    t = jx.Tape(_chain_code(jx), [1.1, 0.9, 2.0], 1, 1)
    src = t.source()
    assert "jx_tape_kernel" in src and "jxm::unary_t<11>" in src
    assert "binary_t<3>" not in src  # no division left
    t.check()


def _folding_tape(jx):
    """y0 = x * -(1/3) (constant-only recip and neg: folded on the host);
    y1 = x + sqrt(-1) (NaN result: left on the device)."""
    U, B = jx.OP_UNARY, jx.OP_BINARY
    code = [(jx.OP_CONST, 1, 0, 0), (U + jx.UN["recip"], 2, 1, 0), (U + jx.UN["neg"], 3, 2, 0),
            (B + jx.BIN["mul"], 4, 0, 3), (jx.OP_CONST, 5, 1, 0), (U + jx.UN["sqrt"], 6, 5, 0),
            (B + jx.BIN["add"], 7, 0, 6), (jx.OP_STORE, 0, 4, 0), (jx.OP_STORE, 1, 7, 0)]
    return jx.Tape(code, [3.0, -1.0], 1, 2)


def test_constant_subexpressions_fold(jx):
    src = _folding_tape(jx).source()
    assert "unary_t<8>" not in src and "unary_t<0>" not in src  # recip and neg of constants folded
    assert "unary_t<7>" in src  # sqrt(-1) is NaN: stays on the device


def test_value_and_grad_shares_gelu_exponential(jx):
    """gelu and its derivative of one value come from one jxm::gelu_pair."""
    import importlib
    tr = importlib.import_module("jax-rs_b200.trace")
    prog = tr.value_and_grad(lambda x: tr.gelu(x * 1.1 + 0.9) * tr.sigmoid(x) - tr.tanh(x) / 2, 1)
    src = prog.tape_source(0)
    assert src.count("jxm::gelu_pair(") == 1 and src.count("jxm::sigmoid_tanh(") == 1
    assert "unary_t<11>" not in src and "unary_t<13>" not in src
    assert "unary_t<8>" not in src  # the constant reciprocal of the division's VJP is folded


def test_every_op_compiles(jx):
    """One tape touching every unary and binary op, in both operand orders."""
    code = [(jx.OP_CONST, 2, 0, 0)]
    r = 3
    for name, u in jx.UN.items():
        code.append((jx.OP_UNARY + u, r, 0, 0))
        r = 3 if r == 12 else r + 1
    for name, b in jx.BIN.items():
        code.append((jx.OP_BINARY + b, r, 0, 1))
        code.append((jx.OP_BINARY + b, r, 2, 0))
    code.append((jx.OP_SELECT_GT, 13, 0, 1))
    code.append((jx.OP_STORE, 0, 13, 0))
    code.append((jx.OP_STORE, 1, r, 0))
    t = jx.Tape(code, [0.5], 2, 2)
    t.check()


def test_layer_argument_checks(jx):
    """conv1d, pooling and normalisation reject bad geometry with the
    reference's assert messages, before touching any memory."""
    with pytest.raises(jx.JaxRsError, match="Kernel size must be <= input size"):
        jx.call("jx_conv1d_f32", 1, 1, 1, 1, 1, 1, 4, 5, 1, 0, None)
    with pytest.raises(jx.JaxRsError, match="Pool size must be positive"):
        jx.call("jx_pool2d_f32", 1, 1, 1, 1, 4, 4, 0, 2, 1, 1, 0, 0, jx.POOL_MAX, None)
    with pytest.raises(jx.JaxRsError, match="Stride must be positive"):
        jx.call("jx_maxpool2d_f32", 1, 1, 1, 1, 4, 4, 2, 2, 0, 0, None)
    with pytest.raises(jx.JaxRsError, match="larger than the padded input"):
        jx.call("jx_avgpool2d_f32", 1, 1, 1, 1, 2, 2, 3, 3, 1, 0, None)
    with pytest.raises(jx.JaxRsError, match="gamma and beta go together"):
        jx.call("jx_batchnorm_f32", 1, 1, None, 1, 2, 3, 4, 1e-5, None, None, None)
    with pytest.raises(jx.JaxRsError):
        jx.call("jx_global_pool2d_f32", 1, 1, 1, 1, 0, 1, 7, None)
    # empty batches are no-ops
    jx.call("jx_conv1d_f32", None, None, None, 0, 1, 4, 8, 3, 1, 0, None)
    jx.call("jx_pool2d_f32", None, None, 0, 3, 4, 4, 2, 2, 2, 2, 0, 0, jx.POOL_AVG, None)


def test_conv2d_argument_checks(jx):
    """conv2d rejects bad geometry with the reference's assert messages
    (src/nn.rs:2062-2067), and the kernel choice and the weight gradient's
    size limit are checked, all before any device work."""
    with pytest.raises(jx.JaxRsError, match="Kernel height too large"):
        jx.call("jx_conv2d_fwd_f32", 1, 1, 1, 1, 3, 4, 4, 8, 7, 7, 1, 0, None)
    with pytest.raises(jx.JaxRsError, match="Stride must be positive"):
        jx.call("jx_conv2d_bwd_data_f32", 1, 1, 1, 1, 3, 4, 4, 8, 3, 3, 0, 0, None)
    with pytest.raises(jx.JaxRsError, match="2\\^31"):
        jx.call("jx_conv2d_bwd_filter_f32", 1, 1, 1, 1 << 20, 1, 64, 64, 1, 1, 1, 1, 0, None)
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_conv_set_kernel", 3)
    assert e.value.status == jx.JX_EINVAL
    for which in (jx.CONV_ONE_CTA, jx.CONV_PAIR, jx.CONV_AUTO):
        jx.call("jx_conv_set_kernel", which)
    # empty batches are no-ops
    jx.call("jx_conv2d_fwd_f32", None, None, None, 0, 3, 8, 8, 4, 3, 3, 1, 1, None)


def test_rust_ffi_block_matches_header():
    """INTEGRATION.md's Rust extern block is the generator's output for the
    current header, and it declares every JX_API function exactly once."""
    import importlib.util
    import os
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("rust_ffi", os.path.join(root, "jax-rs_b200", "rust_ffi.py"))
    rf = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rf)
    block = rf.rust_block()
    with open(os.path.join(root, "INTEGRATION.md")) as f:
        doc = f.read()
    m = re.search(r"<!-- rust-ffi:begin -->\n```rust\n(.*?)```\n<!-- rust-ffi:end -->", doc, flags=re.S)
    assert m, "INTEGRATION.md lacks the generated Rust block"
    assert m.group(1) == block, "regenerate with: python jax-rs_b200/rust_ffi.py"
    with open(os.path.join(root, "include", "jaxrs_cuda.h")) as f:
        header_names = set(re.findall(r"JX_API[^;(]*\b(jx_\w+)\s*\(", f.read()))
    rust_names = re.findall(r"pub fn (jx_\w+)\(", block)
    assert len(rust_names) == len(set(rust_names)) and set(rust_names) == header_names
