"""Runtime checks that need a device but fault nothing.

* JAXRS_CHECK=1: jx_malloc puts canary bytes after each buffer; a write past
  the end (into the guard, which is allocated memory, so the write itself is
  harmless) is reported by jx_check_guards and by jx_free as JX_EDEVICE.
* Allocation-failure injection on the host: an entry point whose scratch
  allocation fails returns JX_ENOMEM, and the next call works.
* jx_init(-1) takes the default device from JAXRS_DEVICE.
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import normwise_rel

pytestmark = pytest.mark.gpu


def test_check_mode_catches_a_write_past_the_end(jx, dev):
    os.environ["JAXRS_CHECK"] = "1"
    try:
        p = C.c_void_p()
        src = np.ones(256, np.float32)
        jx.call("jx_malloc", C.byref(p), 1000, 1, None)
        jx.call("jx_memcpy_h2d", p, src.ctypes.data, 1000, None)  # in bounds
        bad = C.c_int(-1)
        jx.call("jx_check_guards", C.byref(bad))
        assert bad.value == 0
        jx.call("jx_memcpy_h2d", p, src.ctypes.data, 1008, None)  # 8 bytes past the end
        jx.call("jx_check_guards", C.byref(bad))
        assert bad.value == 1
        with pytest.raises(jx.JaxRsError) as e:
            jx.call("jx_free", p, None)
        assert e.value.status == jx.JX_EDEVICE
        assert "past the end" in e.value.message
        # an intact buffer frees cleanly, and the freed one is no longer tracked
        jx.call("jx_malloc", C.byref(p), 1000, 0, None)
        jx.call("jx_memcpy_h2d", p, src.ctypes.data, 1000, None)
        jx.call("jx_free", p, None)
        jx.call("jx_check_guards", C.byref(bad))
        assert bad.value == 0
    finally:
        del os.environ["JAXRS_CHECK"]


def test_injected_allocation_failure_is_reported_and_recovers(jx, dev):
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (96, 80)).astype(np.float32)
    b = rng.uniform(-1, 1, (80, 72)).astype(np.float32)
    A, B = dev.put(a), dev.put(b)
    Cm = dev.full((96, 72), np.nan)
    jx.call("jx_selftest_fail_alloc", 1)
    try:
        with pytest.raises(jx.JaxRsError) as e:
            jx.gemm(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), 96, 72, 80, stream=dev.stream)
        assert e.value.status == jx.JX_ENOMEM
        assert "injected" in e.value.message
    finally:
        jx.call("jx_selftest_fail_alloc", 0)
    jx.gemm(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), 96, 72, 80, stream=dev.stream)
    assert normwise_rel(dev.get(Cm), a.astype(np.float64) @ b) <= 1e-5
    # jx_malloc fails the same way
    jx.call("jx_selftest_fail_alloc", 1)
    p = C.c_void_p()
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_malloc", C.byref(p), 64, 0, None)
    assert e.value.status == jx.JX_ENOMEM and not p.value
    jx.call("jx_malloc", C.byref(p), 64, 0, None)
    jx.call("jx_free", p, None)


def test_default_device_from_environment(jx, dev):
    os.environ["JAXRS_DEVICE"] = "0"
    try:
        jx.call("jx_init", -1)
        d = C.c_int(-1)
        jx.call("jx_get_device", C.byref(d))
        assert d.value == 0
    finally:
        del os.environ["JAXRS_DEVICE"]
