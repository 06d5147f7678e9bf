"""Host jump-ahead of the PRNGKey stream (no GPU): jx_random_jump(k, j)
equals j plain next_u64 steps of the oracle's restated generator
(src/random.rs:78-90)."""
import ctypes as C
import importlib

import pytest


@pytest.mark.parametrize("steps", [0, 1, 2, 63, 64, 65, 1000, 123457, 1 << 20])
def test_jump_equals_stepping(oracle, steps):
    jx = importlib.import_module("jax-rs_b200")
    key = oracle.key_from_seed(42).split()[1]
    a, b = C.c_uint64(key.s0), C.c_uint64(key.s1)
    jx.call("jx_random_jump", C.byref(a), C.byref(b), steps)
    k = oracle.Key(key.s0, key.s1)
    for _ in range(steps):
        oracle.next_u64(k)
    assert (a.value, b.value) == (k.s0, k.s1)


@pytest.mark.parametrize("seed", [0, 1, 42, 2 ** 63 + 5])
def test_key_from_seed_and_split_match_the_oracle(oracle, seed):
    jx = importlib.import_module("jax-rs_b200")
    k = jx.key_from_seed(seed)
    ko = oracle.key_from_seed(seed)
    assert k == (ko.s0, ko.s1)
    a, b = jx.key_split(k)
    ao, bo = ko.split()
    assert a == (ao.s0, ao.s1) and b == (bo.s0, bo.s1)
