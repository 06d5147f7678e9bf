"""Device PRNG streams against the oracle's restatement of the reference's
host loops (src/random.rs:161-285): uniform_range and randint bit-identical,
normal (Box-Muller with CUDA's logf/cosf/sinf) within |d - o| <= 2e-6 |o| + 5e-7."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# around a thread's 2048-value range, a warp's 65536 and a block's 524288
SIZES = [1, 2, 31, 32, 1000, 2047, 2048, 2049, 65535, 65536, 65537, 262143, 262144, 262145, 524287, 524289,
         1 << 20, 3_000_001]


def _key(oracle, seed):
    return oracle.key_from_seed(seed).split()[0]


def _gen(jx, dev, name, key, n, *args):
    Y = dev.full((n,), np.nan)
    jx.call(name, key.s0, key.s1, Y.data_ptr(), n, *args, dev.stream)
    return dev.get(Y)


@pytest.mark.parametrize("n", SIZES)
def test_uniform_range_bit_identical(jx, dev, oracle, n):
    k = _key(oracle, 3)
    y = _gen(jx, dev, "jx_random_uniform_f32", k, n, -1.0, 1.0)
    assert np.array_equal(y, oracle.uniform_range(k, n, -1.0, 1.0))


@pytest.mark.parametrize("lo,hi", [(0, 10), (-5, 5), (0, 1000), (-2147483, 2147483)])
def test_randint_bit_identical(jx, dev, oracle, lo, hi):
    k = _key(oracle, 4)
    n = 100003
    y = _gen(jx, dev, "jx_random_randint_f32", k, n, lo, hi)
    assert np.array_equal(y, oracle.randint(k, n, lo, hi))


@pytest.mark.parametrize("n", [1, 2, 3, 1001, 262145, 1 << 20])
def test_normal_matches_box_muller(jx, dev, oracle, n):
    k = _key(oracle, 5)
    y = _gen(jx, dev, "jx_random_normal_f32", k, n).astype(np.float64)
    o = oracle.normal(k, n).astype(np.float64)
    assert np.all(np.abs(y - o) <= 2e-6 * np.abs(o) + 5e-7)


def test_full_size_uniform_stream(jx, dev, oracle):
    """2^26 draws (256 blocks of jumps): every value equals the host stream."""
    k = _key(oracle, 6)
    n = 1 << 26
    y = _gen(jx, dev, "jx_random_uniform_f32", k, n, 0.5, 1.5)
    assert np.array_equal(y, oracle.uniform_range(k, n, 0.5, 1.5))


def test_zero_size_and_bad_range(jx, dev, oracle):
    k = _key(oracle, 7)
    jx.call("jx_random_uniform_f32", k.s0, k.s1, None, 0, 0.0, 1.0, dev.stream)
    with pytest.raises(jx.JaxRsError) as e:
        jx.call("jx_random_randint_f32", k.s0, k.s1, None, 10, 5, 5, dev.stream)
    assert "minval must be less than maxval" in e.value.message


@pytest.mark.parametrize("n", [5000, 262145])
def test_unaligned_output_stream(jx, dev, oracle, n):
    """An output that is not 16-byte aligned gives the same stream."""
    k = _key(oracle, 9)
    Y = dev.full((n + 1,), np.nan)
    jx.call("jx_random_uniform_f32", k.s0, k.s1, Y.data_ptr() + 4, n, -2.0, 3.0, dev.stream)
    y = dev.get(Y)
    assert np.isnan(y[0])
    assert np.array_equal(y[1:], oracle.uniform_range(k, n, -2.0, 3.0))
    jx.call("jx_random_normal_f32", k.s0, k.s1, Y.data_ptr() + 4, n, dev.stream)
    z = dev.get(Y)[1:]
    ref = oracle.normal(k, n)
    assert np.all(np.abs(z - ref) <= 2e-6 * np.abs(ref) + 5e-7)
