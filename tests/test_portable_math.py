"""The oracle's portable arithmetic (oracle/portable_math.c) against the reference's own
known answers: every assertion of crates/yskn-ref/src/portable_math.rs:440-588, bit
for bit. These functions are what the scalar reference calls for each exponential,
logarithm, inverse square root and rotary sine/cosine, so the layer and attention
oracles built on them reproduce yskn-ref's bits."""
import math

import numpy as np

import oracle as O


def f(bits):
    return float(np.array([bits], np.uint32).view(np.float32)[0])


def bits32(x):
    return int(np.array([x], np.float32).view(np.uint32)[0])


def bits64(x):
    return int(np.array([x], np.float64).view(np.uint64)[0])


def pm(name, x):
    return O.pm_scalar(name, x)


def test_exp2_pins_output_bits():
    # portable_math.rs:440-457
    for value, expected in [(1.0, 0x40000000), (-1.0, 0x3f000000), (0.5, 0x3fb504f3), (-30.0, 0x30800008),
                            (-126.0, 0x007fffe6), (-150.0, 0x00000001), (-1.44e30, 0x00000000),
                            (-math.inf, 0x00000000)]:
        assert bits32(pm("exp2", value)) == expected, value
    assert math.isnan(pm("exp2", math.nan))


def test_exp2_is_the_binary32_product_then_the_portable_exp():
    # portable_math.rs:459-467
    ln2 = np.float32(f(0x3f317218))
    for value in [0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 1.0e-7, -1.0e-7, 30.0, -30.0, -100.0]:
        arg = float(np.float32(value) * ln2)
        assert bits32(pm("exp2", value)) == bits32(pm("exp", arg)), value
    assert bits32(pm("exp2", 0.0)) == bits32(1.0)


def test_square_root_normal_subnormal_and_rounding_boundaries():
    # portable_math.rs:469-485
    for inp, expected in [(0x00000000, 0x00000000), (0x80000000, 0x80000000), (0x3f800000, 0x3f800000),
                          (0x40000000, 0x3fb504f3), (0x40800000, 0x40000000), (0x00000001, 0x1a3504f3),
                          (0x00800000, 0x20000000), (0x7f7fffff, 0x5f7fffff)]:
        assert bits32(pm("sqrt_rn", f(inp))) == expected, hex(inp)
    assert bits32(pm("rsqrt", 4.0)) == bits32(0.5)
    assert math.isnan(pm("sqrt_rn", -1.0))


def test_square_root_agrees_with_correctly_rounded_sqrt():
    # The bisection restatement against IEEE sqrt (also correctly rounded) on random bits.
    rng = np.random.default_rng(3)
    v = rng.integers(0, 0x7f800000, 20000, dtype=np.uint32).view(np.float32)
    got = O.pm("sqrt_rn", v)
    assert np.array_equal(got.view(np.uint32), np.sqrt(v).view(np.uint32))


def test_exact_identity_points():
    # portable_math.rs:487-501
    assert bits32(pm("exp", 0.0)) == bits32(1.0)
    assert bits32(pm("log", 1.0)) == bits32(0.0)
    assert bits32(pm("log1p", 0.0)) == bits32(0.0)
    assert bits32(pm("sigmoid", 0.0)) == bits32(0.5)
    assert bits32(pm("silu", 0.0)) == bits32(0.0)
    assert bits32(pm("softplus", 21.0)) == bits32(21.0)
    assert bits64(pm("exp_d", 0.0)) == bits64(1.0)
    assert bits64(pm("log_d", 1.0)) == bits64(0.0)
    c, s = O.pm_sincos(np.float32(0.0))
    assert bits32(c) == bits32(1.0) and bits32(s) == bits32(0.0)


def test_underflow_and_overflow_rules():
    # portable_math.rs:503-511
    assert bits32(pm("exp", -104.0)) == 0
    assert pm("exp", 89.0) == math.inf
    assert pm("exp", -103.0) > 0.0
    assert bits64(pm("exp_d", -746.0)) == 0
    assert pm("exp_d", 710.0) == math.inf
    import pytest
    with pytest.raises(O.OracleError):
        O.pm_sincos(np.float32(np.finfo(np.float32).max))


def test_polynomial_bit_patterns_match_the_portable_source():
    # portable_math.rs:513-580
    cases = [
        (0.5, [0x3fd3094c, 0xbf317218, 0x3ecf991f, 0x3f1f597f, 0x3e9f597f, 0x3f795d1c]),
        (1.0, [0x402df854, 0x00000000, 0x3f317218, 0x3f3b26a8, 0x3f3b26a8, 0x3fa818f5]),
        (10.0, [0x46ac14ee, 0x40135d8e, 0x4019771e, 0x3f7ffd06, 0x411ffe24, 0x41200030]),
    ]
    for x, expected in cases:
        got = [bits32(pm(n, x)) for n in ("exp", "log", "log1p", "sigmoid", "silu", "softplus")]
        assert got == expected, x
    assert bits32(pm("exp", -102.0)) == 4
    for x, e, lg in [(0.5, 0x3ffa61298e1e069c, 0xbfe62e42fefa39ef), (1.0, 0x4005bf0a8b14576a, 0),
                     (10.0, 0x40d5829dcf950560, 0x40026bb1bbb55516)]:
        assert bits64(pm("exp_d", x)) == e
        assert bits64(pm("log_d", x)) == lg
    for angle, cb, sb in [(1.0, 0x3f0a5140, 0x3f576aa4), (20.0, 0x3ed0f022, 0x3f69b6c8),
                          (1000000.0, 0x3f6fcefd, 0xbeb33259)]:
        c, s = O.pm_sincos(np.float32(angle))
        assert (bits32(c), bits32(s)) == (cb, sb), angle


def test_log_keeps_the_upstream_zero_endpoint_behaviour():
    # portable_math.rs:582-586
    assert bits64(pm("log_d", 0.0)) == 0xc0875427f6acad6f
    assert bits64(pm("log_d", -0.0)) == 0xc0a0ec2b7d284853


def test_array_map_equals_scalar_calls():
    rng = np.random.default_rng(5)
    x = rng.normal(0, 8, 4096).astype(np.float32)
    for name in ("exp", "exp2", "sigmoid", "silu"):
        got = O.pm(name, x)
        want = np.array([pm(name, float(v)) for v in x], np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name
    pos = np.abs(x)
    for name in ("log1p", "softplus", "rsqrt"):
        got = O.pm(name, pos)
        want = np.array([pm(name, float(v)) for v in pos], np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name
