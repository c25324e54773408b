"""The activation quantiser's division shortcut (quant.cuh quotient_rne), restated in
numpy binary32 arithmetic and checked against the exact rule it replaces:
q = rne(fl(v / alpha)) (crates/yskn-ref/src/compressed_linear.rs:57-112), including
values placed on and around every half-integer quotient, where the shortcut must hand
over to the exact division."""
import numpy as np

F = np.float32
MAGIC = F(12582912.0)  # 1.5 * 2^23
LIMIT = F(0.49993896484375)  # 0.5 - 2^-14


def exact(v, scale):
    return np.rint(v / scale).astype(np.int64)  # binary32 division, then ties to even


def shortcut(v, scale):
    rcp = F(1.0) / scale
    y = v * rcp
    t = y + MAGIC
    d = y - (t - MAGIC)
    fast = np.abs(d) < LIMIT
    n_fast = t.view(np.uint32).astype(np.int64) - 0x4B400000
    return np.where(fast, n_fast, exact(v, scale)), fast


def _scales(rng, n):
    # alpha = max|v| / 127 for half-precision maxima across the whole half range
    mx = rng.uniform(-14, 15.9, n).astype(np.float32)
    mx = np.exp2(mx).astype(np.float16).astype(np.float32)
    return (mx / F(127.0)).astype(np.float32), mx


def test_random_values_match_exact_division():
    rng = np.random.default_rng(7)
    scale, mx = _scales(rng, 4096)
    v = (rng.uniform(-1, 1, (4096, 512)).astype(np.float32) * mx[:, None]).astype(np.float16).astype(np.float32)
    got, fast = shortcut(v, scale[:, None])
    assert np.array_equal(got, exact(v, scale[:, None]))
    assert fast.mean() > 0.999


def test_near_half_integer_quotients_match_exact_division():
    rng = np.random.default_rng(11)
    scale, _ = _scales(rng, 2048)
    k = rng.integers(-127, 127, 2048).astype(np.float32)
    base = ((k + F(0.5)) * scale).astype(np.float32)
    cases = [base]
    up, down = base.copy(), base.copy()
    for _ in range(6):  # a few ulps either side of the tie
        up = np.nextafter(up, F(np.inf))
        down = np.nextafter(down, F(-np.inf))
        cases += [up.copy(), down.copy()]
    v = np.stack(cases, 1)
    got, fast = shortcut(v, scale[:, None])
    assert np.array_equal(got, exact(v, scale[:, None]))
    assert (~fast).any()  # the exact path is exercised


def test_quotients_at_the_row_maximum():
    # v = +-max gives quotients at +-127 (within rounding of the scale)
    rng = np.random.default_rng(3)
    scale, mx = _scales(rng, 4096)
    v = np.stack([mx, -mx], 1)
    got, _ = shortcut(v, scale[:, None])
    assert np.array_equal(got, exact(v, scale[:, None]))
    assert np.abs(got).max() <= 128
