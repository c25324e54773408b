"""The library's device portable functions (yskn_b200_portable_math, csrc/pmath.cuh)
against the oracle's restatement of crates/yskn-ref/src/portable_math.rs, which the
reference's own known answers pin (tests/test_portable_math.py): bit for bit over a
million random inputs per function plus the edge cases (zeros, subnormals, overflow and
underflow thresholds, infinities, NaN). The layer kernels call exactly these."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _inputs(rng, positive=False):
    r = [rng.normal(0, 4, 400000), rng.normal(0, 40, 200000), rng.uniform(-110, 110, 200000),
         rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32).view(np.float32)]
    edge = np.array([0.0, -0.0, 1.0, -1.0, 0.5, 10.0, 20.0, 20.000002, -30.0, 88.72, 88.73, -103.0, -104.0, 89.0,
                     -126.0, -150.0, 1e-7, -1e-7, 1e-38, 1e-45, np.inf, -np.inf, np.nan, 3.4e38, -3.4e38],
                    np.float32)
    x = np.concatenate([a.astype(np.float32) for a in r] + [edge])
    x = x[np.isfinite(x) | np.isnan(x) | np.isinf(x)]
    if positive:
        x = np.abs(x)
        x = x[(x > 0) & np.isfinite(x)]
    return np.ascontiguousarray(x, np.float32)


def _same(got, want):
    g, w = got.view(np.uint32), want.view(np.uint32)
    nan = np.isnan(got) & np.isnan(want)
    return np.all((g == w) | nan)


@pytest.mark.parametrize("name,positive", [("exp", False), ("exp2", False), ("sigmoid", False), ("silu", False),
                                           ("softplus", False), ("rsqrt", True), ("log", True),
                                           ("log1p", True)])
def test_device_function_matches_the_portable_contract(cuda, name, positive):
    import torch
    import yskn_b200
    x = _inputs(np.random.default_rng(hash(name) & 0xffff), positive)
    if name == "softplus":  # the contract's domain: exp(x) feeds log1p (nonnegative)
        x = x[~np.isnan(x)]
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    yskn_b200.portable_math(name, dx, dy)
    assert yskn_b200.status() == 0
    got, want = dy.cpu().numpy(), O.pm(name, x)
    bad = np.flatnonzero(~((got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))))
    assert bad.size == 0, (name, x[bad[:5]], got[bad[:5]], want[bad[:5]])


def test_device_sincos_matches_the_portable_contract(cuda):
    import torch
    import yskn_b200
    rng = np.random.default_rng(12)
    freq = np.array(O.ROPE_FREQ_BITS, np.uint32).view(np.float32)
    pos = rng.integers(0, 300000, 20000).astype(np.float32)
    x = np.concatenate([(pos[:, None] * freq[None, :]).reshape(-1), rng.normal(0, 1e4, 200000).astype(np.float32),
                        np.array([0.0, -0.0, 1.0, 20.0, 1e6, -1e6, 3.14159265], np.float32)]).astype(np.float32)
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    dc, ds = torch.empty_like(dx), torch.empty_like(dx)
    yskn_b200.portable_math("sincos", dx, dc, ds)
    assert yskn_b200.status() == 0
    wc, ws = O.pm_sincos(x)
    assert np.array_equal(dc.cpu().numpy().view(np.uint32), wc.view(np.uint32))
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), ws.view(np.uint32))
