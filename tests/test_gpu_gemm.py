"""The tcgen05 GEMM path (M >= 64 activation rows) against the CPU oracle, bit-exact.

Shapes mirror the reference's kernel tests (crates/yskn-engine/tests/linear.rs:9-108)
at prefill sizes: every bit width, both layouts, physical rows that are not a
multiple of the 128-row tile, M not a multiple of the 128-row tile, signed i32
scales and extreme activations; then the 27B gate_proj shape.
"""
import numpy as np
import pytest

import container
import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _inputs(cols, n, seed):
    rnd = fixtures.FixtureRandom(seed)
    act = rnd.take(n * cols).astype(np.uint8).view(np.int8).reshape(n, cols).copy()
    act[1] = 127
    act[2] = -128
    act[3] = 0
    A = rnd.take(n * (cols // 512)).view(np.int32).reshape(n, -1).copy()
    return act, A


@pytest.mark.parametrize("bits", [4, 5, 6, 7, 8])
@pytest.mark.parametrize("layout", ["row", "warp"])
def test_gemm_matches_scalar_reference(cuda, bits, layout):
    import torch
    import yskn_b200
    for rows, phys, cols in [(65, 96, 1024), (300, 320, 512), (1000, 1000, 1536)]:
        if layout == "warp" and (phys * cols // 256) % 32:
            continue
        c = container.Container(fixtures.synthetic(bits, layout, rows, phys, cols, False))
        lut8, _ = O.quantize_weight_table(c.lut16("linear"), c.scale16("linear"))
        act, A = _inputs(cols, 200, 0x5EED + bits)
        ref = O.fast_weighted_sums(c.words("linear"), layout, phys, cols, bits, lut8, act, A)
        d = c.tensors["linear"]
        words = _dev(c.words("linear").view(np.int32))
        m = yskn_b200.Matrix(words, layout, rows, phys, cols, bits, c.lut16("linear"), c.scale16("linear"),
                             O.tensor_signs(d["rot_in"], cols))
        da, dA = _dev(act), _dev(A)
        for M in (64, 129, 200):
            out = torch.full((M, phys), -7, dtype=torch.int64, device="cuda")
            yskn_b200.weighted_sums([m], da[:M], dA[:M], [out])
            assert np.array_equal(out.cpu().numpy(), ref[:M]), (bits, layout, rows, phys, cols, M)
        pre = torch.empty((100, rows), dtype=torch.int64, device="cuda")
        yskn_b200.weighted_sums_prefix(m, da[:100], dA[:100], rows, pre)
        assert np.array_equal(pre.cpu().numpy(), ref[:100, :rows])
        assert yskn_b200.status() == 0


def test_gemm_27b_gate_shape(cuda):
    import torch
    import yskn_b200
    rows, cols, bits, M = 17408, 5120, 8, 256
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, bits, 2024)
    lut8, _ = O.quantize_weight_table(lut16, sc16)
    x = fixtures.normal(5, M * cols).reshape(M, cols)
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    act, _, A, _ = O.quantize_activation(x, si)
    ref = O.fast_weighted_sums(words, "warp", rows, cols, bits, lut8, act, A)
    dw = _dev(words.view(np.int32))
    m = yskn_b200.Matrix(dw, "warp", rows, rows, cols, bits, lut16, sc16, si)
    out = torch.empty((M, rows), dtype=torch.int64, device="cuda")
    yskn_b200.weighted_sums([m], _dev(act), _dev(A), [out])
    assert np.array_equal(out.cpu().numpy(), ref)
    assert yskn_b200.status() == 0
