"""Residual addition and deferred normalisation (yskn_b200_residual_prepare) against the
oracle of docs/spec/05_RESIDUAL_NORM_MLP.md:53-141 (residual_norm_mlp.rs, with the
portable rsqrt and silu of the scalar contract): the updated bf16 hidden row, the next
projection's f32 input, the bf16 gate copy and the inverse RMS bit for bit. The chain
into the next operator: yskn_b200_linear on the prepared input with the device's inverse
RMS equals the oracle's operator bit for bit. The gated product is bit-exact too.
"""
import numpy as np
import pytest

import container
import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _case(M, cols, seed):
    rng = np.random.default_rng(seed)
    hidden = O.bf16_bits(rng.standard_normal((M, cols)).astype(np.float32) * np.float32(0.5))
    proj = (rng.standard_normal((M, cols)) * 0.3).astype(np.float32)
    weight = O.bf16_bits((rng.standard_normal(cols) * 0.1).astype(np.float32))
    return hidden, proj, weight


@pytest.mark.parametrize("M,cols,with_projection", [(1, 5120, True), (3, 5120, True), (2, 1024, False),
                                                    (5, 17408, True)])
def test_residual_prepare_matches_the_oracle(cuda, M, cols, with_projection):
    import torch
    import yskn_b200
    hidden, proj, weight = _case(M, cols, M * cols)
    eps = 1e-6
    dh = torch.from_numpy(hidden.view(np.int16).copy()).cuda()
    dp = torch.from_numpy(proj).cuda() if with_projection else None
    dw = torch.from_numpy(weight.view(np.int16).copy()).cuda()
    inp = torch.empty((M, cols), dtype=torch.float32, device="cuda")
    inv = torch.empty(M, dtype=torch.float32, device="cuda")
    gate = torch.empty((M, cols), dtype=torch.int16, device="cuda")
    yskn_b200.residual_prepare(dh, dp, dw, eps, inp, inv, gate)
    assert yskn_b200.status() == 0
    got_h = dh.cpu().numpy().view(np.uint16)
    got_x, got_inv, got_g = inp.cpu().numpy(), inv.cpu().numpy(), gate.cpu().numpy().view(np.uint16)
    for m in range(M):
        h, x, r, g = O.residual_prepare(hidden[m], proj[m] if with_projection else None, weight, eps)
        assert np.array_equal(got_h[m], h)
        assert np.array_equal(got_x[m].view(np.uint32), x.view(np.uint32))
        assert np.array_equal(got_g[m], g)
        assert np.float32(got_inv[m]).view(np.uint32) == np.float32(r).view(np.uint32), (got_inv[m], r)


def test_prepared_input_feeds_the_next_operator(cuda):
    import torch
    import yskn_b200
    M, cols, rows = 2, 1024, 1024
    hidden, proj, weight = _case(M, cols, 7)
    dh = torch.from_numpy(hidden.view(np.int16).copy()).cuda()
    dw = torch.from_numpy(weight.view(np.int16).copy()).cuda()
    inp = torch.empty((M, cols), dtype=torch.float32, device="cuda")
    inv = torch.empty(M, dtype=torch.float32, device="cuda")
    yskn_b200.residual_prepare(dh, torch.from_numpy(proj).cuda(), dw, 1e-6, inp, inv)
    c = container.Container(fixtures.synthetic(8, "warp", rows, rows, cols, True))
    d = c.tensors["linear"]
    si = O.tensor_signs(d["rot_in"], cols)
    so = O.tensor_signs(d["rot_out"], rows)
    words = torch.from_numpy(c.words("linear").view(np.int32)).cuda()
    m = yskn_b200.Matrix(words, "warp", rows, rows, cols, 8, c.lut16("linear"), c.scale16("linear"), si, so)
    work = torch.empty(yskn_b200.linear_work_bytes([m], M), dtype=torch.uint8, device="cuda")
    y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
    yskn_b200.linear([m], inp, work, [y], inv_rms=inv)
    want = O.linear(c.words("linear"), "warp", rows, cols, 8, c.lut16("linear"), c.scale16("linear"),
                    inp.cpu().numpy(), si, so, inv_rms=inv.cpu().numpy())
    assert np.array_equal(y.cpu().numpy().view(np.uint32), np.asarray(want, np.float32).view(np.uint32))
    assert yskn_b200.status() == 0


def test_gated_product_matches_the_oracle(cuda):
    """bf16(bf16(silu(g)) * u) bit for bit, including +-0, large positive and negative
    gates (exp(-g) overflowing to +inf gives -0 * u)."""
    import torch
    import yskn_b200
    M, n = 3, 17408
    rng = np.random.default_rng(11)
    gate = (rng.standard_normal((M, n)) * 3).astype(np.float32)
    up = rng.standard_normal((M, n)).astype(np.float32)
    gate[0, :6] = [0.0, -0.0, 30.0, -30.0, 88.0, -100.0]
    out = torch.empty((M, n), dtype=torch.float32, device="cuda")
    yskn_b200.gated_product(torch.from_numpy(gate).cuda(), torch.from_numpy(up).cuda(), out)
    got = out.cpu().numpy()
    want = O.gated_product(gate, up)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert yskn_b200.status() == 0
