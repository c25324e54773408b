"""One MLP block as the reference's decode loop runs it (docs/spec/05_RESIDUAL_NORM_MLP.md:
12-44), through the library's calls: residual + normalisation -> gate/up operator (one
call, inverse RMS in its restore) -> gated product -> down operator (no inverse RMS) ->
residual + normalisation of the next layer. The oracle runs the same chain on its own,
from the same inputs only (never the device's intermediate values), and every stage's
device output equals it bit for bit: the operators' integer sums and restores, the
residual steps, and the inverse RMS and SiLU through the scalar contract's portable
functions.
"""
import numpy as np
import pytest

import fixtures
import oracle as O

pytestmark = pytest.mark.gpu

HIDDEN, FFN = 1024, 2048


def _matrix(rows, cols, seed, sign_offset):
    import torch
    import yskn_b200
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, seed, rows)
    si = O.signs("mulberry32_7919_13", 7, sign_offset, cols)
    so = O.signs("mulberry32_7919_13", 7, sign_offset + cols, rows)
    dw = torch.from_numpy(words.view(np.int32)).cuda()
    m = yskn_b200.Matrix(dw, "warp", rows, rows, cols, 8, lut16, sc16, si, so)
    return m, (words, lut16, sc16, si, so), dw


def _oracle_linear(spec, rows, cols, x, inv_rms=None):
    words, lut16, sc16, si, so = spec
    return np.asarray(O.linear(words, "warp", rows, cols, 8, lut16, sc16, x, si, so, inv_rms=inv_rms), np.float32)


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_mlp_block_chain(cuda):
    import torch
    import yskn_b200
    M = 2
    rng = np.random.default_rng(5)
    hidden = O.bf16_bits(rng.standard_normal((M, HIDDEN)).astype(np.float32) * np.float32(0.5))
    attn_out = (rng.standard_normal((M, HIDDEN)) * 0.3).astype(np.float32)
    w_post = O.bf16_bits((rng.standard_normal(HIDDEN) * 0.1).astype(np.float32))
    w_next = O.bf16_bits((rng.standard_normal(HIDDEN) * 0.1).astype(np.float32))
    eps = 1e-6
    gate, gate_spec, _k1 = _matrix(FFN, HIDDEN, 41, 0)
    up, up_spec, _k2 = _matrix(FFN, HIDDEN, 42, 0)
    down, down_spec, _k3 = _matrix(HIDDEN, FFN, 43, 4096)

    dh = torch.from_numpy(hidden.view(np.int16).copy()).cuda()
    w1 = torch.from_numpy(w_post.view(np.int16).copy()).cuda()
    w2 = torch.from_numpy(w_next.view(np.int16).copy()).cuda()
    x = torch.empty((M, HIDDEN), dtype=torch.float32, device="cuda")
    inv = torch.empty(M, dtype=torch.float32, device="cuda")
    g = torch.empty((M, FFN), dtype=torch.float32, device="cuda")
    u = torch.empty((M, FFN), dtype=torch.float32, device="cuda")
    mlp = torch.empty((M, FFN), dtype=torch.float32, device="cuda")
    d = torch.empty((M, HIDDEN), dtype=torch.float32, device="cuda")
    work = torch.empty(max(yskn_b200.linear_work_bytes([gate, up], M), yskn_b200.linear_work_bytes([down], M)),
                       dtype=torch.uint8, device="cuda")

    yskn_b200.residual_prepare(dh, torch.from_numpy(attn_out).cuda(), w1, eps, x, inv)
    yskn_b200.linear([gate, up], x, work, [g, u], inv_rms=inv)
    yskn_b200.gated_product(g, u, mlp)
    yskn_b200.linear([down], mlp, work, [d])
    h1 = dh.clone()
    x2 = torch.empty_like(x)
    inv2 = torch.empty_like(inv)
    yskn_b200.residual_prepare(dh, d, w2, eps, x2, inv2)
    assert yskn_b200.status() == 0

    X, INV, G, U, MLP, D = (t.cpu().numpy() for t in (x, inv, g, u, mlp, d))
    # The oracle's own chain.
    stage1 = [O.residual_prepare(hidden[m], attn_out[m], w_post, eps) for m in range(M)]
    h_o = np.stack([st[0] for st in stage1])
    x_o = np.stack([st[1] for st in stage1])
    inv_o = np.array([st[2] for st in stage1], np.float32)
    g_o = _oracle_linear(gate_spec, FFN, HIDDEN, x_o, inv_o)
    u_o = _oracle_linear(up_spec, FFN, HIDDEN, x_o, inv_o)
    mlp_o = O.gated_product(g_o, u_o)
    d_o = _oracle_linear(down_spec, HIDDEN, FFN, mlp_o)
    stage2 = [O.residual_prepare(h_o[m], d_o[m], w_next, eps) for m in range(M)]
    assert np.array_equal(h1.cpu().numpy().view(np.uint16), h_o)
    assert np.array_equal(_bits(X), _bits(x_o))
    assert np.array_equal(_bits(INV), _bits(inv_o))
    assert np.array_equal(_bits(G), _bits(g_o))
    assert np.array_equal(_bits(U), _bits(u_o))
    assert np.array_equal(_bits(MLP), _bits(mlp_o))
    assert np.array_equal(_bits(D), _bits(d_o))
    assert np.array_equal(dh.cpu().numpy().view(np.uint16), np.stack([st[0] for st in stage2]))
    assert np.array_equal(_bits(x2.cpu().numpy()), _bits(np.stack([st[1] for st in stage2])))
    assert np.array_equal(_bits(inv2.cpu().numpy()), _bits(np.array([st[2] for st in stage2], np.float32)))
