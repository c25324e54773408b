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


@pytest.mark.parametrize("M", [1, 2])
def test_fused_chain_equals_the_separate_calls(cuda, M):
    """The f1 chain inside the operators (yskn_b200_linear_residual -> linear_q8 ->
    gated_product_q8 -> linear_residual) against the same block through the separate
    calls (linear -> residual_prepare -> linear -> gated_product -> linear ->
    residual_prepare -> quantize), stage by stage, bit for bit: the residual stream, the
    next operator's int8 input and scales, the 1/rms, the gate/up outputs, the dense-gate
    copy."""
    import torch
    import yskn_b200
    H, F = 1024, 2048
    rng = np.random.default_rng(11 + M)
    eps = 1e-6
    hidden0 = O.bf16_bits(rng.standard_normal((M, H)).astype(np.float32) * np.float32(0.5))
    attn = (rng.standard_normal((M, F)) * 0.3).astype(np.float32)  # the o projection's input
    w_post = O.bf16_bits((rng.standard_normal(H) * 0.1).astype(np.float32))
    w_next = O.bf16_bits((rng.standard_normal(H) * 0.1).astype(np.float32))
    o, _, _ko = _matrix(H, F, 51, 8192)
    gate, _, _k1 = _matrix(F, H, 41, 0)
    up, _, _k2 = _matrix(F, H, 42, 0)
    down, _, _k3 = _matrix(H, F, 43, 4096)
    nxt, _, _k4 = _matrix(F, H, 44, 100)  # the next layer's first matrix (its input signs)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    x_attn = dev(attn)
    w1, w2 = dev(w_post.view(np.int16)), dev(w_next.view(np.int16))
    f32 = lambda *s: torch.empty(s, dtype=torch.float32, device="cuda")  # noqa: E731
    i8 = lambda *s: torch.empty(s, dtype=torch.int8, device="cuda")  # noqa: E731

    def quant(x, mat):
        a, al = i8(*x.shape), f32(x.shape[0], x.shape[1] // 512)
        yskn_b200.quantize(x, mat.signs_in_ptr, a, al, torch.empty_like(al, dtype=torch.int32), f32(x.shape[0]))
        return a, al

    def same(a, b):
        f = lambda t: t.view(torch.int32) if t.dtype == torch.float32 else t  # noqa: E731
        return torch.equal(f(a), f(b))

    wk = torch.empty(max(yskn_b200.linear_work_bytes(s, M) for s in ([o], [gate, up], [down])), dtype=torch.uint8,
                     device="cuda")
    # stage 1: o projection -> residual -> next input
    h = dev(hidden0.view(np.int16))
    y_o, x2, inv2 = f32(M, H), f32(M, H), f32(M)
    yskn_b200.linear([o], x_attn, wk, [y_o])
    yskn_b200.residual_prepare(h, y_o, w1, eps, x2, inv2)
    a2_want, al2_want = quant(x2, gate)
    hf = dev(hidden0.view(np.int16))
    a2, al2, b2 = i8(M, H), f32(M, H // 512), f32(M, H // 512)
    yskn_b200.linear_residual(o, hf, w1, gate.signs_in_ptr, a2, al2, b2, x=x_attn)
    torch.cuda.synchronize()
    assert same(hf, h), "residual stream after o"
    assert same(al2, al2_want), "group scales of the gate/up input"
    assert same(a2, a2_want), "int8 gate/up input"
    # stage 2: gate/up from the int8 input and the block sums
    g, u, gf, uf, inv2f = f32(M, F), f32(M, F), f32(M, F), f32(M, F), f32(M)
    yskn_b200.linear([gate, up], x2, wk, [g, u], inv_rms=inv2)
    yskn_b200.linear_q8([gate, up], a2, al2, [gf, uf], bss=b2, eps=eps, inv_rms_out=inv2f)
    torch.cuda.synchronize()
    assert same(inv2f, inv2), "1/rms from the block sums"
    assert same(gf, g) and same(uf, u), "gate/up outputs"
    # stage 3: the product quantised for down
    m = f32(M, F)
    yskn_b200.gated_product(g, u, m)
    am_want, alm_want = quant(m, down)
    am, alm = i8(M, F), f32(M, F // 512)
    yskn_b200.gated_product_q8(gf, uf, down.signs_in_ptr, am, alm)
    torch.cuda.synchronize()
    assert same(alm, alm_want) and same(am, am_want), "quantised product"
    # stage 4: down from the int8 input -> residual -> next input with the gate copy
    y_d, x3, inv3 = f32(M, H), f32(M, H), f32(M)
    xg3 = torch.empty((M, H), dtype=torch.int16, device="cuda")
    yskn_b200.linear([down], m, wk, [y_d])
    yskn_b200.residual_prepare(h, y_d, w2, eps, x3, inv3, gate=xg3)
    a3_want, al3_want = quant(x3, nxt)
    a3f, al3f, b3f = i8(M, H), f32(M, H // 512), f32(M, H // 512)
    xg3f = torch.empty((M, H), dtype=torch.int16, device="cuda")
    yskn_b200.linear_residual(down, hf, w2, nxt.signs_in_ptr, a3f, al3f, b3f, act=am, alpha=alm, gate_out=xg3f)
    torch.cuda.synchronize()
    assert yskn_b200.status() == 0
    assert same(hf, h), "residual stream after down"
    assert same(xg3f, xg3), "dense-gate copy"
    assert same(a3f, a3_want) and same(al3f, al3_want), "next layer's int8 input"
    tot = np.zeros(M, np.float32)
    for bidx in range(H // 512):
        tot = (tot + b3f.cpu().numpy()[:, bidx]).astype(np.float32)
    inv_from_blocks = O.pm("rsqrt", ((tot / np.float32(H)).astype(np.float32) + np.float32(eps)).astype(np.float32))
    assert np.array_equal(inv_from_blocks.view(np.uint32), inv3.cpu().numpy().view(np.uint32)), "block sums"


@pytest.mark.parametrize("M", [1, 3])
def test_residual_prologue_equals_residual_prepare_then_linear(cuda, M):
    """yskn_b200_linear_from_residual (the residual add, normalisation and quantiser formed in
    every CTA of the next operator's launch) against residual_prepare followed by the
    operator, bit for bit: the outputs of two matrices sharing the input, the updated
    residual stream (in the other buffer, the input buffer untouched), the dense-gate copy
    and the 1/rms; three calls in a row, so the scratch is reused."""
    import torch
    import yskn_b200
    H, F = 1024, 2048
    eps = 1e-6
    rng = np.random.default_rng(21 + M)
    gate, _, _k1 = _matrix(F, H, 61, 0)
    up, _, _k2 = _matrix(F, H, 62, 0)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    f32 = lambda *s: torch.empty(s, dtype=torch.float32, device="cuda")  # noqa: E731
    i16 = lambda *s: torch.empty(s, dtype=torch.int16, device="cuda")  # noqa: E731
    wk = torch.empty(yskn_b200.linear_work_bytes([gate, up], M), dtype=torch.uint8, device="cuda")
    for call in range(3):
        hidden0 = O.bf16_bits(rng.standard_normal((M, H)).astype(np.float32) * np.float32(0.5))
        y = (rng.standard_normal((M, H)) * 0.3).astype(np.float32)
        w = O.bf16_bits((rng.standard_normal(H) * 0.1).astype(np.float32))
        # separate calls
        h = dev(hidden0.view(np.int16))
        x, inv, xg = f32(M, H), f32(M), i16(M, H)
        yskn_b200.residual_prepare(h, dev(y), dev(w.view(np.int16)), eps, x, inv, gate=xg)
        g, u = f32(M, F), f32(M, F)
        yskn_b200.linear([gate, up], x, wk, [g, u], inv_rms=inv)
        # the residual prologue
        h_in = dev(hidden0.view(np.int16))
        h_out, xg2, inv2 = i16(M, H), i16(M, H), f32(M)
        g2, u2 = f32(M, F), f32(M, F)
        yskn_b200.linear_from_residual([gate, up], dev(y), h_in, h_out, dev(w.view(np.int16)), eps, [g2, u2],
                                       gate_out=xg2, inv_rms_out=inv2)
        torch.cuda.synchronize()
        assert yskn_b200.status() == 0
        assert torch.equal(h_out, h), call
        assert np.array_equal(h_in.cpu().numpy().view(np.uint16), hidden0), call
        assert torch.equal(xg2, xg), call
        assert torch.equal(inv2.view(torch.int32), inv.view(torch.int32)), call
        assert torch.equal(g2.view(torch.int32), g.view(torch.int32)), call
        assert torch.equal(u2.view(torch.int32), u.view(torch.int32)), call

