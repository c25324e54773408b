"""CPU checks of the layer oracles that have no golden vectors in the reference: the Gated
DeltaNet step's commit rules (docs/spec/03_GATED_DELTANET.md:160-186) and its row-by-row
equivalence, at small sizes."""
import numpy as np

import oracle as O


def _gdn_inputs(rng, M):
    return dict(qkv=rng.standard_normal((M, 10240)).astype(np.float32),
                z=rng.standard_normal((M, 6144)).astype(np.float32),
                gates=rng.standard_normal((M, 96)).astype(np.float32))


def _gdn_weights(rng):
    return (O.bf16_bits((rng.standard_normal((10240, 4)) * 0.5).astype(np.float32)),
            O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32)),
            O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32)),
            O.bf16_bits((1 + rng.standard_normal(128) * 0.1).astype(np.float32)))


def test_gdn_commit_rules():
    rng = np.random.default_rng(3)
    w = _gdn_weights(rng)
    state = (rng.standard_normal((48, 128, 128)) * 0.1).astype(np.float32)
    hist = O.bf16_bits(rng.standard_normal((3, 10240)).astype(np.float32))
    x = _gdn_inputs(rng, 4)
    out_all, s_all, h_all = O.gdn_step(x["qkv"], x["z"], x["gates"], *w, 1e-6, state, hist)
    out_p, s_p, h_p = O.gdn_step(x["qkv"], x["z"], x["gates"], *w, 1e-6, state, hist, n_commit=0)
    assert np.array_equal(out_all, out_p)  # the outputs do not depend on the commit point
    assert np.array_equal(s_p, state) and np.array_equal(h_p, hist)
    assert np.array_equal(h_all, O.bf16_bits(x["qkv"][1:4]))
    out_2, s_2, h_2 = O.gdn_step(x["qkv"], x["z"], x["gates"], *w, 1e-6, state, hist, n_commit=2)
    assert np.array_equal(out_2, out_all)
    assert np.array_equal(h_2, np.stack([hist[2], O.bf16_bits(x["qkv"][0]), O.bf16_bits(x["qkv"][1])]))
    # the state committed after two rows, then two more rows, is the state after four
    _, s_4, _ = O.gdn_step(x["qkv"][2:], x["z"][2:], x["gates"][2:], *w, 1e-6, s_2, h_2)
    assert np.array_equal(s_4, s_all)
    assert not np.array_equal(s_2, s_all)


def test_gdn_rows_one_by_one():
    rng = np.random.default_rng(4)
    w = _gdn_weights(rng)
    state = (rng.standard_normal((48, 128, 128)) * 0.1).astype(np.float32)
    hist = O.bf16_bits(rng.standard_normal((3, 10240)).astype(np.float32))
    x = _gdn_inputs(rng, 3)
    out_all, s_all, h_all = O.gdn_step(x["qkv"], x["z"], x["gates"], *w, 1e-6, state, hist)
    s, h = state, hist
    for r in range(3):
        out, s, h = O.gdn_step(x["qkv"][r:r + 1], x["z"][r:r + 1], x["gates"][r:r + 1], *w, 1e-6, s, h)
        assert np.array_equal(out[0], out_all[r])
    assert np.array_equal(s, s_all) and np.array_equal(h, h_all)


def test_cache_rotation_round_trip():
    """The attention-input rotation (signs, H256, 1/16; docs/spec/04_ATTENTION.md:80-100)
    is undone by the KV oracle's inverse rotation, written separately from the reference's
    decoder (H256, 1/16, signs): bit for bit on small integers, where every butterfly sum is
    exact, and within float rounding on normal values; the rotation keeps the norm."""
    import kv
    rng = np.random.default_rng(9)
    x = rng.integers(-8, 9, 256).astype(np.float32)
    assert np.array_equal(kv.inverse_rotate(O.rotate_cache(x)), x)
    y = rng.standard_normal(256).astype(np.float32)
    back = kv.inverse_rotate(O.rotate_cache(y))
    assert np.abs(back - y).max() <= 1e-5 * np.abs(y).max()
    assert abs(np.linalg.norm(O.rotate_cache(y)) - np.linalg.norm(y)) <= 1e-5 * np.linalg.norm(y)


def _scan_top8(logits):
    """The reference's candidate comparison as a scalar scan (docs/spec/06_OUTPUT_HEAD_SAMPLER.md:
    31-64): start from (-FLT_MAX, INT_MAX), a candidate enters when it has the larger logit,
    or the same logit and the smaller id; NaN compares false and never enters."""
    top = [(np.float32(-3.4028234663852886e38), 2**31 - 1)] * 8
    for i, v in enumerate(np.asarray(logits, np.float32)):
        c = (v, i)
        for k in range(8):
            tv, ti = top[k]
            if c[0] > tv or (c[0] == tv and c[1] < ti):
                top[k], c = c, top[k]
    return top


def test_head_select_matches_a_scalar_scan():
    rng = np.random.default_rng(11)
    rows = [rng.standard_normal(300).astype(np.float32),
            np.round(rng.standard_normal(300) * 2).astype(np.float32),  # many ties
            np.full(20, np.nan, np.float32),
            np.array([np.nan, -np.inf, -3.4028234663852886e38, 1.0, np.inf, 1.0, np.nan], np.float32),
            np.array([-np.inf] * 5 + [2.0], np.float32)]
    for r in rows:
        token, vals, ids = O.head_select(r)
        want = _scan_top8(r)
        assert [int(i) for i in ids] == [i for _, i in want]
        assert np.array_equal(vals.view(np.uint32), np.array([v for v, _ in want], np.float32).view(np.uint32))
        assert token == want[0][1]


def _rsqrt(x):
    """portable_math.rs:106-109 one step at a time: the square root rounded to binary32
    (numpy's float32 sqrt is correctly rounded), then a rounded division."""
    return _f(_f(1.0) / np.sqrt(_f(x)))


def _pexp(x):
    return _f(O.pm_scalar("exp", float(_f(x))))


def _f(x):
    return np.float32(x)


def _scalar_total_squares(h):
    """docs/spec/05_RESIDUAL_NORM_MLP.md:70-101 one operation at a time: per 512 block, 128
    partials of four squares from +0, xor_sum32 of each group of 32 (every lane updated from
    the old values), the group sums added from +0, blocks added in order from +0."""
    total = _f(0.0)
    for b in range(0, h.size, 512):
        part = []
        for t in range(128):
            s = _f(0.0)
            for j in range(4):
                x = h[b + t + 128 * j]
                s = _f(s + _f(x * x))
            part.append(s)
        block = _f(0.0)
        for g in range(4):
            a = part[32 * g:32 * g + 32]
            for off in (16, 8, 4, 2, 1):
                a = [_f(a[i] + a[i ^ off]) for i in range(32)]
            block = _f(block + a[0])
        total = _f(total + block)
    return total


def test_residual_sum_of_squares_matches_a_scalar_restatement():
    rng = np.random.default_rng(13)
    for scale in (1e-3, 1.0, 300.0):
        hidden = O.bf16_bits((rng.standard_normal(1024) * scale).astype(np.float32))
        proj = (rng.standard_normal(1024) * scale).astype(np.float32)
        h, _, inv, _ = O.residual_prepare(hidden, proj, O.bf16_bits(np.zeros(1024, np.float32)), 1e-6)
        total = _scalar_total_squares(O.bf16_float(h))
        mean = _f(_f(total / _f(1024.0)) + _f(1e-6))
        assert np.float32(inv).view(np.uint32) == _rsqrt(mean).view(np.uint32)


def test_gdn_gates_match_a_scalar_restatement():
    """docs/spec/03_GATED_DELTANET.md:57-76 one operation at a time for a few outputs of one
    row (hidden 2048: two chunks of 1024)."""
    rng = np.random.default_rng(17)
    hidden = 2048
    x = O.bf16_bits(rng.standard_normal(hidden).astype(np.float32))
    wb = O.bf16_bits((rng.standard_normal((48, hidden)) * 0.05).astype(np.float32))
    wa = O.bf16_bits((rng.standard_normal((48, hidden)) * 0.05).astype(np.float32))
    inv = np.float32(0.731)
    got = O.gdn_gates(x, inv, wb, wa)
    xf = O.bf16_float(x)
    for o in (0, 17, 47, 48, 70, 95):
        w = O.bf16_float(wb[o] if o < 48 else wa[o - 48])
        partial = []
        for p in range(128):
            s = _f(0.0)
            for chunk in range(hidden // 1024):
                for e in range(8):
                    i = 8 * p + 1024 * chunk + e
                    s = _f(s + _f(w[i] * xf[i]))
            partial.append(s)
        grouped = []
        for g in range(4):
            a = partial[32 * g:32 * g + 32]
            for off in (16, 8, 4, 2, 1):
                a = [_f(a[i] + a[i ^ off]) for i in range(32)]
            grouped.append(a[0])
        s4 = _f(_f(_f(grouped[0] + grouped[1]) + grouped[2]) + grouped[3])
        want = O.bf16_float(O.bf16_bits(_f(s4 * inv)))
        assert np.float32(got[o]).view(np.uint32) == np.float32(want).view(np.uint32), o


def _bf(x):
    return O.bf16_float(O.bf16_bits(_f(x)))


def test_head_norm_and_rope_match_a_scalar_restatement():
    """docs/spec/04_ATTENTION.md:27-66 one operation at a time for one 256-channel head:
    xor_sum32 of each group's squares added from +0, the inverse RMS, bf16(y * inv * (1 + w)),
    then RoPE on channels (i, i + 32), i < 32, with bf16 cos/sin and the spec's roundings."""
    rng = np.random.default_rng(19)
    y = O.bf16_float(O.bf16_bits(rng.standard_normal(256).astype(np.float32) * 3))
    w_bits = O.bf16_bits((rng.standard_normal(256) * 0.1).astype(np.float32))
    w = O.bf16_float(w_bits)
    pos, eps = 1234, 1e-6
    got = O.rope(O.normalize_head(y, w_bits, eps), pos)
    total = _f(0.0)
    for g in range(8):
        a = [_f(y[32 * g + i] * y[32 * g + i]) for i in range(32)]
        for off in (16, 8, 4, 2, 1):
            a = [_f(a[i] + a[i ^ off]) for i in range(32)]
        total = _f(total + a[0])
    inv = _rsqrt(_f(_f(total / _f(256.0)) + _f(eps)))
    n = [_bf(_f(_f(y[i] * inv) * _f(_f(1.0) + w[i]))) for i in range(256)]
    freq = np.array(O.ROPE_FREQ_BITS, np.uint32).view(np.float32)
    want = list(n)
    for i in range(32):
        arg = _f(_f(pos) * freq[i])
        cs, sn = O.pm_sincos(np.float32(arg))
        c, s = _bf(cs), _bf(sn)
        want[i] = _bf(_bf(n[i] * c) + _bf(-n[i + 32] * s))
        want[i + 32] = _bf(_bf(n[i + 32] * c) + _bf(n[i] * s))
    assert np.array_equal(np.asarray(got, np.float32).view(np.uint32), np.array(want, np.float32).view(np.uint32))


def test_gdn_step_matches_a_scalar_restatement_for_one_head():
    """docs/spec/03_GATED_DELTANET.md:86-155 one operation at a time for value head 7 (key
    head 2) of one row after a history: convolution, q/k normalisation, beta and decay,
    the two 32-term passes per group over the state column, the output norm and z gate."""
    rng = np.random.default_rng(29)
    conv_bits, a_log_bits, dt_bits, norm_bits = _gdn_weights(rng)
    state = (rng.standard_normal((48, 128, 128)) * 0.1).astype(np.float32)
    hist = O.bf16_bits(rng.standard_normal((3, 10240)).astype(np.float32))
    x = _gdn_inputs(rng, 1)
    out, new_state, _ = O.gdn_step(x["qkv"], x["z"], x["gates"], conv_bits, a_log_bits, dt_bits, norm_bits, 1e-6,
                                   state, hist)
    vh, kh = 7, 2
    cw = O.bf16_float(conv_bits).reshape(-1, 4)
    hf = O.bf16_float(hist)
    silu = lambda v: _f(_f(v) / _f(_f(1.0) + _pexp(-_f(v))))  # noqa: E731

    def conv(c):
        taps = [hf[0, c], hf[1, c], hf[2, c], _bf(x["qkv"][0, c])]
        a = _f(cw[c, 0] * taps[0])
        for t in range(1, 4):
            a = _f(a + _f(cw[c, t] * taps[t]))
        return _bf(silu(_bf(a)))

    def squares128(v):
        parts = []
        for g in range(4):
            a = [_f(v[32 * g + i] * v[32 * g + i]) for i in range(32)]
            for off in (16, 8, 4, 2, 1):
                a = [_f(a[i] + a[i ^ off]) for i in range(32)]
            parts.append(a[0])
        return _f(_f(_f(parts[0] + parts[1]) + parts[2]) + parts[3])

    q = [conv(128 * kh + j) for j in range(128)]
    k = [conv(2048 + 128 * kh + j) for j in range(128)]
    v = [conv(4096 + 128 * vh + j) for j in range(128)]
    rq = _rsqrt(_f(squares128(q) + _f(1e-6)))
    rk = _rsqrt(_f(squares128(k) + _f(1e-6)))
    query = [_f(_f(qq * rq) * _f(0.08838834764831845)) for qq in q]
    key = [_f(kk * rk) for kk in k]
    g = x["gates"][0]
    beta = _bf(_f(_f(1.0) / _f(_f(1.0) + _pexp(-_f(g[vh])))))
    xa = _f(g[48 + vh] + O.bf16_float(dt_bits)[vh])
    sp = xa if xa > _f(20.0) else _f(O.pm_scalar("log1p", _pexp(xa)))
    decay = _pexp(_f(-_pexp(O.bf16_float(a_log_bits)[vh]) * sp))
    R = state[vh].copy()
    core = []
    for j in range(128):
        parts = []
        for grp in range(4):
            acc = _f(0.0)
            for r in range(32):
                i = 32 * grp + r
                R[i, j] = _f(R[i, j] * decay)
                acc = _f(acc + _f(R[i, j] * key[i]))
            parts.append(acc)
        corr = _f(_f(v[j] - _f(_f(_f(parts[0] + parts[1]) + parts[2]) + parts[3])) * beta)
        parts = []
        for grp in range(4):
            acc = _f(0.0)
            for r in range(32):
                i = 32 * grp + r
                R[i, j] = _f(R[i, j] + _f(key[i] * corr))
                acc = _f(acc + _f(R[i, j] * query[i]))
            parts.append(acc)
        core.append(_bf(_f(_f(_f(parts[0] + parts[1]) + parts[2]) + parts[3])))
    inv = _rsqrt(_f(_f(squares128(core) / _f(128.0)) + _f(1e-6)))
    nw = O.bf16_float(norm_bits)
    want = [_bf(_f(_bf(_f(nw[j] * _bf(_f(core[j] * inv)))) * silu(x["z"][0, 128 * vh + j]))) for j in range(128)]
    assert np.array_equal(out[0, 128 * vh:128 * vh + 128].view(np.uint32), np.array(want, np.float32).view(np.uint32))
    assert np.array_equal(new_state[vh].view(np.uint32), R.view(np.uint32))
