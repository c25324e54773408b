"""Attention inputs (yskn_b200_attention_prep) against the oracle of docs/spec/
04_ATTENTION.md:15-106. The gate copies and the rotated values use no transcendental
function and match bit for bit. Queries and keys pass through CUDA's rsqrtf, cosf and
sinf (as in the reference; ATT-02: their bits are not portable, the oracle uses correctly
rounded / numpy float32 values): at least 90 % of them match bit for bit and every one
lies within 2^-8 of its head's largest magnitude (about one bf16 unit of the head's scale).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def test_attention_prep_matches_the_oracle(cuda):
    import torch
    import yskn_b200
    M, n_qh, n_kvh, eps = 3, 24, 4, 1e-6
    rng = np.random.default_rng(21)
    q = (rng.standard_normal((M, n_qh, 512)) * 2).astype(np.float32)
    k = (rng.standard_normal((M, n_kvh, 256)) * 2).astype(np.float32)
    v = rng.standard_normal((M, n_kvh, 256)).astype(np.float32)
    qn = O.bf16_bits((rng.standard_normal(256) * 0.1).astype(np.float32))
    kn = O.bf16_bits((rng.standard_normal(256) * 0.1).astype(np.float32))
    pos = np.array([0, 7, 40000], np.int32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    query = torch.empty((M, n_qh, 256), dtype=torch.int16, device="cuda")
    gate = torch.empty((M, n_qh, 256), dtype=torch.int16, device="cuda")
    kr = torch.empty((M, n_kvh, 256), dtype=torch.float32, device="cuda")
    vr = torch.empty((M, n_kvh, 256), dtype=torch.float32, device="cuda")
    yskn_b200.attention_prep(dev(q), dev(k), dev(v), dev(qn.view(np.int16)), dev(kn.view(np.int16)), dev(pos), eps,
                             query, gate, kr, vr)
    assert yskn_b200.status() == 0
    gq = O.bf16_float(query.cpu().numpy().view(np.uint16))
    gg, gk, gv = gate.cpu().numpy().view(np.uint16), kr.cpu().numpy(), vr.cpu().numpy()
    same_q = same_k = total_q = total_k = 0
    for m in range(M):
        wq, wg, wk, wv = O.attention_prep(q[m], k[m], v[m], qn, kn, int(pos[m]), eps)
        assert np.array_equal(gg[m], wg)
        assert np.array_equal(gv[m].view(np.uint32), wv.view(np.uint32))
        wq = O.bf16_float(wq)
        for got, want in ((gq[m], wq), (gk[m], wk)):
            bound = np.abs(want).max(axis=1, keepdims=True) * 2.0 ** -8
            assert (np.abs(got - want) <= bound).all(), m
        same_q += int((gq[m] == wq).sum())
        total_q += wq.size
        same_k += int((gk[m].view(np.uint32) == wk.view(np.uint32)).sum())
        total_k += wk.size
        if pos[m] == 0:  # cos 0 = 1, sin 0 = 0: only rsqrtf is left to differ
            assert (gq[m] == wq).mean() >= 0.99
    assert same_q >= 0.9 * total_q and same_k >= 0.9 * total_k, (same_q / total_q, same_k / total_k)
