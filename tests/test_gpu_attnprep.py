"""Attention inputs (yskn_b200_attention_prep) against the oracle of docs/spec/
04_ATTENTION.md:15-106 (attention.rs:570-775): queries, gates, keys and values bit for
bit. The head norm's rsqrt and RoPE's cosine and sine are the scalar contract's portable
functions on the device (portable_math.rs:106-109,406-434), as in the oracle; positions
up to 40000 and beyond 2^16 exercise the binary64 argument reduction.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def test_attention_prep_matches_the_oracle(cuda):
    import torch
    import yskn_b200
    M, n_qh, n_kvh, eps = 4, 24, 4, 1e-6
    rng = np.random.default_rng(21)
    q = (rng.standard_normal((M, n_qh, 512)) * 2).astype(np.float32)
    k = (rng.standard_normal((M, n_kvh, 256)) * 2).astype(np.float32)
    v = rng.standard_normal((M, n_kvh, 256)).astype(np.float32)
    qn = O.bf16_bits((rng.standard_normal(256) * 0.1).astype(np.float32))
    kn = O.bf16_bits((rng.standard_normal(256) * 0.1).astype(np.float32))
    pos = np.array([0, 7, 40000, 262141], np.int32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    query = torch.empty((M, n_qh, 256), dtype=torch.int16, device="cuda")
    gate = torch.empty((M, n_qh, 256), dtype=torch.int16, device="cuda")
    kr = torch.empty((M, n_kvh, 256), dtype=torch.float32, device="cuda")
    vr = torch.empty((M, n_kvh, 256), dtype=torch.float32, device="cuda")
    yskn_b200.attention_prep(dev(q), dev(k), dev(v), dev(qn.view(np.int16)), dev(kn.view(np.int16)), dev(pos), eps,
                             query, gate, kr, vr)
    assert yskn_b200.status() == 0
    gg, gk, gv = gate.cpu().numpy().view(np.uint16), kr.cpu().numpy(), vr.cpu().numpy()
    for m in range(M):
        wq, wg, wk, wv = O.attention_prep(q[m], k[m], v[m], qn, kn, int(pos[m]), eps)
        assert np.array_equal(gg[m], wg)
        assert np.array_equal(gv[m].view(np.uint32), wv.view(np.uint32))
        assert np.array_equal(query.cpu().numpy()[m].view(np.uint16), wq), m
        assert np.array_equal(gk[m].view(np.uint32), wk.view(np.uint32)), m
