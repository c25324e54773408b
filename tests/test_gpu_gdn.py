"""Gated DeltaNet decode step (yskn_b200_gdn_gates, yskn_b200_gdn_step) against the oracle of
docs/spec/03_GATED_DELTANET.md:57-186, ordinary causal rows, three calls in a row (the state
and the convolution history carried between them): a committed row, a provisional four-row
verification (state and history untouched, bit for bit) and four rows committing two.
The dense gates, the history, the gated outputs and the state match bit for bit: the step
uses the scalar contract's portable exp, rsqrt, sigmoid, softplus and silu
(gated_deltanet.rs:332-577) on the device, and the oracle restates the same functions.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mixer", [False, True])
def test_gdn_gates_and_steps(cuda, mixer):
    """mixer: yskn_b200_gdn_mixer (gates, step and history in one launch) in place of the
    gates and step calls, against the same oracle."""
    import torch
    import yskn_b200
    rng = np.random.default_rng(17)
    hidden, eps = 5120, 1e-6
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wb = O.bf16_bits((rng.standard_normal((48, hidden)) * 0.02).astype(np.float32))
    wa = O.bf16_bits((rng.standard_normal((48, hidden)) * 0.02).astype(np.float32))
    conv = O.bf16_bits((rng.standard_normal((10240, 4)) * 0.5).astype(np.float32))
    a_log = O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32))
    dt_bias = O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32))
    norm_w = O.bf16_bits((1 + rng.standard_normal(128) * 0.1).astype(np.float32))
    state = (rng.standard_normal((48, 128, 128)) * 0.1).astype(np.float32)
    history = O.bf16_bits(rng.standard_normal((3, 10240)).astype(np.float32))
    d_state, d_hist = dev(state), dev(history.view(np.int16))
    for call, (M, n_commit) in enumerate([(1, 1), (4, 0), (4, 2)]):
        x = O.bf16_bits(rng.standard_normal((M, hidden)).astype(np.float32))
        inv = (0.5 + rng.random(M)).astype(np.float32)
        qkv = rng.standard_normal((M, 10240)).astype(np.float32)
        z = rng.standard_normal((M, 6144)).astype(np.float32)
        out = torch.empty((M, 6144), dtype=torch.float32, device="cuda")
        before = d_state.cpu().numpy()
        step_args = (dev(conv.view(np.int16)), dev(a_log.view(np.int16)), dev(dt_bias.view(np.int16)),
                     dev(norm_w.view(np.int16)), eps, d_state, d_hist, out)
        want_g = np.stack([O.gdn_gates(x[m], inv[m], wb, wa) for m in range(M)])
        if mixer:
            yskn_b200.gdn_mixer(dev(x.view(np.int16)), dev(inv), dev(wb.view(np.int16)), dev(wa.view(np.int16)),
                                dev(qkv), dev(z), *step_args, n_commit=n_commit)
            g = want_g
        else:
            gates = torch.empty((M, 96), dtype=torch.float32, device="cuda")
            yskn_b200.gdn_gates(dev(x.view(np.int16)), dev(inv), dev(wb.view(np.int16)), dev(wa.view(np.int16)),
                                gates)
            g = gates.cpu().numpy()
            assert np.array_equal(g.view(np.uint32), want_g.view(np.uint32)), call
            yskn_b200.gdn_step(dev(qkv), dev(z), gates, *step_args, n_commit=n_commit)
        assert yskn_b200.status() == 0
        want_out, state, history = O.gdn_step(qkv, z, g, conv, a_log, dt_bias, norm_w, eps, state, history, n_commit)
        got = out.cpu().numpy()
        assert np.array_equal(d_hist.cpu().numpy().view(np.uint16), history), call
        assert np.array_equal(got.view(np.uint32), want_out.view(np.uint32)), call
        got_state = d_state.cpu().numpy()
        if n_commit == 0:
            assert np.array_equal(got_state.view(np.uint32), before.view(np.uint32))
        assert np.array_equal(got_state.view(np.uint32), state.view(np.uint32)), call


def test_gdn_rows_together_equal_rows_one_by_one(cuda):
    """Causal rows in one call and one row per call give the same bits: the recurrence and
    the convolution see the same operands in the same order (M = 5, longer than the history)."""
    import torch
    import yskn_b200
    rng = np.random.default_rng(23)
    M = 5
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    conv = dev(O.bf16_bits((rng.standard_normal((10240, 4)) * 0.5).astype(np.float32)).view(np.int16))
    a_log = dev(O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32)).view(np.int16))
    dt_bias = dev(O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32)).view(np.int16))
    norm_w = dev(O.bf16_bits((1 + rng.standard_normal(128) * 0.1).astype(np.float32)).view(np.int16))
    state0 = (rng.standard_normal((48, 128, 128)) * 0.1).astype(np.float32)
    hist0 = O.bf16_bits(rng.standard_normal((3, 10240)).astype(np.float32)).view(np.int16)
    qkv = dev(rng.standard_normal((M, 10240)).astype(np.float32))
    z = dev(rng.standard_normal((M, 6144)).astype(np.float32))
    gates = dev(rng.standard_normal((M, 96)).astype(np.float32))
    s1, h1, o1 = dev(state0), dev(hist0), torch.empty((M, 6144), dtype=torch.float32, device="cuda")
    yskn_b200.gdn_step(qkv, z, gates, conv, a_log, dt_bias, norm_w, 1e-6, s1, h1, o1)
    s2, h2, o2 = dev(state0), dev(hist0), torch.empty((M, 6144), dtype=torch.float32, device="cuda")
    for r in range(M):
        yskn_b200.gdn_step(qkv[r:r + 1], z[r:r + 1], gates[r:r + 1], conv, a_log, dt_bias, norm_w, 1e-6, s2, h2,
                           o2[r:r + 1])
    assert yskn_b200.status() == 0
    assert torch.equal(o1.view(torch.int32), o2.view(torch.int32))
    assert torch.equal(s1.view(torch.int32), s2.view(torch.int32))
    assert torch.equal(h1, h2)
