"""The layer-op oracles (oracle/oracle.py) against the reference's own unit tests of
those layers, restated case by case:

* crates/yskn-ref/src/residual_norm_mlp.rs:124-133 (the projection is rounded to BF16
  before the residual sum);
* crates/yskn-ref/src/gated_deltanet.rs:762-786 (the convolution history keeps the raw
  BF16-rounded projections), :897-904 (dense gates of a 512-wide hidden row cover
  every element once) and :816-875 (M rows in one pass equal M one-row steps);
* crates/yskn-ref/src/attention.rs:1325-1342 (the cache rotation round trip is exact on
  small integer vectors) and :1345-1356 (each head's gate stays interleaved with its
  query; zero queries stay zero).

Together with the portable-math pins (tests/test_portable_math.py), which fix every
exp/log/rsqrt/sincos bit the layers use, these tie the layer oracles to yskn-ref."""
import numpy as np

import kv
import oracle as O


def _bits(x):
    return O.bf16_bits(np.asarray(x, np.float32))


def test_residual_rounds_projection_before_sum():
    # 1.00390625 is the midpoint between BF16 1 and 1.0078125: rounded before the sum it
    # cancels -1 exactly; rounding only the sum would not.
    hidden = np.zeros(512, np.float32)
    hidden[0] = -1.0
    proj = np.zeros(512, np.float32)
    proj[0] = np.array([0x3f808000], np.uint32).view(np.float32)[0]
    h, _, _, _ = O.residual_prepare(_bits(hidden), proj, _bits(np.zeros(512)), 1e-6)
    assert int(h[0]) == 0x0000


def test_dense_gates_cover_a_small_hidden_width_once():
    w = _bits(np.ones((4, 512), np.float32))
    out = O.gdn_gates(_bits(np.full(512, 0.5, np.float32)), np.float32(0.25), w, w)
    assert np.all(out == np.float32(64.0))


def _zero_gdn_weights():
    conv = _bits(np.full(10240 * 4, 0.25, np.float32))
    a_log = _bits(np.full(48, -2.0, np.float32))
    dt = _bits(np.zeros(48, np.float32))
    norm = _bits(np.ones(128, np.float32))
    return conv, a_log, dt, norm


def test_history_retains_raw_projected_bfloat_values():
    conv, a_log, dt, norm = _zero_gdn_weights()
    state = np.zeros((48, 128, 128), np.float32)
    hist = _bits(np.zeros((3, 10240), np.float32))
    z = np.full((1, 6144), 0.125, np.float32)
    gates = np.zeros((1, 96), np.float32)  # dense gates of a zero hidden row
    for x in (0.1, -0.2, 0.3, 0.4):
        _, state, hist = O.gdn_step(np.full((1, 10240), x, np.float32), z, gates, conv, a_log, dt, norm, 1e-6,
                                    state, hist)
    for age, x in enumerate((-0.2, 0.3, 0.4)):
        assert np.all(hist[age] == _bits(np.float32(x)))


def test_rows_in_one_pass_equal_one_row_steps():
    c = np.arange(10240)
    rows = [(((c * 7 + r * 5) % 23) / 32.0 - 0.3).astype(np.float32) for r in range(6)]
    zs = [(((np.arange(6144) + r) % 9) / 8.0 - 0.5).astype(np.float32) for r in range(6)]
    conv, a_log, dt, norm = _zero_gdn_weights()
    gates = np.tile(((np.arange(96) % 13) / 64.0 - 0.09).astype(np.float32), (6, 1))
    s0 = np.zeros((48, 128, 128), np.float32)
    h0 = _bits(np.zeros((3, 10240), np.float32))
    out_all, s_all, h_all = O.gdn_step(np.stack(rows), np.stack(zs), gates, conv, a_log, dt, norm, 1e-6, s0, h0)
    s, h = s0, h0
    for r in range(6):
        out, s, h = O.gdn_step(rows[r][None], zs[r][None], gates[r:r + 1], conv, a_log, dt, norm, 1e-6, s, h)
        assert np.array_equal(out[0].view(np.uint32), out_all[r].view(np.uint32))
    assert np.array_equal(s.view(np.uint32), s_all.view(np.uint32)) and np.array_equal(h, h_all)


def test_cache_rotation_roundtrip_preserves_small_integer_vectors():
    values = ((np.arange(256) % 23) * 2.0 - 21.0).astype(np.float32)
    restored = kv.inverse_rotate(O.rotate_cache(values))
    assert np.array_equal(restored.view(np.uint32), values.view(np.uint32))


def test_query_projection_keeps_each_heads_gate_interleaved():
    q = np.zeros((2, 512), np.float32)
    q[0, 256:] = 0.25
    q[1, 256:] = -0.5
    zero_norm = _bits(np.zeros(256, np.float32))
    query, gate, _, _ = O.attention_prep(q, np.zeros((2, 256), np.float32), np.zeros((2, 256), np.float32),
                                         zero_norm, zero_norm, 0, 1e-6)
    assert np.all(O.bf16_float(gate[0]) == 0.25) and np.all(O.bf16_float(gate[1]) == -0.5)
    assert np.all(O.bf16_float(query) == 0.0)
