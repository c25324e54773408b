"""The KV codec / attention oracle against the reference's own known answers.

Pins:
  * the frozen SHA-256 of encoded rows at 4 and 5 bits
    (crates/yskn-ref/src/kv_codec_tests.rs:427-470): every encode path (packed,
    int8, residual with basis and mean, guard, Viterbi) byte for byte;
  * the prefix schedule's expected plans (crates/yskn-ref/src/attention.rs:1117-1138);
  * attend_head's 256 output bit patterns of the length-76 int8-row case
    (crates/yskn-ref/src/attention.rs:1244-1306), with the portable exp2/exp;
  * packed_state of the vectorised decoder against the C restatement of
    kv_codec.rs:467-475, and attend_head against plain float64 softmax attention.
"""
import hashlib

import numpy as np
import pytest

import kv

FROZEN = {
    4: "03ff805b36bd010e21ec2c5b722fa806811e21fd85e0710f2cf59c40d4263d0b",
    5: "1935bdce14986fc445e26499fe2b942aa0ebd0ef00b7eed6ac47e48402b60bb7",
}


@pytest.mark.parametrize("bits", [4, 5])
def test_frozen_codec_hash(bits):
    b = kv.test_profile(2, 2, bits)
    kv.replace_group(b, 1, 1, 1, 2, True)
    kv.replace_group(b, 3, 0, 0, 0, True)
    kv.replace_group(b, 5, 0, 0, 1, True)
    kv.replace_group(b, 7, 2, 0, 0, False)
    p = kv.parse_profile(b)
    out = bytearray()
    for x in kv.test_rows(0x05a0c0de, 4):
        for group in range(8):
            for pos in (0, 7):
                k, scale, words, ints, _, rs, ri = kv.encode(p, group, pos, x)
                out += kv.encoded_bytes(k, scale, words, ints)
                out += kv.encoded_bytes(8, rs, None, ri)
    assert hashlib.sha256(bytes(out)).hexdigest() == FROZEN[bits]


def test_prefix_schedule_known_plans():
    only_self = kv.prefix_schedule(1)
    assert len(only_self) == 31
    assert only_self[0] == ([], True)
    assert all(p == ([], False) for p in only_self[1:])
    short = kv.prefix_schedule(5)
    assert len(short) == 31
    assert short[:5] == [([(0, 0, 1)], False), ([(0, 1, 2)], False), ([(0, 2, 3)], False), ([(0, 3, 4)], False),
                         ([], True)]
    assert all(p == ([], False) for p in short[5:])
    assert len(kv.prefix_schedule(4095)) == 31 and len(kv.prefix_schedule(4096)) == 42
    for length in (1, 2, 33, 100, 4095, 4096, 5000):  # every prefix key exactly once, self exactly once
        plans = kv.prefix_schedule(length)
        keys = [k for tiles, _ in plans for _, a, e in tiles for k in range(a, e)]
        assert keys == list(range(length - 1))
        assert sum(s for _, s in plans) == 1


@pytest.mark.parametrize("bits", [4, 5])
def test_packed_states_match_c(bits):
    rng = np.random.default_rng(bits)
    words = rng.integers(0, 2**32, size=(3, 8 * bits), dtype=np.uint64).astype(np.uint32)
    st = kv.packed_states(words, bits)
    L = kv._lib()
    for r in range(3):
        w = np.ascontiguousarray(words[r])
        for c in range(256):
            assert st[r, c] == L.orc_kv_packed_state(w.ctypes.data, bits, c)


@pytest.mark.parametrize("bits", [4, 5])
def test_row_decoder_matches_packed_state(bits):
    rng = np.random.default_rng(10 + bits)
    words = rng.integers(0, 2**32, size=(5, 8 * bits), dtype=np.uint64).astype(np.uint32)
    book = rng.integers(0, 2**16, size=256, dtype=np.uint64).astype(np.uint16) & np.uint16(0x7F7F)
    table = (book.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(kv.decode_packed_rows(words, bits, book), table[kv.packed_states(words, bits)])


def test_encoded_bases_decode_back():
    p = kv.parse_profile(kv.synthetic_profile(1, 1, 4))
    table = kv.base_table_bf16(p, 0)
    for x in kv.test_rows(7, 2):
        kind, _, words, _, bases, _, _ = kv.encode(p, 0, 3, x)
        assert kind == 4
        assert np.array_equal(kv.decode_packed_rows(words, 4, table)[0],
                              (bases.astype(np.uint32) << 16).view(np.float32))


def _softmax_reference(q, kb, ks, vb, vs, vmean):
    s = (kb.astype(np.float64) @ q.astype(np.float64)) * (ks.astype(np.float64) * 0.0625)
    e = np.exp(s - s.max())
    out = (e * vs) @ vb.astype(np.float64) / e.sum()
    return out + (vmean if vmean is not None else 0.0)


@pytest.mark.parametrize("length,splits", [(1, 31), (5, 31), (77, 31), (300, 42), (300, 7)])
def test_attend_head_is_softmax_attention(length, splits):
    rng = np.random.default_rng(length)
    q = rng.standard_normal(256).astype(np.float32)
    kb = rng.standard_normal((length, 256)).astype(np.float32)
    vb = rng.standard_normal((length, 256)).astype(np.float32)
    ks = rng.uniform(0.02, 0.2, length).astype(np.float32)
    vs = rng.uniform(0.01, 0.1, length).astype(np.float32)
    vmean = rng.standard_normal(256).astype(np.float32) * 0.1
    got = kv.attend_head(q, kb, ks, vb, vs, vmean, length, splits)
    ref = _softmax_reference(q, kb, ks, vb, vs, vmean)
    assert np.max(np.abs(got - ref)) <= 1e-2 * np.max(np.abs(ref))  # bf16 value weights


def test_inverse_rotation_is_orthogonal_up_to_scale():
    v = np.random.default_rng(3).standard_normal(256).astype(np.float32)
    r = kv.inverse_rotate(v)
    assert abs(np.linalg.norm(r) - np.linalg.norm(v)) < 1e-4 * np.linalg.norm(v)  # H256/16 is orthonormal


def test_length_76_attention_pins_absolute_tile_output_bits():
    """attention.rs:1244-1306: a query over 75 int8 prefix rows plus the self row; the 31
    splits of prefix_schedule(76) cross 32-key tile boundaries at absolute positions."""
    c = np.arange(256)
    query = (((c * 7) % 29).astype(np.float32) - np.float32(14.0)) * np.float32(0.03125)
    kb = np.stack([(((p * 13 + c * 7) % 255) - 127).astype(np.float32) for p in range(76)])
    vb = np.stack([(((p * 19 + (c % 16) * 11) % 255) - 127).astype(np.float32) for p in range(76)])
    ks = np.array([(p % 7 + 1) * 0.0078125 for p in range(76)], np.float32)
    vs = np.array([(p % 11 + 1) * 0.015625 for p in range(76)], np.float32)
    out = kv.attend_head(query, kb, ks, vb, vs, None, 76, 31)
    expected = [0xbede440b, 0xbeacaee9, 0x3ce1ab7d, 0xbdb714de, 0xbd938526, 0x3ef5474a, 0x3e3fbe6c, 0x3f4c2f7e,
                0x3f26e245, 0x3f811d5b, 0x3f09e0ce, 0x3f0e8ea2, 0xbde6e0e7, 0xbeb1494b, 0xbccde3de, 0xbf2b79d6]
    assert out.view(np.uint32).tolist() == expected * 16
