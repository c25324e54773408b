"""Quantised-KV row encoder (packed trellis rows) through the C ABI, bit-exact against
the oracle's encode_packed (oracle/kv_oracle.c, pinned by the reference's frozen
codec hashes): words and scales of every row, for the compressed (vit2) and the
general Viterbi recurrence at 4 and 5 bits, with and without group means, rows
scattered into a cache through destination indices, and an i32 overflow reported as
an error (the reference's Err)."""
import struct

import numpy as np
import pytest

import kv

pytestmark = pytest.mark.gpu


def profile(bits, general=False, means=()):
    b = kv.test_profile(2, 4, bits)  # 2 layers x 4 KV heads x 2 sides, multipliers 0.9 / 1.0 / 1.1
    if general:  # codes beyond +-1100 make the profile ineligible for the compressed recurrence
        to = struct.unpack_from("<I", b, 112)[0]
        for s in range(256):
            struct.pack_into("<h", b, to + 12 + 2 * s, ((s * 97 + 5) % 4001) - 2000)
    for g in means:
        kv.replace_group(b, g, 0, 0, 0, True)
    return kv.parse_profile(b)


def device_profile(p, cuda):
    import torch
    ng = len(p.groups)
    tables = np.stack([p.tables[g["table"]][1] for g in p.groups]).astype(np.int16)
    gains = np.array([p.tables[g["table"]][0] for g in p.groups], np.float32)
    means = np.stack([g["mean"] if g["mean"] is not None else np.zeros(256, np.float32) for g in p.groups])
    has = np.array([g["mean"] is not None for g in p.groups], np.uint8)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    return t(tables), t(gains), t(means.astype(np.float32)), t(has), t(p.mults.astype(np.float32)), ng


def run(cuda, p, rows, groups, dest=None, capacity=None):
    import torch
    import yskn_b200
    kb = kv.packed_bits(p)
    tables, gains, means, has, mults, _ = device_profile(p, cuda)
    n = len(rows)
    cap = capacity or n
    words = torch.zeros((cap, 8 * kb), dtype=torch.int32, device=cuda)
    scales = torch.zeros(cap, dtype=torch.float32, device=cuda)
    d = None if dest is None else torch.from_numpy(np.asarray(dest, np.int64)).to(cuda)
    yskn_b200.kv_encode(torch.from_numpy(np.stack(rows).astype(np.float32)).to(cuda),
                        torch.from_numpy(np.asarray(groups, np.int32)).to(cuda), tables, gains, mults, kb,
                        kv.vit2_eligible(p), words, scales, means=means, has_mean=has, dest=d)
    torch.cuda.synchronize()
    return words.cpu().numpy().view(np.uint32), scales.cpu().numpy(), yskn_b200.status()


def rows_for(seed, n):
    rng = np.random.default_rng(seed)
    return [(rng.standard_normal(256) * rng.uniform(0.1, 3.0)).astype(np.float32) for _ in range(n)]


@pytest.mark.parametrize("bits", [4, 5])
@pytest.mark.parametrize("general", [False, True])
def test_encode_matches_oracle(cuda, bits, general):
    p = profile(bits, general, means=(1, 6, 9))
    assert kv.vit2_eligible(p) == (not general)
    rows = rows_for(bits * 10 + general, 48) + kv.test_rows(0x05a0c0de, 4)
    groups = [i % len(p.groups) for i in range(len(rows))]
    words, scales, status = run(cuda, p, rows, groups)
    assert status == 0
    for i, (x, g) in enumerate(zip(rows, groups)):
        kind, scale, w, *_ = kv.encode(p, g, 5, x)
        assert kind == bits
        assert np.array_equal(words[i], w), i
        assert scales[i].view(np.uint32) == np.float32(scale).view(np.uint32), i


def test_encode_scatters_into_a_cache(cuda):
    p = profile(4, means=(0,))
    rows = rows_for(3, 8)
    groups = [0, 2, 4, 6, 1, 3, 5, 7]  # one token: 4 heads x K, V of layer 0
    dest = [h * 100 + 37 for h in range(8)]  # [head-side][capacity 100] at position 37
    words, scales, status = run(cuda, p, rows, groups, dest=dest, capacity=800)
    assert status == 0
    written = set(dest)
    for r in range(800):
        if r not in written:
            assert not words[r].any() and scales[r] == 0.0
    for i, (x, g) in enumerate(zip(rows, groups)):
        _, scale, w, *_ = kv.encode(p, g, 37, x)
        assert np.array_equal(words[dest[i]], w) and scales[dest[i]] == np.float32(scale)


def test_encode_overflow_is_an_error(cuda):
    import yskn_b200
    b = kv.test_profile(1, 1, 4)
    to = struct.unpack_from("<I", b, 112)[0]
    for s in range(256):
        struct.pack_into("<h", b, to + 12 + 2 * s, 32767 if s % 2 else -32768)
    p = kv.parse_profile(b)
    x = rows_for(9, 1)
    with pytest.raises(Exception):
        kv.encode(p, 0, 0, x[0])  # the oracle (like the reference) rejects the row
    _, _, status = run(cuda, p, x, [0])
    assert status == yskn_b200.ENONFINITE
    assert yskn_b200.status() == 0  # reported once, then clear
