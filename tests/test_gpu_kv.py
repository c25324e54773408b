"""Quantised-KV decode attention (packed 4-bit rows) through the C ABI against the oracle.

The oracle (oracle/kv_oracle.c orc_kv_attend_head, restating crates/yskn-ref/src/
attention.rs with the portable exp2/exp; pinned to the 256 output bits of
attention.rs:1244-1306) reproduces yskn-ref's order. The CUDA kernel sums scores and
values on the tensor cores in their own order (the spec leaves the MMA's internal order
open, ATT-01) with the hardware exp2 inside the key loop; its split combine and output
gate use the portable exp and sigmoid. Value weights are rounded to BF16
(attention.rs), so one weight whose rounding flips moves the output by up to 2^-8 of
that key's share.
Tolerances, written here:
  attended (f32, before the inverse rotation): max |gpu - oracle| <= 5e-3 * max |oracle|,
      mean |gpu - oracle| <= 2e-4 * max |oracle|;
  out (bf16, after rotation and gate): |gpu - oracle| <= 2^-7 |oracle| + 8e-3 * max |oracle|.
"""
import numpy as np
import pytest

import kv
import oracle as O

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_float(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def make_cache(rng, n_kvh, capacity):
    words = rng.integers(0, 2**32, size=(2, n_kvh, capacity, 32), dtype=np.uint64).astype(np.uint32)
    ks = rng.uniform(0.02, 0.2, (n_kvh, capacity)).astype(np.float32)
    vs = rng.uniform(0.01, 0.1, (n_kvh, capacity)).astype(np.float32)
    books = bf16_bits(rng.standard_normal((2, n_kvh, 256)) * 2.0)
    return words, ks, vs, books


def oracle_case(q_bits, gate_bits, words, ks, vs, books, vmean, M, n_qh, n_kvh, length, n_splits):
    G = n_qh // n_kvh
    att = np.zeros((M, n_qh, 256), np.float32)
    out = np.zeros((M, n_qh, 256), np.float32)
    dec = [(kv.decode_packed_rows(words[0, h, :length], 4, books[0, h]),
            kv.decode_packed_rows(words[1, h, :length], 4, books[1, h])) for h in range(n_kvh)]
    for m in range(M):
        L = length - M + 1 + m
        splits = n_splits or (31 if L < 4096 else 42)
        for j in range(n_qh):
            h = j // G
            a = kv.attend_head(bf16_float(q_bits[m, j]), dec[h][0][:L], ks[h, :L], dec[h][1][:L], vs[h, :L],
                               None if vmean is None else vmean[h], L, splits)
            att[m, j] = a
            r = bf16_float(bf16_bits(kv.inverse_rotate(a)))
            if gate_bits is not None:
                g = bf16_float(gate_bits[m, j])
                sg = bf16_float(bf16_bits(O.pm("sigmoid", g)))  # attention.rs:505-514
                r = bf16_float(bf16_bits(r * sg))
            out[m, j] = r
    return att, out


def run_case(cuda, M, n_qh, n_kvh, length, capacity, n_splits=0, gate=True, mean=True, seed=0, codebook=None,
             oracle_splits=None):
    import torch
    import yskn_b200
    rng = np.random.default_rng(seed)
    words, ks, vs, books = make_cache(rng, n_kvh, capacity)
    if codebook is not None:
        books[:] = codebook
    q = bf16_bits(rng.standard_normal((M, n_qh, 256)))
    g = bf16_bits(rng.standard_normal((M, n_qh, 256)) * 2.0) if gate else None
    vmean = (rng.standard_normal((n_kvh, 256)) * 0.05).astype(np.float32) if mean else None
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int32 if a.dtype == np.uint32 else  # noqa: E731
                                                                 np.int16 if a.dtype == np.uint16 else a.dtype)).to(cuda)
    work = torch.empty(yskn_b200.kv4_attention_work_bytes(M, n_qh, length, n_splits), dtype=torch.uint8, device=cuda)
    att = torch.empty((M, n_qh, 256), dtype=torch.float32, device=cuda)
    out = torch.empty((M, n_qh, 256), dtype=torch.int16, device=cuda)
    yskn_b200.kv4_attention(dev(q), dev(words[0]), dev(ks), dev(words[1]), dev(vs), dev(books[0]), dev(books[1]),
                            length, work, out, gate=None if g is None else dev(g),
                            v_mean=None if vmean is None else dev(vmean), attended=att, n_splits=n_splits)
    torch.cuda.synchronize()
    got_att = att.cpu().numpy()
    got_out = bf16_float(out.cpu().numpy().view(np.uint16))
    exp_att, exp_out = oracle_case(q, g, words, ks, vs, books, vmean, M, n_qh, n_kvh, length,
                                   n_splits if oracle_splits is None else oracle_splits)
    scale = np.max(np.abs(exp_att))
    err = np.abs(got_att - exp_att)
    assert np.all(np.isfinite(got_att))
    assert err.max() <= 5e-3 * scale, (err.max(), scale)
    assert err.mean() <= 2e-4 * scale, (err.mean(), scale)
    oscale = np.max(np.abs(exp_out))
    assert np.all(np.abs(got_out - exp_out) <= 2.0**-7 * np.abs(exp_out) + 8e-3 * oscale)


@pytest.mark.parametrize("length", [1, 2, 5, 33, 64, 65, 2048])
def test_decode_lengths(cuda, length):
    run_case(cuda, 1, 24, 4, length, length + 40, seed=length)


def test_split_count_switch_4096(cuda):
    run_case(cuda, 1, 24, 4, 4096, 4096, gate=False, mean=False, seed=11)


def test_rows_straddling_the_split_switch(cuda):
    run_case(cuda, 8, 24, 4, 4100, 4200, seed=12)  # rows see 4093..4100: 31 then 42 splits


@pytest.mark.parametrize("n_qh,n_kvh,splits", [(8, 1, 64), (4, 4, 0), (6, 1, 1), (16, 2, 37)])
def test_head_groups_and_fixed_splits(cuda, n_qh, n_kvh, splits):
    run_case(cuda, 2, n_qh, n_kvh, 300, 333, n_splits=splits, seed=n_qh * 7 + splits)


def test_profile_codebook(cuda):
    p = kv.parse_profile(kv.synthetic_profile(1, 1, 4))
    run_case(cuda, 1, 6, 1, 700, 700, codebook=kv.base_table_bf16(p, 0), seed=5)


def test_full_context_32k(cuda):
    run_case(cuda, 1, 24, 4, 32768, 32768, seed=32)



@pytest.mark.parametrize("length", [65, 4097, 32768])
def test_one_wave_splits_against_the_reference_schedule(cuda, length):
    """The decode pass launches with n_splits = -1 (as many splits as fill one wave of
    CTAs); the oracle keeps the reference's schedule (31 splits below 4096 rows, else 42,
    attention.rs:207-232), so this is the deviation of the shipped configuration from
    yskn-ref itself, within the same tolerance."""
    run_case(cuda, 1, 24, 4, length, length, n_splits=-1, seed=40 + length % 7, oracle_splits=0)
