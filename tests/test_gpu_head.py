"""Greedy token and top-8 raw logits (yskn_b200_head_select) against the oracle of
docs/spec/06_OUTPUT_HEAD_SAMPLER.md: order (larger logit, smaller id) from (-FLT_MAX,
INT_MAX), exactly. Planted ties, NaN, -inf and +inf; and the head as the reference runs
it: the fused operator on a head matrix (no output rotation) with the row's inverse RMS,
then the selection, against the oracle's operator and selection.
"""
import numpy as np
import pytest

import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _select(logits):
    import torch
    import yskn_b200
    M = logits.shape[0]
    d = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    tok = torch.full((M,), -5, dtype=torch.int32, device="cuda")
    tv = torch.empty((M, 8), dtype=torch.float32, device="cuda")
    ti = torch.empty((M, 8), dtype=torch.int32, device="cuda")
    yskn_b200.head_select(d, tok, tv, ti)
    assert yskn_b200.status() == 0
    return tok.cpu().numpy(), tv.cpu().numpy(), ti.cpu().numpy()


def test_selection_order_ties_and_nonfinite(cuda):
    rng = np.random.default_rng(3)
    n = 151936
    logits = rng.standard_normal((5, n)).astype(np.float32)
    logits[0, [70000, 12, 151935]] = 9.0   # a three-way tie at the top: the smallest id wins
    logits[0, [5, 6]] = 8.5                # and a tie further down the top 8
    logits[1, 100] = np.nan
    logits[1, 200] = np.inf                # +inf beats everything
    logits[2, :] = -np.inf
    logits[2, [9, 4]] = -3.4028234663852886e38  # only -FLT_MAX entries are eligible: ids 4, 9
    logits[3, :] = np.nan                  # nothing eligible: (-FLT_MAX, INT_MAX) everywhere
    logits[4, ::2] = 0.0
    logits[4, 1::2] = -0.0
    tok, tv, ti = _select(logits)
    for m in range(logits.shape[0]):
        t, v, i = O.head_select(logits[m])
        assert tok[m] == t, m
        assert np.array_equal(tv[m].view(np.uint32), v.view(np.uint32)) or np.array_equal(tv[m], v), m
        assert np.array_equal(ti[m], i), m
    assert tok[0] == 12 and list(ti[0][:5]) == [12, 70000, 151935, 5, 6]
    assert tok[1] == 200 and tok[3] == 2**31 - 1 and list(ti[2][:2]) == [4, 9]


def test_head_operator_then_selection(cuda):
    import torch
    import yskn_b200
    vocab, hidden, M = 4096, 1024, 3
    words, lut16, sc16 = fixtures.model_matrix(vocab, hidden, 8, 77, vocab)
    si = O.signs("mulberry32_7919_13", 7, 0, hidden)
    dw = torch.from_numpy(words.view(np.int32)).cuda()
    head = yskn_b200.Matrix(dw, "warp", vocab, vocab, hidden, 8, lut16, sc16, si)  # no output rotation
    rng = np.random.default_rng(9)
    x = rng.standard_normal((M, hidden)).astype(np.float32)
    inv = np.array([0.7, 1.3, 0.9], np.float32)
    work = torch.empty(yskn_b200.linear_work_bytes([head], M), dtype=torch.uint8, device="cuda")
    logits = torch.empty((M, vocab), dtype=torch.float32, device="cuda")
    yskn_b200.linear([head], torch.from_numpy(x).cuda(), work, [logits], inv_rms=torch.from_numpy(inv).cuda())
    want_logits = np.asarray(O.linear(words, "warp", vocab, hidden, 8, lut16, sc16, x, si, None, inv_rms=inv),
                             np.float32)
    got = logits.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want_logits.view(np.uint32))
    tok, tv, ti = _select(got)
    for m in range(M):
        t, v, i = O.head_select(want_logits[m])
        assert tok[m] == t and np.array_equal(ti[m], i) and np.array_equal(tv[m], v)


@pytest.mark.parametrize("M,n", [(70, 3000), (2, 300), (64, 151936)])
def test_both_selection_levels_and_repeated_calls(cuda, M, n):
    """Up to 64 rows of at least 592 logits take the two-level selection (148 chunks per row,
    the last chunk's CTA merges); more rows or shorter rows take one CTA per row. Two calls
    in a row give the same result (the two-level arrival counters return to zero)."""
    rng = np.random.default_rng(M * 7 + n)
    logits = rng.standard_normal((M, n)).astype(np.float32)
    logits[:, rng.integers(0, n, 5)] = 2.5  # ties inside and across chunks
    first = _select(logits)
    second = _select(logits)
    for a, b in zip(first, second):
        assert np.array_equal(a, b)
    tok, tv, ti = first
    for m in range(M):
        t, v, i = O.head_select(logits[m])
        assert tok[m] == t and np.array_equal(ti[m], i) and np.array_equal(tv[m], v), m


@pytest.mark.parametrize("M,n", [(1, 151936), (5, 3000), (64, 151936), (2, 300)])
def test_greedy_token_alone_equals_the_oracle(cuda, M, n):
    """With no top-8 output requested, the selection takes one candidate per thread and one
    block-wide round per level; the token equals the oracle's over ties inside and across
    chunks, NaN and -inf logits, a row of only NaN, and two calls in a row."""
    import torch
    import yskn_b200
    rng = np.random.default_rng(M * 13 + n)
    logits = rng.standard_normal((M, n)).astype(np.float32)
    logits[:, rng.integers(0, n, 5)] = 3.25  # ties
    logits[0, : n // 3] = np.nan
    logits[-1, n // 2:] = -np.inf
    if M > 2:
        logits[1, :] = np.nan
    d = torch.from_numpy(logits).cuda()
    for _ in range(2):
        tok = torch.full((M,), -1, dtype=torch.int32, device="cuda")
        yskn_b200.head_select(d, token=tok)
        assert yskn_b200.status() == 0
        got = tok.cpu().numpy()
        for m in range(M):
            assert got[m] == O.head_select(logits[m])[0], m
