"""The tensor-parallel decode pass's split (yskn_b200/tp_stack.py TPPlan), host arithmetic only:
every head, row and column of the one-GPU pass is run by some rank, the ranks' parts of the
row-parallel inputs partition them, and each rank's local head mappings are the ones the
kernels compute (query head j reads local KV head j / (n_q / n_kv); value head h reads key
head h / 3 among the rank's query/key channels)."""
import pytest

pytest.importorskip("torch")

from yskn_b200 import stack as S  # noqa: E402
from yskn_b200.tp_stack import DK, QK, TPPlan  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_the_pass(world):
    plans = [TPPlan(r, world).check() for r in range(world)]
    # value heads and query heads: each exactly once, in rank order
    assert [h for p in plans for h in range(p.v0, p.v0 + p.n_v)] == list(range(48))
    assert [h for p in plans for h in range(p.h0, p.h0 + p.n_q)] == list(range(S.N_QH))
    # row-parallel inputs partition the columns; they match the heads
    for key, total in (("gdn_cols", S.ZDIM), ("attn_cols", S.N_QH * S.HEAD)):
        cols = [getattr(p, key) for p in plans]
        assert cols[0][0] == 0 and cols[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
        assert all(c0 % 512 == 0 and c1 % 512 == 0 for c0, c1 in cols)
    for p in plans:
        assert p.gdn_cols == (p.v0 * DK, (p.v0 + p.n_v) * DK)
        assert p.attn_cols == (p.h0 * S.HEAD, (p.h0 + p.n_q) * S.HEAD)
        # in_proj_qkv rows: whole 512-blocks of the query and key parts, then the value heads
        (q0, q1), (k0, k1), (v0, v1) = p.qkv_ranges
        assert q0 % 512 == 0 and q1 % 512 == 0 and (k0 - QK, k1 - QK) == (q0, q1) and q1 <= QK
        assert (v0, v1) == (2 * QK + p.v0 * DK, 2 * QK + (p.v0 + p.n_v) * DK)
        assert (p.qk0 * DK, p.qk0 * DK + p.qk_ch) == (q0, q1)
        for h in range(p.v0, p.v0 + p.n_v):  # the key head each value head reads is local
            assert p.qk0 <= h // 3 < p.qk0 + p.qk_ch // DK
        # KV heads: whole 512-blocks of k_proj / v_proj (two heads each) around the used ones
        r0, r1 = p.kv_rows
        assert r0 % 512 == 0 and r1 % 512 == 0 and r1 <= S.N_KVH * S.HEAD
        assert r0 // S.HEAD + p.kv_skip == p.kv0 and p.kv0 + p.n_kv <= r1 // S.HEAD
        for h in range(p.h0, p.h0 + p.n_q):
            assert p.kv0 <= h // (S.N_QH // S.N_KVH) < p.kv0 + p.n_kv
    # MLP rows / down columns and the vocabulary partition
    for key, total in (("ffn", S.FFN), ("vocab", S.VOCAB)):
        parts = [getattr(p, key) for p in plans]
        assert parts[0][0] == 0 and parts[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        assert all(a[0] % 512 == 0 for a in parts)
    assert all(p.vocab_ranges == plans[0].vocab_ranges for p in plans)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_plan_shards_are_whole_blocks(world):
    rows_cols = {"qkv": (S.QKV, S.HIDDEN), "z": (S.ZDIM, S.HIDDEN), "out": (S.HIDDEN, S.ZDIM),
                 "q": (S.N_QH * 2 * S.HEAD, S.HIDDEN), "k": (S.N_KVH * S.HEAD, S.HIDDEN),
                 "v": (S.N_KVH * S.HEAD, S.HIDDEN), "o": (S.HIDDEN, S.N_QH * S.HEAD), "gate": (S.FFN, S.HIDDEN),
                 "up": (S.FFN, S.HIDDEN), "down": (S.HIDDEN, S.FFN), "head": (S.VOCAB, S.HIDDEN)}
    for r in range(world):
        p = TPPlan(r, world)
        for role, (rows, cols) in rows_cols.items():
            sh = p.shard(role, rows, cols)
            if len(sh) == 3:
                ranges, c0, c1 = sh
            else:
                ranges, c0, c1 = [(sh[0], sh[1])], sh[2], sh[3]
            assert (c0, c1) == (0, cols) or (c0 % 512 == 0 and c1 % 512 == 0 and c1 <= cols)
            for r0, r1 in ranges:
                assert 0 <= r0 < r1 <= rows
                if role != "head":  # every rotated projection keeps whole 512-row blocks
                    assert r0 % 512 == 0 and r1 % 512 == 0
                else:
                    assert r0 % 8 == 0
