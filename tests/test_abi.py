"""The C ABI library loads and exports every symbol include/yskn_b200.h declares
(no GPU needed: only host-side entry points are called here)."""
import os
import re

import numpy as np
import pytest

import oracle as O
from conftest import ROOT


def _declared():
    names = set()
    with open(os.path.join(ROOT, "include", "yskn_b200.h")) as f:
        text = f.read()
    for m in re.finditer(r"YSKN_B200_API\s+[^;{]*?\b(yskn_\w+)\s*\(", text):
        names.add(m.group(1))
    return names


def test_header_declares_the_reference_repack_exports():
    names = _declared()
    assert {"yskn_repack_warp_to_frag", "yskn_repack_warp_to_frag_host"} <= names
    assert "yskn_b200_weighted_sums" in names and "yskn_b200_last_error" in names


def test_library_exports_every_declared_symbol():
    import yskn_b200
    L = yskn_b200.lib()
    declared = _declared()
    for name in declared:
        assert hasattr(L, name), name
    assert declared == set(yskn_b200.exported_symbols())


@pytest.mark.parametrize("rule", ["splitmix64", "mulberry32_7919_13"])
def test_host_sign_streams_match_the_oracle(rule):
    import yskn_b200
    for seed, offset, n in [(7, 0, 5120), (11, 1024, 512), (0, 3, 64), (2 ** 40 + 5, 2 ** 33, 1000)]:
        assert np.array_equal(yskn_b200.signs(rule, seed, offset, n), O.signs(rule, seed, offset, n))


def test_shape_errors_are_returned_not_trapped():
    import yskn_b200
    L = yskn_b200.lib()
    assert L.yskn_b200_pack_bytes(17408, 5120, 8) == 17408 * 20 * 8 * 16
    assert L.yskn_b200_pack_bytes(13, 512, 6) == 16 * 2 * 6 * 16
    assert L.yskn_b200_pack_bytes(16, 500, 8) == -1
    assert L.yskn_b200_pack_bytes(16, 512, 9) == -1
    # The reference's repack rejects rows % 64 and wps % 4 with -1 before touching memory.
    assert L.yskn_repack_warp_to_frag(None, None, 65, 2, 32, None) == -1
    assert L.yskn_repack_warp_to_frag(None, None, 64, 2, 30, None) == -1
    lut = np.zeros(8192, np.uint16)
    sc = np.zeros(16, np.uint16)
    si = np.ones(512, np.int8)
    for args in [(1, 13, 16, 500, 8), (1, 13, 16, 512, 3), (1, 17, 16, 512, 8), (1, 13, 11, 512, 8)]:
        layout, rows, phys, cols, bits = args
        h = L.yskn_b200_matrix_create(None, layout, rows, phys, cols, bits, lut.ctypes.data, sc.ctypes.data,
                                      si.ctypes.data, None)
        assert not h
        assert yskn_b200.last_error()


def test_kv_attention_argument_errors_are_returned():
    import yskn_b200
    L = yskn_b200.lib()
    call = lambda M, nq, nk, length, cap, kb, splits: L.yskn_b200_kv4_attention(  # noqa: E731
        *([None] * 9), M, nq, nk, length, cap, kb, splits, None, None, None, None)
    assert call(1, 24, 4, 10, 10, 5, 0) == yskn_b200.EINVAL  # kb 5 rows are not supported by this kernel
    assert call(1, 24, 5, 10, 10, 4, 0) == yskn_b200.EINVAL  # heads not a multiple
    assert call(1, 36, 4, 10, 10, 4, 0) == yskn_b200.EINVAL  # more than 8 query heads per KV head
    assert call(1, 24, 4, 11, 10, 4, 0) == yskn_b200.EINVAL  # length beyond capacity
    assert call(4, 24, 4, 3, 10, 4, 0) == yskn_b200.EINVAL  # more query rows than cache rows
    assert call(1, 24, 4, 10, 10, 4, 65) == yskn_b200.EINVAL
    assert call(1, 24, 4, 10, 10, 4, 0) == yskn_b200.EINVAL  # null buffers
    assert L.yskn_b200_kv4_attention_work_bytes(1, 24, 2048, 0) == 24 * 31 * 260 * 4
    assert L.yskn_b200_kv4_attention_work_bytes(8, 24, 4100, 0) == 8 * 24 * 42 * 260 * 4
    assert L.yskn_b200_kv4_attention_work_bytes(1, 24, 100, 65) == -1


def test_layer_op_argument_errors_are_returned():
    """The layer ops between operators reject bad shapes and commit counts with EINVAL and a
    message before any device work (fake, never dereferenced pointers)."""
    import yskn_b200
    L = yskn_b200.lib()
    p = 4096  # stands for a device pointer; 16-byte aligned
    EINVAL = yskn_b200.EINVAL
    cases = [
        L.yskn_b200_residual_prepare(p, None, p, 1, 500, 1e-6, p, p, None, None),      # cols % 512
        L.yskn_b200_residual_prepare(p, None, p, 0, 512, 1e-6, p, p, None, None),      # M < 1
        L.yskn_b200_gated_product(p, p, 0, 16, p, None),                               # M < 1
        L.yskn_b200_head_select(p, 1, 16, None, None, None, None),                     # no output
        L.yskn_b200_attention_prep(p, p, p, p, p, p, 1e-6, 0, 24, 4, p, p, p, p, None),  # M < 1
        L.yskn_b200_gdn_gates(p, p, p, p, 1, 1000, p, None),                           # hidden % 1024
        L.yskn_b200_gdn_gates(p + 2, p, p, p, 1, 1024, p, None),                       # unaligned rows
        L.yskn_b200_gdn_step(p, p, p, p, p, p, p, 1e-6, 2, 3, p, p, p, None),          # n_commit > M
        L.yskn_b200_gdn_step(p, p, p, p, p, p, p, 1e-6, 2, -1, p, p, p, None),         # n_commit < 0
        L.yskn_b200_widen_bf16(p, 0, p, None),                                         # n < 1
    ]
    for i, rc in enumerate(cases):
        assert rc == EINVAL, i
    assert yskn_b200.last_error()
