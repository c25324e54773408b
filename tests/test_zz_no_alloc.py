"""yskn_b200_weighted_sums_noalloc against yskn_b200_weighted_sums, through the C ABI.

The no-allocation entry point exists for callers that must not have the library
allocate device memory (a process whose HBM is already handed to its own pool, or a
latency-critical loop where cudaMalloc could synchronise the device). It keeps its
scratch in a static device array shared by every call on the device, so the test
makes three calls in a row (different shapes and inputs; the third is three launches)
and checks each against the regular entry point bit for bit (integer sums: the
tolerance is zero). This file is
collected last so that a run that stops at the first failure has run every other test.
"""
import numpy as np
import pytest

import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _matrices():
    import yskn_b200
    mats, keep = [], []
    for rows, phys, bits, seed in [(12288, 12288, 8, 31), (1024, 1024, 8, 32), (1000, 1024, 8, 33)]:
        words, lut16, sc16 = fixtures.model_matrix(rows, 5120, bits, seed, phys)
        dw = _dev(words.view(np.int32))
        keep.append(dw)
        mats.append(yskn_b200.Matrix(dw, "warp", rows, phys, 5120, bits, lut16, sc16,
                                     O.signs("mulberry32_7919_13", 7, 0, 5120)))
    return mats, keep


def test_noalloc_matches_the_regular_entry_point_on_two_calls(cuda):
    import torch
    import yskn_b200
    mats, _keep = _matrices()
    # M = 40 runs as three GEMV launches of 16, 16 and 8 rows that reuse the static array.
    for call, (M, group) in enumerate([(1, mats), (13, mats[:2]), (40, mats)]):
        rnd = fixtures.FixtureRandom(0xA110C + call)
        act = _dev(rnd.take(M * 5120).astype(np.uint8).view(np.int8).reshape(M, 5120))
        scales = _dev(rnd.take(M * 10).view(np.int32).reshape(M, 10))
        want = [torch.empty((M, m.physical_rows), dtype=torch.int64, device="cuda") for m in group]
        got = [torch.full((M, m.physical_rows), 7, dtype=torch.int64, device="cuda") for m in group]
        yskn_b200.weighted_sums(group, act, scales, want)
        yskn_b200.weighted_sums_noalloc(group, act, scales, got)
        torch.cuda.synchronize()
        for w, g in zip(want, got):
            assert torch.equal(w, g), "call %d differs" % call
    assert yskn_b200.status() == 0


def test_noalloc_rejects_sizes_beyond_its_static_scratch(cuda):
    import yskn_b200
    mats, _keep = _matrices()
    act = _dev(np.zeros((65, 5120), np.int8))
    scales = _dev(np.zeros((65, 10), np.int32))
    import torch
    out = [torch.empty((65, mats[0].physical_rows), dtype=torch.int64, device="cuda")]
    with pytest.raises(yskn_b200.YsknError) as e:
        yskn_b200.weighted_sums_noalloc(mats[:1], act, scales, out)
    assert e.value.code == yskn_b200.EINVAL and "M must be" in str(e.value)
