"""Parity of the CUDA path with the CPU oracle (bit-exact), through the C ABI.

Mirrors the reference's kernel tests (crates/yskn-engine/tests/linear.rs): every
bit width 4..8 x {row, warp} layout x shapes with padded physical rows x
M in {1, 2, 3, 8, 16, 17, 40}, extreme activations (+-127, 0), random signed i32
scales, prefix row counts, overflow as an error, and shape errors. Then the
quantiser and restore (bit-exact, the spec pins their binary32 op order) and the
whole operator at 27B shapes.
"""
import numpy as np
import pytest

import container
import fixtures
import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(17, 32, 512), (65, 96, 1024), (17, 32, 5120), (13, 16, 512), (9, 11, 512)]


def _dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda")


def _matrix(c, name="linear", signs_out=None):
    import yskn_b200
    d = c.tensors[name]
    words = _dev(c.words(name).view(np.int32))
    si = O.tensor_signs(d["rot_in"], d["cols"])
    m = yskn_b200.Matrix(words, d["layout"], d["rows"], d["physical_rows"], d["cols"], d["bits"], c.lut16(name),
                         c.scale16(name), si, signs_out)
    return m, words


def _inputs(cols, n, seed):
    rnd = fixtures.FixtureRandom(seed)
    act = rnd.take(n * cols).astype(np.uint8).view(np.int8).reshape(n, cols).copy()
    act[1 % n] = 127
    if n > 2:
        act[2] = -127
    if n > 3:
        act[3] = 0
    A = rnd.take(n * (cols // 512)).view(np.int32).reshape(n, -1).copy()
    return act, A


@pytest.mark.parametrize("bits", [4, 5, 6, 7, 8])
@pytest.mark.parametrize("layout", ["row", "warp"])
def test_weighted_sums_match_scalar_reference(cuda, bits, layout):
    import torch
    import yskn_b200
    for rows, phys, cols in SHAPES:
        if layout == "warp" and (phys * cols // 256) % 32:
            continue
        c = container.Container(fixtures.synthetic(bits, layout, rows, phys, cols, False))
        lut8, _ = O.quantize_weight_table(c.lut16("linear"), c.scale16("linear"))
        act, A = _inputs(cols, 40, 0xE79A170F88AB203D + bits)
        ref = O.fast_weighted_sums(c.words("linear"), layout, phys, cols, bits, lut8, act, A)
        if cols <= 1024:
            assert np.array_equal(ref, O.weighted_sums(c.words("linear"), layout, phys, cols, bits, lut8, act, A))
        m, _ = _matrix(c)
        da, dA = _dev(act), _dev(A)
        for M in [1, 2, 3, 8, 16, 17, 40]:
            out = torch.full((M, phys), -7, dtype=torch.int64, device="cuda")
            yskn_b200.weighted_sums([m], da[:M], dA[:M], [out])
            got = out.cpu().numpy()
            assert np.array_equal(got, ref[:M]), (bits, layout, rows, phys, cols, M)
            if M == 3:
                for n in sorted({1, rows, phys - 1}):
                    pre = torch.empty((M, n), dtype=torch.int64, device="cuda")
                    yskn_b200.weighted_sums_prefix(m, da[:M], dA[:M], n, pre)
                    assert np.array_equal(pre.cpu().numpy(), ref[:M, :n])
        assert yskn_b200.status() == 0
        m.close()


def test_grouped_matrices_share_one_input(cuda):
    """Up to three matrices in one launch (Engine35::gemv groups q/k/v, src/engine35.cpp:403-430)."""
    import torch
    import yskn_b200
    specs = [(300, 320, 1024, 6, 11), (64, 96, 1024, 6, 12), (512, 512, 1024, 6, 13)]
    mats, refs, keep = [], [], []
    act, A = _inputs(1024, 5, 99)
    for rows, phys, cols, bits, seed in specs:
        words, lut16, sc16 = fixtures.model_matrix(rows, cols, bits, seed, phys)
        lut8, _ = O.quantize_weight_table(lut16, sc16)
        refs.append(O.fast_weighted_sums(words, "warp", phys, cols, bits, lut8, act, A))
        dw = _dev(words.view(np.int32))
        keep.append(dw)
        mats.append(yskn_b200.Matrix(dw, "warp", rows, phys, cols, bits, lut16, sc16, np.ones(cols, np.int8)))
    for M in (1, 5):
        outs = [torch.empty((M, s[1]), dtype=torch.int64, device="cuda") for s in specs]
        yskn_b200.weighted_sums(mats, _dev(act[:M]), _dev(A[:M]), outs)
        for o, r in zip(outs, refs):
            assert np.array_equal(o.cpu().numpy(), r[:M])


def test_quantize_is_bit_exact(cuda):
    import torch
    import yskn_b200
    for M, K, seed in [(1, 5120, 1), (3, 512, 2), (17, 17408, 3), (2, 6144, 4)]:
        x = fixtures.normal(seed, M * K).reshape(M, K) * np.float32(3.0)
        x[0, :512] = 0.0  # an all-zero group
        si = O.signs("mulberry32_7919_13", 7, 0, K)
        ra, ral, rA, rq = O.quantize_activation(x, si)
        dsi = _dev(si)
        act = torch.empty((M, K), dtype=torch.int8, device="cuda")
        alpha = torch.empty((M, K // 512), dtype=torch.float32, device="cuda")
        A = torch.empty((M, K // 512), dtype=torch.int32, device="cuda")
        rqd = torch.empty(M, dtype=torch.float32, device="cuda")
        yskn_b200.quantize(_dev(x), dsi.data_ptr(), act, alpha, A, rqd)
        assert np.array_equal(act.cpu().numpy(), ra)
        assert np.array_equal(alpha.cpu().numpy().view(np.uint32), ral.view(np.uint32))
        assert np.array_equal(A.cpu().numpy(), rA)
        assert np.array_equal(rqd.cpu().numpy().view(np.uint32), rq.view(np.uint32))
        assert yskn_b200.status() == 0


def test_quantize_reports_non_finite(cuda):
    import torch
    import yskn_b200
    x = np.zeros((1, 1024), np.float32)
    x[0, 5] = np.inf
    act = torch.empty((1, 1024), dtype=torch.int8, device="cuda")
    f = torch.empty((1, 2), dtype=torch.float32, device="cuda")
    A = torch.empty((1, 2), dtype=torch.int32, device="cuda")
    rq = torch.empty(1, dtype=torch.float32, device="cuda")
    yskn_b200.quantize(_dev(x), _dev(np.ones(1024, np.int8)).data_ptr(), act, f, A, rq)
    assert yskn_b200.status() == yskn_b200.ENONFINITE
    assert yskn_b200.status() == 0


@pytest.mark.parametrize("rotate", [True, False])
def test_restore_is_bit_exact(cuda, rotate):
    import torch
    import yskn_b200
    rows, phys, cols, bits = 1000, 1024, 512, 8
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, bits, 41, phys)
    so = O.signs("mulberry32_7919_13", 7, cols, phys) if rotate else None
    dw = _dev(words.view(np.int32))
    m = yskn_b200.Matrix(dw, "warp", rows, phys, cols, bits, lut16, sc16, np.ones(cols, np.int8), so)
    _, tau = O.quantize_weight_table(lut16, sc16)
    rnd = fixtures.FixtureRandom(5)
    M = 3
    ws = (rnd.take(M * phys).view(np.int32).astype(np.int64) * 4099).reshape(M, phys)
    rq = np.float32([2.0 ** -30, 3.1e-9, 1.7e-10])
    for inv_rms in (None, np.float32([0.5, 1.25, 3.0])):
        ref = O.restore(ws, rq, tau, so, inv_rms, rows)
        dws = _dev(ws)
        y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
        yskn_b200.restore(dws, _dev(rq), None if inv_rms is None else _dev(inv_rms), m, rotate, rows, True, y)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        assert not dws.any().item()  # consumed accumulators are cleared


@pytest.mark.parametrize("bits", [6, 8])
def test_linear_27b_shape_matches_oracle(cuda, bits):
    """y = W x end to end (CompressedLinear::project) at gate_proj's shape, bit-exact."""
    import torch
    import yskn_b200
    rows, cols = 17408, 5120
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, bits, 1000 + bits)
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    so = O.signs("mulberry32_7919_13", 7, cols, rows)
    dw = _dev(words.view(np.int32))
    m = yskn_b200.Matrix(dw, "warp", rows, rows, cols, bits, lut16, sc16, si, so)
    for M in (1, 8):
        x = fixtures.normal(77 + M, M * cols).reshape(M, cols)
        lut8, tau = O.quantize_weight_table(lut16, sc16)
        act, _, A, rq = O.quantize_activation(x, si)
        ws = O.fast_weighted_sums(words, "warp", rows, cols, bits, lut8, act, A)
        ref = O.restore(ws, rq, tau, so)
        work = torch.empty(yskn_b200.linear_work_bytes([m], M), dtype=torch.uint8, device="cuda")
        y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
        yskn_b200.linear([m], _dev(x), work, [y])
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        assert yskn_b200.status() == 0


@pytest.mark.parametrize("M,cols", [(1, 2048), (3, 2048), (16, 2048), (17, 2048), (8, 17408), (64, 2048),
                                    (130, 1024)])
def test_linear_fused_and_staged_paths(cuda, M, cols):
    """Three matrices sharing one input, two with an output rotation and one without
    (rows < physical rows), with 1/rms, bit-exact. M <= 16 with the activations in
    shared memory runs the one-launch fused operator; M = 17 and (8, 17408) run the
    staged quantise / sums / restore launches; M >= 64 puts the tcgen05 GEMM between
    the quantiser and the restore. Twice in a row, so the per-block counters of the
    fused restore are seen to reset."""
    import torch
    import yskn_b200
    specs = [(1024, 1024, True), (512, 512, True), (300, 304, False)]
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    mats, keep, refs = [], [], []
    x = fixtures.normal(900 + M, M * cols).reshape(M, cols)
    inv_rms = (1.0 + 0.01 * np.arange(M)).astype(np.float32)
    for i, (rows, phys, rot) in enumerate(specs):
        words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, 500 + i, physical_rows=phys)
        so = O.signs("mulberry32_7919_13", 7, cols + 4096 * i, phys) if rot else None
        dw = _dev(words.view(np.int32))
        mats.append(yskn_b200.Matrix(dw, "warp", rows, phys, cols, 8, lut16, sc16, si, so))
        keep.append(dw)
        refs.append(O.linear(words, "warp", phys, cols, 8, lut16, sc16, x, si, so, inv_rms, rows))
    work = torch.empty(yskn_b200.linear_work_bytes(mats, M), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        ys = [torch.full((M, r), float("nan"), dtype=torch.float32, device="cuda") for r, _, _ in specs]
        yskn_b200.linear(mats, _dev(x), work, ys, inv_rms=_dev(inv_rms))
        for y, ref in zip(ys, refs):
            assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        assert yskn_b200.status() == 0


def test_overflow_is_an_error_and_the_library_recovers(cuda):
    """crates/yskn-engine/tests/linear.rs:277-308."""
    import torch
    import yskn_b200
    cols, rows, bits = 264704, 96, 6
    words = (fixtures.stream64(5, rows * (cols // 256) * 4 * bits) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    lut16 = np.full(8192, 0x3C00, np.uint16)  # every table value 1.0 -> int8 127
    sc16 = np.full(rows, 0x3C00, np.uint16)
    dw = _dev(words.view(np.int32))
    m = yskn_b200.Matrix(dw, "row", rows, rows, cols, bits, lut16, sc16, np.ones(cols, np.int8))
    A = _dev(np.full((1, cols // 512), np.iinfo(np.int32).min, np.int32))
    out = torch.empty((1, rows), dtype=torch.int64, device="cuda")
    with pytest.raises(yskn_b200.YsknError) as e:
        yskn_b200.weighted_sums([m], _dev(np.full((1, cols), -128, np.int8)), A, [out])
    assert e.value.code == yskn_b200.EOVERFLOW
    yskn_b200.weighted_sums([m], _dev(np.zeros((1, cols), np.int8)), A, [out])
    assert not out.any().item()


def test_repack_is_identical_to_the_reference_permutation(cuda):
    import torch
    import yskn_b200
    for rows, seqs, bits in [(64, 2, 6), (128, 20, 8), (192, 4, 4)]:
        wps = 4 * bits
        words = (fixtures.stream64(rows + seqs, rows * seqs * wps) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        ref = O.repack_warp_to_frag(words, rows, seqs, wps)
        dw = _dev(words.view(np.int32))
        df = torch.empty_like(dw)
        assert yskn_b200.repack_warp_to_frag(dw, df, rows, seqs, wps) == 0
        torch.cuda.synchronize()
        assert np.array_equal(df.cpu().numpy().view(np.uint32), ref)
        host = np.empty_like(words)
        assert yskn_b200.lib().yskn_repack_warp_to_frag_host(words.ctypes.data, host.ctypes.data, rows, seqs, wps) == 0
        assert np.array_equal(host, ref)
