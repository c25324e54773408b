"""Matrices loaded from `.yskn` files (yskn_b200_file_load_matrix[_shard]) on the GPU.

A matrix the library builds from a file must be the matrix built from the same
tensor's arrays through yskn_b200_matrix_create (the path the other GPU tests pin to
the oracle): identical weighted sums and identical fused-operator outputs, bit for
bit, for every non-embedding tensor of the reference's tiny.yskn (bits 6 and 8,
both sign rules) and of the kernel-test containers (row layout, padded physical rows,
an output rotation), whole and as tensor-parallel shards. One tensor is also checked
against the oracle's integer sums directly.
"""
import numpy as np
import pytest

import container
import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _created(c, name, shard=None):
    import yskn_b200
    d = c.tensors[name]
    words = _dev(c.words(name).view(np.int32))
    m = yskn_b200.Matrix(words, d["layout"], d["rows"], d["physical_rows"], d["cols"], d["bits"], c.lut16(name),
                         c.scale16(name), O.tensor_signs(d["rot_in"], d["cols"]),
                         O.tensor_signs(d["rot_out"], d["physical_rows"]), shard=shard)
    return m, words


def _inputs(cols, M, seed):
    rnd = fixtures.FixtureRandom(seed)
    act = rnd.take(M * cols).astype(np.uint8).view(np.int8).reshape(M, cols).copy()
    A = rnd.take(M * (cols // 512)).view(np.int32).reshape(M, -1).copy()
    x = (rnd.take(M * cols) % 4001).astype(np.float32).reshape(M, cols) / np.float32(1000.0) - np.float32(2.0)
    return act, A, x


def _sums(m, act, A):
    import torch
    import yskn_b200
    out = torch.full((act.shape[0], m.physical_rows), -7, dtype=torch.int64, device="cuda")
    yskn_b200.weighted_sums([m], _dev(act), _dev(A), [out])
    return out.cpu().numpy()


def _linear(m, x):
    import torch
    import yskn_b200
    M = x.shape[0]
    work = torch.empty(yskn_b200.linear_work_bytes([m], M), dtype=torch.uint8, device="cuda")
    y = torch.full((M, m.rows), float("nan"), dtype=torch.float32, device="cuda")
    yskn_b200.linear([m], _dev(x), work, [y])
    return y.cpu().numpy()


FILES = [
    ("tiny", fixtures.tiny_container),
    ("row6", lambda: fixtures.synthetic(6, "row", 65, 96, 1024, False)),
    ("warp8", lambda: fixtures.synthetic(8, "warp", 1024, 1024, 1024, True)),
    ("warp5", lambda: fixtures.synthetic(5, "warp", 17, 32, 5120, False)),
]


@pytest.mark.parametrize("label,make", FILES, ids=[f[0] for f in FILES])
def test_file_matrices_equal_created_matrices(cuda, tmp_path, label, make):
    import yskn_b200
    data = make()
    path = tmp_path / (label + ".yskn")
    path.write_bytes(data)
    c = container.Container(data)
    f = yskn_b200.File(str(path))
    checked = 0
    for name, d in c.tensors.items():
        if d["role"] == "embedding":
            continue
        got = f.load_matrix(name)
        want, _keep = _created(c, name)
        assert got.info() == want.info(), name
        for M in (1, 3):
            act, A, x = _inputs(d["cols"], M, 0x5EED + M + checked)
            assert np.array_equal(_sums(got, act, A), _sums(want, act, A)), (label, name, M)
            # The fused operator also reads the handle's row scales and both sign streams.
            assert np.array_equal(_linear(got, x).view(np.uint32), _linear(want, x).view(np.uint32)), (label, name)
        got.close()
        want.close()
        checked += 1
    assert checked > 0
    assert yskn_b200.status() == 0
    f.close()


def test_file_matrix_sums_equal_the_oracle(cuda, tmp_path):
    import yskn_b200
    data = fixtures.tiny_container()
    path = tmp_path / "tiny.yskn"
    path.write_bytes(data)
    c = container.Container(data)
    name = "tiny.body8"
    d = c.tensors[name]
    m = yskn_b200.File(str(path)).load_matrix(name)
    lut8, _ = O.quantize_weight_table(c.lut16(name), c.scale16(name))
    act, A, _ = _inputs(d["cols"], 5, 77)
    ref = O.weighted_sums(c.words(name), d["layout"], d["physical_rows"], d["cols"], d["bits"], lut8, act, A)
    assert np.array_equal(_sums(m, act, A), ref)


def test_file_shards_equal_created_shards(cuda, tmp_path):
    import yskn_b200
    data = fixtures.synthetic(8, "warp", 1024, 1024, 1024, True)
    path = tmp_path / "warp8.yskn"
    path.write_bytes(data)
    c = container.Container(data)
    f = yskn_b200.File(str(path))
    for shard in [(0, 512, 0, 1024), (512, 1024, 0, 1024), (0, 1024, 512, 1024)]:
        got = f.load_matrix("linear", shard=shard)
        want, _keep = _created(c, "linear", shard=shard)
        act, A, _ = _inputs(got.cols, 3, 0xA11 + shard[0] + shard[2])
        assert np.array_equal(_sums(got, act, A), _sums(want, act, A)), shard
    with pytest.raises(yskn_b200.YsknError):
        f.load_matrix("linear", shard=(0, 500, 0, 1024))  # not whole 512-row blocks with a rotation
