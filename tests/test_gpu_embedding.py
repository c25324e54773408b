"""Coded embedding rows on the GPU (yskn_b200_embedding_* through the C ABI) against the
oracle, bit for bit (bf16 bits): the reference's tiny.yskn embedding read from the file,
and a main table with one and two residual tables of other bit widths (from a file and
from arrays), repeated and edge token ids, and an out-of-range id (a zero row and
YSKN_EINVAL from the status call, no fault).
"""
import numpy as np
import pytest

import container
import fixtures
import oracle as O

pytestmark = pytest.mark.gpu

MAIN_ROT = ("mulberry32_7919_13", 7, 0)
PARTS = [("emb", 6, 101, MAIN_ROT), ("emb.res", 4, 202, ("splitmix64", 9, 0)), ("emb.res2", 8, 303, MAIN_ROT)]


def _lookup(e, tokens):
    import torch
    t = torch.tensor(tokens, dtype=torch.int32, device="cuda")
    out = torch.full((len(tokens), e.cols), -1, dtype=torch.int16, device="cuda")
    e.lookup(t, out)
    return out.cpu().numpy().view(np.uint16)


def _oracle(c, names, tokens):
    parts = []
    for n in names:
        d = c.tensors[n]
        parts.append((c.words(n), d["layout"], d["physical_rows"], d["cols"], d["bits"], c.lut16(n), c.scale16(n)))
    main = c.tensors[names[0]]
    # The main table's signs for every part (docs/spec/02_COMPRESSED_LINEAR.md:305-312).
    return O.embedding_rows(parts, tokens, O.tensor_signs(main["rot_in"], main["cols"]))


def test_tiny_embedding_from_the_file(cuda, tmp_path):
    import yskn_b200
    data = fixtures.tiny_container()
    path = tmp_path / "tiny.yskn"
    path.write_bytes(data)
    e = yskn_b200.File(str(path)).load_embedding("tiny.embed")
    tokens = [0, 5, 42, 95, 5, 17]
    assert np.array_equal(_lookup(e, tokens), _oracle(container.Container(data), ["tiny.embed"], tokens))
    assert yskn_b200.status() == 0


@pytest.mark.parametrize("n_parts", [1, 2, 3])
def test_residual_tables(cuda, tmp_path, n_parts):
    import torch
    import yskn_b200
    rows, cols = 300, 1024
    data = fixtures.embedding_container(rows, cols, PARTS[:n_parts])
    path = tmp_path / "emb.yskn"
    path.write_bytes(data)
    c = container.Container(data)
    names = [p[0] for p in PARTS[:n_parts]]
    rnd = fixtures.FixtureRandom(n_parts)
    tokens = [0, rows - 1, 7, 7] + [int(x % rows) for x in rnd.take(60)]
    want = _oracle(c, names, tokens)
    from_file = yskn_b200.File(str(path)).load_embedding(*names)
    assert np.array_equal(_lookup(from_file, tokens), want)
    keep = [torch.from_numpy(c.words(n).view(np.int32)).cuda() for n in names]
    from_arrays = yskn_b200.Embedding([(k, c.tensors[n]["bits"], c.lut16(n), c.scale16(n)) for k, n in zip(keep, names)],
                                      rows, cols, O.tensor_signs(c.tensors[names[0]]["rot_in"], cols))
    assert np.array_equal(_lookup(from_arrays, tokens), want)
    assert yskn_b200.status() == 0


def test_token_outside_the_table(cuda, tmp_path):
    import yskn_b200
    rows, cols = 300, 1024
    data = fixtures.embedding_container(rows, cols, PARTS[:1])
    path = tmp_path / "emb.yskn"
    path.write_bytes(data)
    e = yskn_b200.File(str(path)).load_embedding("emb")
    got = _lookup(e, [3, rows, -1, 4])
    want = _oracle(container.Container(data), ["emb"], [3, 4])
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[3], want[1])
    assert not got[1].any() and not got[2].any()
    assert yskn_b200.status() == yskn_b200.EINVAL
    assert yskn_b200.status() == 0  # the status call cleared the error word
