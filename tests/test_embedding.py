"""Coded embedding rows on the CPU: the oracle pinned to the reference's golden values,
and the file-level checks the library applies before it touches a GPU.

tools/testdata/tiny_expected.json (the reference's test data, rebuilt byte for byte by
the oracle) holds decoded weights of its embedding tensor at twelve positions; the
oracle's bf16 rows (docs/spec/02_COMPRESSED_LINEAR.md:271-303) must round them.
"""
import json
import os

import numpy as np
import pytest

import container
import fixtures
import oracle as O
from conftest import GOLDEN


def _bf16_to_f32(bits):
    return (np.asarray(bits, np.uint32) << np.uint32(16)).view(np.float32)


def _tiny_embed():
    c = container.Container(fixtures.tiny_container())
    d = c.tensors["tiny.embed"]
    parts = [(c.words("tiny.embed"), d["layout"], d["physical_rows"], d["cols"], d["bits"], c.lut16("tiny.embed"),
              c.scale16("tiny.embed"))]
    return c, d, parts


def test_oracle_rounds_the_reference_decoded_weights():
    c, d, parts = _tiny_embed()
    with open(os.path.join(GOLDEN, "tiny_expected.json")) as f:
        exp = json.load(f)["tensors"]["tiny.embed"]
    rows = sorted({r for r, _ in exp["sample_at"]})
    got = O.embedding_rows(parts, rows, O.tensor_signs(d["rot_in"], d["cols"]))
    for (r, col), v in zip(exp["sample_at"], exp["sample_values"]):
        x = float(_bf16_to_f32(got[rows.index(r), col]))
        half_ulp = 2.0 ** (np.floor(np.log2(abs(v))) - 8)  # bf16 keeps 8 significant bits
        assert abs(x - v) <= half_ulp + 1e-6 * abs(v), (r, col, x, v)


def test_oracle_adds_residual_tables_in_order():
    """A residual table equal to the main one doubles every decoded value exactly."""
    c, d, parts = _tiny_embed()
    s = O.tensor_signs(d["rot_in"], d["cols"])
    one = _bf16_to_f32(O.embedding_rows(parts, [7, 50], s))
    two = _bf16_to_f32(O.embedding_rows(parts * 2, [7, 50], s))
    assert np.array_equal(two, one * 2)


def test_file_embedding_checks(tmp_path):
    import yskn_b200
    path = tmp_path / "tiny.yskn"
    path.write_bytes(fixtures.tiny_container())
    f = yskn_b200.File(str(path))
    with pytest.raises(yskn_b200.YsknError) as e:
        f.load_embedding("tiny.body6")
    assert "role embedding" in str(e.value)
    with pytest.raises(yskn_b200.YsknError) as e:
        f.load_embedding("tiny.embed", res2="tiny.embed")
    assert "needs the first" in str(e.value)
    data = fixtures.embedding_container(64, 1024, [("e", 6, 1, ("mulberry32_7919_13", 7, 0)),
                                                   ("e.off", 6, 11, ("mulberry32_7919_13", 7, 5))])
    path2 = tmp_path / "emb.yskn"
    path2.write_bytes(data)
    g = yskn_b200.File(str(path2))
    with pytest.raises(yskn_b200.YsknError) as e:
        g.load_embedding("e", "e.off")
    assert "input-rotation offset" in str(e.value)
