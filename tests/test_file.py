"""The library's `.yskn` reader (yskn_b200_file_*) on the CPU: no GPU is touched.

It must read what the reference reader reads and reject what it rejects
(crates/yskn-format/src/lib.rs:97-172, tensor.rs:31-63,83-196,212-236). The
reference's own test file tools/testdata/tiny.yskn is rebuilt byte for byte by the
oracle (pinned by its SHA-256 in test_oracle_golden.py); the library's descriptors
and vectors are compared with the oracle reader's on it, and every rejection case
changes one member of it and names the check it trips.
"""
import json
import struct

import numpy as np
import pytest

import container
import fixtures


@pytest.fixture(scope="module")
def yskn():
    import yskn_b200
    return yskn_b200


def _open(yskn, tmp_path, data, name="t.yskn"):
    path = tmp_path / name
    path.write_bytes(bytes(data))
    return yskn.File(str(path))


def _with_header(data, edit):
    """The tiny container with its JSON header edited by `edit(root)` (data blocks kept)."""
    hb, data_off = struct.unpack_from("<QQ", data, 8)
    root = json.loads(data[32:32 + hb].decode("utf-8"))
    edit(root)
    head = json.dumps(root, separators=(",", ":")).encode("utf-8")
    assert 32 + len(head) <= data_off
    out = bytearray(data[:4] + struct.pack("<IQQQ", 1, len(head), data_off, len(data)) + head)
    out += b"\0" * (data_off - len(out))
    return bytes(out) + data[data_off:]


def _expected(desc):
    d = dict(desc)
    d.pop("index", None)
    return d


def test_tiny_container_reads_like_the_oracle(yskn, tmp_path):
    data = fixtures.tiny_container()
    want = container.Container(data)
    f = _open(yskn, tmp_path, data)
    assert f.model == want.model
    assert list(f.tensors) == list(want.tensors)
    for name, t in want.tensors.items():
        assert _expected(f.tensors[name]) == t, name
    assert list(f.vectors) == list(want.vectors)
    for name in want.vectors:
        got = f.vector(name)
        assert got.dtype == np.float32
        assert np.array_equal(got.view(np.uint32), want.vector(name).view(np.uint32)), name
    f.close()


def test_defaults_of_absent_members(yskn, tmp_path):
    """Absent members take the format's defaults (tensor.rs:97-188, FORMAT.md:66-87)."""
    def edit(root):
        for t in root["tensors"]:
            if t["name"] in ("tiny.body6", "tiny.head"):
                for key in ("physical_rows", "l", "d", "t", "start", "layout", "rot_in", "rot_out", "rar",
                            "bias_off"):
                    t.pop(key)
        for v in root["vectors"]:
            if v["name"] == "tiny.half":
                v.pop("dtype")
    data = _with_header(fixtures.tiny_container(), edit)
    want = container.Container(data)
    f = _open(yskn, tmp_path, data)
    for name in ("tiny.body6", "tiny.head"):
        assert _expected(f.tensors[name]) == want.tensors[name]
    body, head = f.tensors["tiny.body6"], f.tensors["tiny.head"]
    assert body["layout"] == "warp" and body["physical_rows"] == body["rows"]
    assert body["rot_in"] == dict(rule="mulberry32_7919_13", seed=7, offset=0)
    assert body["rot_out"] == dict(rule="mulberry32_7919_13", seed=7, offset=body["cols"])
    assert head["rot_out"] is None
    assert f.vectors["tiny.half"]["dtype"] == "f16"


def test_json_escapes_duplicate_keys_and_none_output_rotation(yskn, tmp_path):
    def edit(root):
        t = root["tensors"][0]
        t["name"] = "tiny.é\U0001f600/\"q\""
        t["rot_out"] = dict(kind="none", qm_off=0)
    data = _with_header(fixtures.tiny_container(), edit)
    # A member given twice keeps its last value, as in the reference's JSON reader.
    hb = struct.unpack_from("<Q", data, 8)[0]
    head = data[32:32 + hb].replace(b'"bits":6', b'"bits":7,"bits":6', 1)
    data = data[:8] + struct.pack("<Q", len(head)) + data[16:32] + head + data[32 + len(head):]
    f = _open(yskn, tmp_path, data)
    t = f.tensors["tiny.é\U0001f600/\"q\""]
    assert t["bits"] == 6 and t["rot_out"] is None
    assert f.tensors["tiny.body8"]["rot_out"] is not None


def _tensor(name):
    def pick(root):
        return next(t for t in root["tensors"] if t["name"] == name)
    return pick


def _set(name, key, value):
    def edit(root):
        t = _tensor(name)(root)
        if value is _DEL:
            t.pop(key)
        else:
            t[key] = value
    return edit


_DEL = object()
_REJECT = [  # (case, header edit, part of the message)
    ("model not an object", lambda r: r.update(model=[]), "model must be an object"),
    ("no tensors", lambda r: r.pop("tensors"), "missing tensors"),
    ("no vectors", lambda r: r.pop("vectors"), "missing vectors"),
    ("tensors not a list", lambda r: r.update(tensors={}), "tensors must be an array"),
    ("empty name", _set("tiny.body6", "name", ""), "empty tensor name"),
    ("unknown role", _set("tiny.body6", "role", "encoder"), "tensor role encoder"),
    ("cols not a multiple of 512", _set("tiny.body6", "cols", 500), "invalid matrix dimensions"),
    ("physical rows below rows", _set("tiny.body6", "physical_rows", 256), "invalid matrix dimensions"),
    ("rows as a float", _set("tiny.body6", "rows", 512.0), "rows must be an unsigned integer"),
    ("negative rows", _set("tiny.body6", "rows", -512), "rows must be an unsigned integer"),
    ("no bits", _set("tiny.body6", "bits", _DEL), "missing bits"),
    ("state bits", _set("tiny.body6", "l", 10), "l must be 12"),
    ("weights per step", _set("tiny.body6", "d", 4), "d must be 2"),
    ("bits 9", _set("tiny.body6", "bits", 9), "bits must be 4..8"),
    ("bits 3", _set("tiny.body6", "bits", 3), "bits must be 4..8"),
    ("carry start", _set("tiny.body6", "start", "carry"), "start=carry"),
    ("rar object", _set("tiny.body6", "rar", {}), "rar is unspecified"),
    ("bias", _set("tiny.body6", "bias_off", 4), "bias_off must be zero"),
    ("unknown layout", _set("tiny.body6", "layout", "tile"), "layout tile"),
    ("warp sequences", _set("tiny.head", "physical_rows", 65), "multiple of 32 sequences"),
    ("stream length", lambda r: _tensor("tiny.body6")(r).update(stream_bytes=_tensor("tiny.body6")(r)["stream_bytes"]
                                                                 + 16), "stream_bytes differs"),
    ("table outside the file", _set("tiny.body6", "lut_off", 1 << 40), "lies outside payload"),
    ("scales before the data", _set("tiny.body6", "scale_off", 100), "lies outside payload"),
    ("stream offset overflow", _set("tiny.body6", "stream_off", (1 << 64) - 8), "overflow"),
    ("input rotation null", _set("tiny.body6", "rot_in", None), "rotation must be an object"),
    ("input rotation none", _set("tiny.body6", "rot_in", dict(kind="none", qm_off=0)), "rotation none"),
    ("AYA rotation", _set("tiny.body6", "rot_in", dict(kind="AYA", m=1, sign_seed=7, sign_offset=0, qm_off=3)),
     "rotation AYA"),
    ("rotation blocks", _set("tiny.body6", "rot_in", dict(kind="H512", m=2, sign_seed=7, sign_offset=0)),
     "rotation block count"),
    ("qm_off", _set("tiny.body6", "rot_in", dict(kind="H512", m=1, sign_seed=7, sign_offset=0, qm_off=1)),
     "must have qm_off=0"),
    ("sign rule", _set("tiny.body6", "rot_in", dict(kind="H512", m=1, sign_seed=7, sign_offset=0, rule="xorshift")),
     "sign rule xorshift"),
    ("no sign seed", _set("tiny.body6", "rot_in", dict(kind="H512", m=1, sign_offset=0)), "missing sign_seed"),
    ("output rotation of partial blocks", _set("tiny.head", "rot_out", dict(kind="H512", m=0, sign_seed=7,
                                                                            sign_offset=512)),
     "whole 512-row blocks"),
    ("duplicate tensor", lambda r: r["tensors"][1].update(name="tiny.body6"), "duplicate parameter tiny.body6"),
    ("vector named like a tensor", lambda r: r["vectors"][0].update(name="tiny.head"),
     "duplicate parameter tiny.head"),
    ("vector dtype", lambda r: r["vectors"][0].update(dtype="f32"), "vector dtype f32"),
    ("vector outside the file", lambda r: r["vectors"][1].update(n=1 << 40), "lies outside payload"),
    ("empty vector name", lambda r: r["vectors"][1].update(name=""), "empty vector name"),
]


@pytest.mark.parametrize("case,edit,message", _REJECT, ids=[c[0] for c in _REJECT])
def test_rejects_like_the_reference_reader(yskn, tmp_path, case, edit, message):
    data = _with_header(fixtures.tiny_container(), edit)
    with pytest.raises(yskn.YsknError) as e:
        _open(yskn, tmp_path, data)
    assert e.value.code == yskn.EINVAL
    assert message in str(e.value), str(e.value)


def _patched(data, offset, raw):
    out = bytearray(data)
    out[offset:offset + len(raw)] = raw
    return bytes(out)


def test_rejects_broken_prefix_and_padding(yskn, tmp_path):
    data = fixtures.tiny_container()
    hb = struct.unpack_from("<Q", data, 8)[0]
    cases = [
        (data[:20], "magic must be YSKN"),
        (_patched(data, 0, b"YSKX"), "magic must be YSKN"),
        (_patched(data, 4, struct.pack("<I", 2)), "version 2"),
        (data + b"\0", "declared file length differs"),
        (_patched(data, 16, struct.pack("<Q", 40)), "header or first data offset lies outside the file"),
        (_patched(data, 16, struct.pack("<Q", len(data) + 1)), "header or first data offset lies outside"),
        (_patched(data, 32 + hb + 7, b"\x01"), "nonzero bytes between header and first data block"),
        (_patched(data, 32, b"["), "not valid JSON"),
        (_patched(data, 33, b"\xff"), "not valid UTF-8"),
    ]
    for i, (bad, message) in enumerate(cases):
        with pytest.raises(yskn.YsknError) as e:
            _open(yskn, tmp_path, bad, "bad%d.yskn" % i)
        assert message in str(e.value), (i, str(e.value))
    with pytest.raises(yskn.YsknError) as e:
        yskn.File(str(tmp_path / "absent.yskn"))
    assert "cannot open" in str(e.value)


def test_embedding_is_not_a_linear_operator(yskn, tmp_path):
    """Loading needs no GPU to refuse an embedding (its table stays 16-bit in the reference)."""
    f = _open(yskn, tmp_path, fixtures.tiny_container())
    with pytest.raises(yskn.YsknError) as e:
        f.load_matrix("tiny.embed")
    assert "embedding" in str(e.value)
