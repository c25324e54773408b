"""TEST INFRASTRUCTURE ONLY: a numpy reader and writer of `.yskn` containers.

Restates the container layout of the reference's docs/FORMAT.md:25-107 (prefix,
JSON header, tensor descriptors with their defaults) and the descriptor checks of
crates/yskn-format/src/lib.rs:97-172 and crates/yskn-format/src/tensor.rs:83-196.
Used by tests/, bench.py's synthetic-weight generator and the golden-fixture
script; the product library takes raw device pointers and never reads files.
"""
import json
import struct

import numpy as np

MAGIC = b"YSKN"
PREFIX = 32


class FormatError(ValueError):
    pass


def _rot(value, blocks, allow_none, default):
    if value is None and "missing" == default:
        return None
    if value is None:
        if allow_none:
            return None
        raise FormatError("input rotation is required")
    if value.get("kind") == "none" and allow_none:
        return None
    if value.get("kind") != "H512":
        raise FormatError("unsupported rotation %r" % value.get("kind"))
    if value.get("qm_off", 0) != 0:
        raise FormatError("rotation H512 must have qm_off=0")
    if int(value["m"]) != blocks:
        raise FormatError("rotation block count differs from tensor dimensions")
    rule = value.get("rule", "splitmix64")
    if rule not in ("splitmix64", "mulberry32_7919_13"):
        raise FormatError("unsupported sign rule %r" % rule)
    return dict(rule=rule, seed=int(value["sign_seed"]), offset=int(value["sign_offset"]))


def parse_descriptor(t, first, end):
    """tensor.rs:83-196: a validated descriptor with the format's defaults."""
    name = t["name"]
    rows, cols = int(t["rows"]), int(t["cols"])
    phys = int(t.get("physical_rows", rows))
    if rows == 0 or cols == 0 or cols % 512 or phys < rows:
        raise FormatError("invalid matrix dimensions for %s" % name)
    for key, want in (("l", 12), ("d", 2), ("t", 256)):
        if t.get(key, want) != want:
            raise FormatError("%s: %s must be %d" % (name, key, want))
    bits = int(t["bits"])
    if not 4 <= bits <= 8:
        raise FormatError("%s: bits must be 4..8" % name)
    if t.get("start", "zero") != "zero" or t.get("rar") or t.get("bias_off", 0) != 0:
        raise FormatError("%s: unsupported start/rar/bias_off" % name)
    layout = t.get("layout", "warp")
    if layout not in ("row", "warp"):
        raise FormatError("layout %r" % layout)
    seqs = phys * (cols // 256)
    if layout == "warp" and seqs % 32:
        raise FormatError("warp layout requires a multiple of 32 sequences")
    if int(t["stream_bytes"]) != seqs * bits * 16:
        raise FormatError("%s: stream_bytes differs from matrix shape" % name)
    for off, n in ((t["stream_off"], t["stream_bytes"]), (t["lut_off"], 16384), (t["scale_off"], 2 * phys)):
        if off < first or off + n > end:
            raise FormatError("%s: data region outside the file" % name)
    role = t["role"]
    if role not in ("body", "head", "embedding", "draft"):
        raise FormatError("tensor role %r" % role)
    if "rot_in" in t:
        rot_in = _rot(t["rot_in"], cols // 512, False, None)
    else:
        rot_in = dict(rule="mulberry32_7919_13", seed=7, offset=0)
    if "rot_out" in t:
        rot_out = _rot(t["rot_out"], rows // 512, True, None)
    elif role in ("head", "embedding"):
        rot_out = None
    else:
        rot_out = dict(rule="mulberry32_7919_13", seed=7, offset=cols)
    if rot_out is not None and (rows % 512 or phys % 512):
        raise FormatError("output rotation requires whole 512-row blocks")
    return dict(name=name, role=role, rows=rows, cols=cols, physical_rows=phys, bits=bits, layout=layout,
                stream_off=int(t["stream_off"]), stream_bytes=int(t["stream_bytes"]),
                lut_off=int(t["lut_off"]), scale_off=int(t["scale_off"]), rot_in=rot_in, rot_out=rot_out)


class Container:
    """lib.rs:97-172: prefix, JSON header, zero padding, unique names."""

    def __init__(self, data):
        data = bytes(data)
        if len(data) < PREFIX or data[:4] != MAGIC:
            raise FormatError("magic must be YSKN")
        self.version, = struct.unpack_from("<I", data, 4)
        if self.version != 1:
            raise FormatError("version %d" % self.version)
        self.header_bytes, self.data_offset, self.file_bytes = struct.unpack_from("<QQQ", data, 8)
        if self.file_bytes != len(data):
            raise FormatError("declared file length differs from actual length")
        end = PREFIX + self.header_bytes
        if end > self.data_offset or self.data_offset > self.file_bytes:
            raise FormatError("header or first data offset lies outside the file")
        root = json.loads(data[PREFIX:end].decode("utf-8"))
        if any(data[end:self.data_offset]):
            raise FormatError("nonzero bytes between header and first data block")
        self.data = data
        self.model = root["model"]
        if not isinstance(self.model, dict):
            raise FormatError("model must be an object")
        self.tensors, self.vectors, names = {}, {}, set()
        for t in root["tensors"]:
            d = parse_descriptor(t, self.data_offset, self.file_bytes)
            if d["name"] in names:
                raise FormatError("duplicate parameter %s" % d["name"])
            names.add(d["name"])
            self.tensors[d["name"]] = d
        for v in root["vectors"]:
            if v["name"] in names:
                raise FormatError("duplicate parameter %s" % v["name"])
            names.add(v["name"])
            if v["off"] < self.data_offset or v["off"] + 2 * v["n"] > self.file_bytes:
                raise FormatError("vector outside the file")
            self.vectors[v["name"]] = dict(v)

    def words(self, name):
        d = self.tensors[name]
        return np.frombuffer(self.data, "<u4", d["stream_bytes"] // 4, d["stream_off"]).copy()

    def lut16(self, name):
        return np.frombuffer(self.data, "<u2", 8192, self.tensors[name]["lut_off"]).copy()

    def scale16(self, name):
        d = self.tensors[name]
        return np.frombuffer(self.data, "<u2", d["physical_rows"], d["scale_off"]).copy()

    def vector(self, name):
        v = self.vectors[name]
        raw = np.frombuffer(self.data, "<u2", v["n"], v["off"])
        if v.get("dtype", "f16") == "bf16":
            return (raw.astype(np.uint32) << np.uint32(16)).view(np.float32)
        return raw.view("<f2").astype(np.float32)


def write_container(model, tensors, vectors, blobs, data_offset=4096, align=64):
    """Lay out `blobs` (a list of bytes) after the header; descriptors refer to them
    through the placeholders {"$blob": i}. Returns the file bytes (FORMAT.md:25-36)."""
    pos, body, offsets = data_offset, [], []
    for b in blobs:
        pad = (-pos) % align
        body.append(b"\0" * pad + bytes(b))
        pos += pad
        offsets.append(pos)
        pos += len(b)

    def resolve(x):
        if isinstance(x, dict):
            if set(x) == {"$blob"}:
                return offsets[x["$blob"]]
            return {k: resolve(v) for k, v in x.items()}
        if isinstance(x, list):
            return [resolve(v) for v in x]
        return x

    head = json.dumps(dict(model=model, tensors=resolve(tensors), vectors=resolve(vectors)),
                      separators=(",", ":")).encode("utf-8")
    if PREFIX + len(head) > data_offset:
        raise FormatError("the header does not fit before the data")
    total = pos
    out = MAGIC + struct.pack("<IQQQ", 1, len(head), data_offset, total) + head
    return out + b"\0" * (data_offset - len(out)) + b"".join(body)
