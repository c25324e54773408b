"""TEST INFRASTRUCTURE ONLY: KVQP profiles and the KV row codec / attention oracle.

* `parse_profile` restates crates/yskn-ref/src/kv_profile.rs:107-217 (KVQP v1) and the
  predicates `packed_bits`, `packable`, `vit2_eligible` (:251-286).
* `encode` calls the C restatement of encode_packed / requantize_int8
  (crates/yskn-ref/src/kv_codec.rs:398-441) in oracle/kv_oracle.c.
* `test_profile` / `replace_group` / `test_rows` restate the fixture builders of the
  reference's frozen-hash test (crates/yskn-ref/src/kv_codec_tests.rs:14-98), and
  `synthetic_profile` the writer of crates/yskn-ref/tests/support/kv_profile.rs:12-79.
"""
import ctypes as C
import struct

import numpy as np

import oracle as O

_sig = False


def _lib():
    global _sig
    L = O.lib()
    if not _sig:
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        L.orc_kv_encode.argtypes = [vp, i, i, i, vp, f, i, i, vp, vp, vp, i, i, i, vp, vp, vp, vp, vp, vp, vp]
        L.orc_kv_attend_head.argtypes = [vp, vp, vp, vp, vp, vp, i, i, vp]
        L.orc_kv_packed_state.argtypes = [vp, i, i]
        L.orc_kv_cache_sign.restype = C.c_float
        L.orc_kv_inverse_rotate.argtypes = [vp]
        L.orc_kv_decode_rows.argtypes = [vp, C.c_int64, i, vp, vp]
        _sig = True
    return L


def _f16(v):
    return np.asarray(v, np.float32).astype("<f2").view("<u2")


class Profile:
    pass


def parse_profile(b):
    b = bytes(b)
    u16 = lambda o: struct.unpack_from("<H", b, o)[0]  # noqa: E731
    u32 = lambda o: struct.unpack_from("<I", b, o)[0]  # noqa: E731
    if len(b) < 100 or b[:4] != b"KVQP" or u16(4) != 1 or u16(6) != 96 or u32(8) != len(b) or u16(16) != 256:
        raise ValueError("invalid KVQP v1 header")
    p = Profile()
    p.layers, p.kv_heads, nt, nm, ng = u16(18), u16(20), u16(22), u16(24), u32(28)
    if p.layers == 0 or p.kv_heads == 0 or ng != p.layers * p.kv_heads * 2 or not 1 <= nm <= 16:
        raise ValueError("invalid dimensions")
    om, ot, og = u32(32), u32(36), u32(40)
    p.mults = np.array([struct.unpack_from("<f", b, om + 4 * k)[0] for k in range(nm)], np.float32)
    p.tables = []
    for k in range(nt):
        o = u32(ot + 4 * k)
        if b[o] != 8 or b[o + 2] != 64 or b[o + 3] != 8:
            raise ValueError("table requires state bits 8, chain 64, fractional bits 8")
        gain = struct.unpack_from("<f", b, o + 4)[0]
        codes = np.frombuffer(b, "<i2", 256, o + 12).copy()
        p.tables.append((np.float32(gain), codes))
    p.groups = []
    for k in range(ng):
        o = u32(og + 4 * k)
        mode, bits, table, guard, nb, has_mean = b[o], b[o + 1], b[o + 2], b[o + 3], b[o + 4], b[o + 5] != 0
        if mode == 0 and (not 3 <= bits <= 5 or table >= nt):
            raise ValueError("inconsistent trellis bits or table index")
        cur = o + 8
        mean = None
        if has_mean:
            mean = np.frombuffer(b, "<f2", 256, cur).astype(np.float32)
            cur += 512
        basis = []
        for _ in range(min(nb, 2)):
            basis.append(np.frombuffer(b, "<f2", 256, cur).astype(np.float32))
            cur += 512
        p.groups.append(dict(mode=mode, bits=bits, table=table, guard=guard, basis_count=nb, mean=mean,
                             basis=basis))
    return p


def packed_bits(p):
    c = lambda bits: sum(1 for g in p.groups if g["mode"] == 0 and g["bits"] == bits)  # noqa: E731
    return 5 if c(5) > c(4) else 4


def packable(p, layer, side):
    pb = packed_bits(p)
    return layer < p.layers and side < 2 and all(
        (lambda g: g["mode"] == 0 and g["bits"] == pb and g["guard"] == 0 and g["basis_count"] == 0)(
            p.groups[(layer * p.kv_heads + h) * 2 + side]) for h in range(p.kv_heads))


def vit2_eligible(p):
    found = False
    for g in p.groups:
        if g["mode"] == 0 and g["bits"] in (4, 5):
            found = True
            if np.any((p.tables[g["table"]][1] < -1100) | (p.tables[g["table"]][1] > 1100)):
                return False
    return found


def encode(p, group, position, row):
    """encode_packed + requantize_int8 of one row -> (kind, scale, words, ints, bases, req_scale, req_ints)."""
    g = p.groups[group]
    gain, codes = p.tables[g["table"]] if g["table"] < len(p.tables) else p.tables[0]
    row = np.ascontiguousarray(row, np.float32)
    basis = np.ascontiguousarray(np.concatenate(g["basis"]) if g["basis"] else np.zeros(1), np.float32)
    mean = None if g["mean"] is None else np.ascontiguousarray(g["mean"], np.float32)
    kind, scale, req_scale = C.c_int(), C.c_float(), C.c_float()
    words = np.zeros(40, np.uint32)
    ints = np.zeros(256, np.int8)
    bases = np.zeros(256, np.uint16)
    req_ints = np.zeros(256, np.int8)
    vit2 = int(vit2_eligible(p) and g["bits"] in (4, 5))
    pk = int(packable(p, group // (p.kv_heads * 2), group % 2))
    rc = _lib().orc_kv_encode(O._p(row), position, g["mode"], g["bits"], O._p(codes), float(gain), g["guard"],
                              len(g["basis"]), O._p(basis), None if mean is None else O._p(mean), O._p(p.mults),
                              len(p.mults), vit2, pk, C.byref(kind), C.byref(scale), O._p(words), O._p(ints),
                              O._p(bases), C.byref(req_scale), O._p(req_ints))
    if rc:
        raise O.OracleError("kv encode failed")
    k = kind.value
    return (k, np.float32(scale.value), words[:8 * k].copy() if k != 8 else None, ints, bases,
            np.float32(req_scale.value), req_ints)


def encoded_bytes(kind, scale, words, ints):
    """kv_codec_tests.rs:408-425."""
    out = bytes([kind]) + np.float32(scale).tobytes()
    if kind == 8:
        return out + ints.astype(np.int8).tobytes()
    return out + words.astype("<u4").tobytes()


# --------------------------------------------------------------- fixtures
def test_profile(layers, heads, bits):
    """kv_codec_tests.rs:14-58."""
    ng = layers * heads * 2
    b = bytearray(100 + 12 + 4 + 4 * ng)
    b[:4] = b"KVQP"
    for o, v in [(4, 1), (6, 96), (16, 256), (18, layers), (20, heads), (22, 1), (24, 3)]:
        struct.pack_into("<H", b, o, v)
    struct.pack_into("<I", b, 28, ng)
    for o, v in [(32, 100), (36, 112), (40, 116)]:
        struct.pack_into("<I", b, o, v)
    for i, m in enumerate([0.9, 1.0, 1.1]):
        struct.pack_into("<f", b, 100 + 4 * i, m)
    to = len(b)
    struct.pack_into("<I", b, 112, to)
    b += bytes(524)
    b[to], b[to + 1], b[to + 2], b[to + 3] = 8, bits, 64, 8
    struct.pack_into("<f", b, to + 4, 1.0)
    for s in range(256):
        struct.pack_into("<h", b, to + 12 + 2 * s, ((s * 73 + 19) % 2049) - 1024)
    for g in range(ng):
        go = len(b)
        struct.pack_into("<I", b, 116 + 4 * g, go)
        b += bytes([0, bits, 0, 0, 0, 0, 0, 0])
    struct.pack_into("<I", b, 8, len(b))
    return b


def replace_group(b, group, mode, guard, basis, mean):
    """kv_codec_tests.rs:60-82."""
    og = struct.unpack_from("<I", b, 40)[0]
    old = struct.unpack_from("<I", b, og + 4 * group)[0]
    header = bytearray(b[old:old + 8])
    header[0], header[3], header[4], header[5] = mode, guard, basis, int(mean)
    go = len(b)
    struct.pack_into("<I", b, og + 4 * group, go)
    b += header
    for vector in range(min(basis, 2) + int(mean)):
        if mean and vector == 0:
            v = (np.arange(256, dtype=np.float32) - np.float32(128.0)) / np.float32(1024.0)
        else:
            v = np.where(((np.arange(256) >> vector) & 1) == 0, 0.0625, -0.0625).astype(np.float32)
        b += _f16(v).tobytes()
    struct.pack_into("<I", b, 8, len(b))


def test_rows(seed, n):
    """kv_codec_tests.rs:84-98: xorshift32, 12-uniform sums, (x - 6) * 0.75 in binary32."""
    rows = []
    s = seed
    for _ in range(n):
        row = np.empty(256, np.float32)
        for c in range(256):
            x = np.float32(0.0)
            for _ in range(12):
                s ^= (s << 13) & 0xFFFFFFFF
                s ^= s >> 17
                s ^= (s << 5) & 0xFFFFFFFF
                x = np.float32(x + np.float32(np.float32(s >> 8) / np.float32(16777216.0)))
            row[c] = np.float32(np.float32(x - np.float32(6.0)) * np.float32(0.75))
        rows.append(row)
    return rows


def synthetic_profile(layers, heads, bits=4):
    """tests/support/kv_profile.rs:12-79 with the group bits byte set to `bits`: one table
    (codes (s*73+19)%2049-1024, gain 257/256), one multiplier 1.0, every group mode 0."""
    ng = layers * heads * 2
    b = bytearray(108 + 4 * ng)
    b[:4] = b"KVQP"
    for o, v in [(4, 1), (6, 96), (16, 256), (18, layers), (20, heads), (22, 1), (24, 1)]:
        struct.pack_into("<H", b, o, v)
    struct.pack_into("<I", b, 28, ng)
    for o, v in [(32, 100), (36, 104), (40, 108)]:
        struct.pack_into("<I", b, o, v)
    struct.pack_into("<f", b, 100, 1.0)
    table = len(b)
    struct.pack_into("<I", b, 104, table)
    b += bytes([8, 0, 64, 8]) + struct.pack("<f", 257.0 / 256.0) + bytes(4)
    for s in range(256):
        b += struct.pack("<h", ((s * 73 + 19) % 2049) - 1024)
    for g in range(ng):
        struct.pack_into("<I", b, 108 + 4 * g, len(b))
        b += bytes([0, bits, 0, 0, 0, 0, 0, 0])
    struct.pack_into("<I", b, 8, len(b))
    return b


def base_table_bf16(p, group):
    """The 256-entry BF16 codebook of a packed group: bfloat(reconstruction(state))."""
    g = p.groups[group]
    gain, codes = p.tables[g["table"]]
    rec = (codes.astype(np.float32) * np.float32(0.00390625)) * np.float32(gain)
    return np.array([O.f32_to_bf16(float(v)) for v in rec], np.uint16)


def attend_head(q, kb, ks, vb, vs, vmean, length, n_splits):
    """One query head over one KV head's cache (rows [0, length), last row = self)."""
    out = np.zeros(256, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    kb = np.ascontiguousarray(kb, np.float32)
    vb = np.ascontiguousarray(vb, np.float32)
    ks = np.ascontiguousarray(ks, np.float32)
    vs = np.ascontiguousarray(vs, np.float32)
    vm = None if vmean is None else np.ascontiguousarray(vmean, np.float32)
    rc = _lib().orc_kv_attend_head(O._p(q), O._p(kb), O._p(ks), O._p(vb), O._p(vs), None if vm is None else O._p(vm),
                                   length, n_splits, O._p(out))
    if rc:
        raise O.OracleError("attend_head failed")
    return out


def inverse_rotate(v):
    v = np.array(v, np.float32).copy()
    _lib().orc_kv_inverse_rotate(O._p(v))
    return v


def packed_states(words, bits):
    """packed_state (kv_codec.rs:467-475) for every channel of rows words[n][8*bits]:
    the last eight stream bits ending at the channel's field, reset at each 64-channel chain."""
    words = np.asarray(words, np.uint32).reshape(-1, 8 * bits)
    n = words.shape[0]
    bitstream = np.unpackbits(words.astype(">u4").view(np.uint8).reshape(n, -1), axis=1)  # MSB first per word
    fields = bitstream.reshape(n, 256, bits)
    f = np.zeros((n, 256), np.int64)
    for j in range(bits):
        f = (f << 1) | fields[:, :, j]
    state = np.zeros((n, 256), np.int64)
    c = np.arange(256)
    for back in range(7 // bits, -1, -1):  # oldest contributing field first
        src = c - back
        ok = (src >= c // 64 * 64)
        prev = np.where(ok, f[:, np.clip(src, 0, 255)], 0)
        state = ((state << bits) | prev) & 0xFF
    return state


def decode_packed_rows(words, bits, codebook_bf16):
    """decode_packed (kv_codec.rs:485-495) as floats: codebook[packed_state] (C loop)."""
    words = np.ascontiguousarray(np.asarray(words, np.uint32).reshape(-1, 8 * bits))
    book = np.ascontiguousarray(codebook_bf16, np.uint16)
    out = np.empty((words.shape[0], 256), np.float32)
    _lib().orc_kv_decode_rows(O._p(words), C.c_int64(words.shape[0]), bits, O._p(book), O._p(out))
    return out


def prefix_schedule(length):
    """attention.rs:207-232: (tiles [(tile_start, first, end)], include_self) per split."""
    count = 31 if length < 4096 else 42
    per = -(-length // count)
    plans = []
    for s in range(count):
        first = s * per
        last = min(first + per, length)
        prefix_end = max(first, min(last, length - 1))
        tiles = []
        if first < prefix_end:
            t = first // 32 * 32
            while t < prefix_end:
                tiles.append((t, max(first, t), min(prefix_end, t + 32)))
                t += 32
        plans.append((tiles, first < length and length - 1 < first + per))
    return plans
