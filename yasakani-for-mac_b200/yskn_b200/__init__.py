"""ctypes binding of libyskn_b200.so (include/yskn_b200.h).

This mirrors how the reference's Python front end binds its native library
(python/yasakani/_native.py:26-39): a CDLL with declared argument types, integer
status codes and a thread-local error string. Device buffers are torch tensors
(plumbing only); every computation runs in the CUDA library. Import fails loudly
if the library has not been built; there is no fallback path.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "libyskn_b200.so")

OK, EINVAL, ECUDA, EOVERFLOW, ENONFINITE, ETIMEDOUT, ENOMEM = 0, -1, -2, -3, -4, -5, -6
LAYOUT_ROW, LAYOUT_WARP = 0, 1
LAYOUTS = {"row": LAYOUT_ROW, "warp": LAYOUT_WARP}
SIGN_RULES = {"splitmix64": 0, "mulberry32_7919_13": 1}

_vp, _i, _i64, _u64 = C.c_void_p, C.c_int, C.c_int64, C.c_uint64

_SIGNATURES = {
    "yskn_b200_last_error": (C.c_char_p, []),
    "yskn_b200_status": (_i, [_vp]),
    "yskn_repack_warp_to_frag": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "yskn_repack_warp_to_frag_host": (_i, [_vp, _vp, _i, _i, _i]),
    "yskn_b200_signs": (_i, [_i, _u64, _u64, _i64, _vp]),
    "yskn_b200_pack_bytes": (_i64, [_i, _i, _i]),
    "yskn_b200_pack": (_i, [_vp, _i, _i, _i, _i, _vp, _vp]),
    "yskn_b200_matrix_create": (_vp, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_matrix_create_shard": (_vp, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "yskn_b200_matrix_destroy": (None, [_vp]),
    "yskn_b200_matrix_info": (_i, [_vp, _vp]),
    "yskn_b200_matrix_lut8": (_vp, [_vp]),
    "yskn_b200_matrix_tau": (_vp, [_vp]),
    "yskn_b200_matrix_signs_in": (_vp, [_vp]),
    "yskn_b200_matrix_signs_out": (_vp, [_vp]),
    "yskn_b200_weighted_sums": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp]),
    "yskn_b200_weighted_sums_prefix": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp]),
    "yskn_b200_weighted_sums_noalloc": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp]),
    "yskn_b200_quantize": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    "yskn_b200_rescale": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp]),
    "yskn_b200_tp_create": (_vp, [_i, _i, _i, _vp]),
    "yskn_b200_tp_connect": (_i, [_vp, _vp]),
    "yskn_b200_tp_destroy": (None, [_vp]),
    "yskn_b200_tp_area": (_vp, [_vp]),
    "yskn_b200_tp_connect_peers": (_i, [_vp, _vp]),
    "yskn_b200_tp_set_wait": (_i, [_vp, C.c_double]),
    "yskn_b200_linear_rowpar": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "yskn_b200_restore": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "yskn_b200_linear_work_bytes": (_i64, [_vp, _i, _i]),
    "yskn_b200_linear": (_i, [_vp, _i, _vp, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_kv4_attention_work_bytes": (_i64, [_i, _i, _i, _i]),
    "yskn_b200_kv4_attention": (_i, [_vp] * 9 + [_i] * 7 + [_vp] * 4),
    "yskn_b200_kv_encode": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_file_open": (_vp, [C.c_char_p]),
    "yskn_b200_file_close": (None, [_vp]),
    "yskn_b200_file_model_json": (C.c_char_p, [_vp]),
    "yskn_b200_file_tensor_count": (_i, [_vp]),
    "yskn_b200_file_vector_count": (_i, [_vp]),
    "yskn_b200_file_find": (_i, [_vp, C.c_char_p, _vp]),
    "yskn_b200_file_tensor_name": (C.c_char_p, [_vp, _i]),
    "yskn_b200_file_tensor_info": (_i, [_vp, _i, _vp]),
    "yskn_b200_file_vector_name": (C.c_char_p, [_vp, _i]),
    "yskn_b200_file_vector_info": (_i, [_vp, _i, _vp]),
    "yskn_b200_file_vector_read": (_i, [_vp, _i, _vp, _i64]),
    "yskn_b200_file_load_matrix": (_vp, [_vp, _i]),
    "yskn_b200_file_load_matrix_shard": (_vp, [_vp, _i, _i, _i, _i, _i]),
    "yskn_b200_embedding_create": (_vp, [_i, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "yskn_b200_embedding_destroy": (None, [_vp]),
    "yskn_b200_embedding_lookup": (_i, [_vp, _vp, _i, _vp, _vp]),
    "yskn_b200_file_load_embedding": (_vp, [_vp, _i, _i, _i]),
    "yskn_b200_residual_prepare": (_i, [_vp, _vp, _vp, _i, _i, C.c_float, _vp, _vp, _vp, _vp]),
    "yskn_b200_gated_product": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "yskn_b200_head_select": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_attention_prep": (_i, [_vp] * 6 + [C.c_float, _i, _i, _i] + [_vp] * 5),
    "yskn_b200_gdn_gates": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _vp]),
    "yskn_b200_widen_bf16": (_i, [_vp, C.c_int64, _vp, _vp]),
    "yskn_b200_portable_math": (_i, [_i, _vp, C.c_int64, _vp, _vp, _vp]),
    "yskn_b200_linear_residual": (_i, [_vp] * 4 + [_i] + [_vp] * 8),
    "yskn_b200_linear_q8": (_i, [_vp, _i, _vp, _vp, _vp, C.c_float, _i, _vp, _vp, _vp]),
    "yskn_b200_gated_product_q8": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_gdn_step": (_i, [_vp] * 7 + [C.c_float, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_matrix_create_rows": (_vp, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _vp, _i, _i]),
    "yskn_b200_gdn_gates_heads": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "yskn_b200_gdn_step_heads": (_i, [_vp] * 7 + [C.c_float, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_gdn_mixer": (_i, [_vp] * 4 + [_i] + [_vp] * 6 + [C.c_float, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_gdn_mixer_heads": (_i, [_vp] * 4 + [_i] + [_vp] * 6 + [C.c_float, _i, _i, _i, _i, _i, _i, _vp, _vp,
                                                                        _vp, _vp]),
    "yskn_b200_linear_rowpar_residual": (_i, [_vp] * 5 + [_i] + [_vp] * 8),
    "yskn_b200_head_merge": (_i, [_vp, _vp, _i64, _vp, _i, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_linear_from_residual": (_i, [_vp, _i, _vp, _vp, _vp, _vp, C.c_float, _i, _vp, _vp, _vp, _vp]),
    "yskn_b200_linear_rowpar_q8": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp]),
}

_lib = None


class YsknError(RuntimeError):
    def __init__(self, code, message):
        super().__init__("%s (code %d)" % (message, code))
        self.code = code


def lib():
    """Load the library and declare every exported symbol of include/yskn_b200.h."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError("libyskn_b200.so is not built (run yasakani-for-mac_b200/build.py)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return sorted(_SIGNATURES)


def last_error():
    msg = lib().yskn_b200_last_error()
    return msg.decode() if msg else ""


def check(rc, what=""):
    if rc != OK:
        raise YsknError(rc, "%s: %s" % (what, last_error()))
    return rc


def _ptr(t):
    """A device tensor's address, or a raw device address given as an int."""
    if t is None:
        return None
    if isinstance(t, int):
        return C.c_void_p(t)
    return C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def signs(rule, seed, offset, n):
    import numpy as np
    out = np.empty(n, np.int8)
    check(lib().yskn_b200_signs(SIGN_RULES[rule], seed, offset, n, out.ctypes.data), "signs")
    return out


class Matrix:
    """One compressed matrix on the device (yskn_b200_matrix_create)."""

    def __init__(self, d_codes, layout, rows, physical_rows, cols, bits, lut16, scale16, signs_in, signs_out=None,
                 shard=None):
        """shard: (row_begin, row_end, col_begin, col_end) of the whole tensor described by
        the other arguments (yskn_b200_matrix_create_shard), or None for the whole tensor;
        or ([(row_begin, row_end), ...], col_begin, col_end): several row ranges stored one
        after another (yskn_b200_matrix_create_rows)."""
        import numpy as np
        lut16 = np.ascontiguousarray(lut16, np.uint16)
        scale16 = np.ascontiguousarray(scale16, np.uint16)
        signs_in = np.ascontiguousarray(signs_in, np.int8)
        so = None if signs_out is None else np.ascontiguousarray(signs_out, np.int8)
        args = (_ptr(d_codes), LAYOUTS.get(layout, layout), rows, physical_rows, cols, bits, lut16.ctypes.data,
                scale16.ctypes.data, signs_in.ctypes.data, None if so is None else so.ctypes.data)
        if shard is None:
            h = lib().yskn_b200_matrix_create(*args)
            shard = (0, physical_rows, 0, cols)
        elif len(shard) == 3:
            ranges, c0, c1 = shard
            flat = (C.c_int * (2 * len(ranges)))(*[int(v) for r in ranges for v in r])
            h = lib().yskn_b200_matrix_create_rows(*args, len(ranges), flat, c0, c1)
        else:
            h = lib().yskn_b200_matrix_create_shard(*args, *shard)
        if not h:
            raise YsknError(EINVAL, "matrix_create: " + last_error())
        self.handle = C.c_void_p(h)
        self.shard = tuple(shard)
        if len(shard) == 3:
            ranges, c0, c1 = shard
            self.rows = sum(min(rows, r1) - r0 for r0, r1 in ranges)
            self.physical_rows = sum(r1 - r0 for r0, r1 in ranges)
        else:
            r0, r1, c0, c1 = shard
            self.rows, self.physical_rows = min(rows, r1) - r0, r1 - r0
        self.cols, self.bits = c1 - c0, bits
        self.has_rotation = so is not None

    @classmethod
    def _from_handle(cls, h, rows, physical_rows, cols, bits, has_rotation, shard):
        """A Matrix around a handle the library created (e.g. File.load_matrix)."""
        m = cls.__new__(cls)
        m.handle = C.c_void_p(h)
        r0, r1, c0, c1 = shard
        m.shard = tuple(shard)
        m.rows, m.physical_rows = min(rows, r1) - r0, r1 - r0
        m.cols, m.bits = c1 - c0, bits
        m.has_rotation = has_rotation
        return m

    def info(self):
        out = (C.c_int64 * 6)()
        check(lib().yskn_b200_matrix_info(self.handle, out), "matrix_info")
        return list(out)

    def close(self):
        if self.handle:
            lib().yskn_b200_matrix_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def signs_in_ptr(self):
        return lib().yskn_b200_matrix_signs_in(self.handle)


ROLES = ("body", "head", "embedding", "draft")
_RULE_NAMES = ("splitmix64", "mulberry32_7919_13")  # YSKN_SIGNS_* order


class File:
    """A `.yskn` container opened and checked by the library (yskn_b200_file_open):
    `model` (the header's model object), `tensors` and `vectors` (name -> descriptor with
    the format's defaults applied), `vector(name)` (f32 values) and `load_matrix(name)`
    (a Matrix whose codes, table, scales and signs come from the file)."""

    def __init__(self, path):
        import json
        h = lib().yskn_b200_file_open(os.fsencode(path))
        if not h:
            raise YsknError(EINVAL, last_error())
        self.handle = C.c_void_p(h)
        self.path = path
        self.model = json.loads(lib().yskn_b200_file_model_json(self.handle).decode("utf-8"))
        self.tensors, self.vectors = {}, {}
        info = (C.c_int64 * 17)()
        for i in range(lib().yskn_b200_file_tensor_count(self.handle)):
            check(lib().yskn_b200_file_tensor_info(self.handle, i, info), "file_tensor_info")
            v = list(info)
            rot = lambda r, seed, off: dict(rule=_RULE_NAMES[r], seed=seed, offset=off)
            name = lib().yskn_b200_file_tensor_name(self.handle, i).decode("utf-8")
            self.tensors[name] = dict(
                index=i, name=name, role=ROLES[v[0]], rows=v[1], cols=v[2], physical_rows=v[3], bits=v[4],
                layout="warp" if v[5] == LAYOUTS["warp"] else "row", stream_off=v[6], stream_bytes=v[7],
                lut_off=v[8], scale_off=v[9], rot_in=rot(v[10], v[11], v[12]),
                rot_out=rot(v[14], v[15], v[16]) if v[13] else None)
        vinfo = (C.c_int64 * 3)()
        for i in range(lib().yskn_b200_file_vector_count(self.handle)):
            check(lib().yskn_b200_file_vector_info(self.handle, i, vinfo), "file_vector_info")
            name = lib().yskn_b200_file_vector_name(self.handle, i).decode("utf-8")
            self.vectors[name] = dict(index=i, name=name, off=vinfo[0], n=vinfo[1],
                                      dtype="bf16" if vinfo[2] == 1 else "f16")

    def vector(self, name):
        import numpy as np
        v = self.vectors[name]
        out = np.empty(v["n"], np.float32)
        check(lib().yskn_b200_file_vector_read(self.handle, v["index"], out.ctypes.data, v["n"]), "file_vector_read")
        return out

    def load_matrix(self, name, shard=None):
        t = self.tensors[name]
        if shard is None:
            h = lib().yskn_b200_file_load_matrix(self.handle, t["index"])
            shard = (0, t["physical_rows"], 0, t["cols"])
        else:
            h = lib().yskn_b200_file_load_matrix_shard(self.handle, t["index"], *shard)
        if not h:
            raise YsknError(EINVAL, "file_load_matrix: " + last_error())
        return Matrix._from_handle(h, t["rows"], t["physical_rows"], t["cols"], t["bits"], t["rot_out"] is not None,
                                   shard)

    def load_embedding(self, main, res=None, res2=None):
        """An Embedding from the coded table `main` and up to two residual tables."""
        idx = [self.tensors[n]["index"] if n is not None else -1 for n in (main, res, res2)]
        h = lib().yskn_b200_file_load_embedding(self.handle, *idx)
        if not h:
            raise YsknError(EINVAL, "file_load_embedding: " + last_error())
        t = self.tensors[main]
        return Embedding._from_handle(h, t["rows"], t["cols"])

    def close(self):
        if self.handle:
            lib().yskn_b200_file_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Embedding:
    """Coded embedding rows on the device (yskn_b200_embedding_create / _lookup)."""

    def __init__(self, parts, rows, cols, signs_in):
        """parts: 1..3 tuples (d_codes, bits, lut16, scale16), the main table first; d_codes
        a device tensor holding the row-layout code stream; signs_in the main table's."""
        import numpy as np
        keep = [(np.ascontiguousarray(l, np.uint16), np.ascontiguousarray(s, np.uint16)) for _, _, l, s in parts]
        n = len(parts)
        codes = (C.c_void_p * n)(*[_ptr(c) for c, _, _, _ in parts])
        bits = (C.c_int * n)(*[b for _, b, _, _ in parts])
        luts = (C.c_void_p * n)(*[l.ctypes.data for l, _ in keep])
        scales = (C.c_void_p * n)(*[s.ctypes.data for _, s in keep])
        si = np.ascontiguousarray(signs_in, np.int8)
        h = lib().yskn_b200_embedding_create(n, codes, bits, rows, cols, luts, scales, si.ctypes.data)
        if not h:
            raise YsknError(EINVAL, "embedding_create: " + last_error())
        self.handle, self.rows, self.cols = C.c_void_p(h), rows, cols

    @classmethod
    def _from_handle(cls, h, rows, cols):
        e = cls.__new__(cls)
        e.handle, e.rows, e.cols = C.c_void_p(h), rows, cols
        return e

    def lookup(self, tokens, out, stream=None):
        """bf16 bits [M][cols] into `out` (a 16-bit device tensor) for int32 `tokens` [M]."""
        check(lib().yskn_b200_embedding_lookup(self.handle, _ptr(tokens), tokens.shape[0], _ptr(out), _stream(stream)),
              "embedding_lookup")

    def close(self):
        if self.handle:
            lib().yskn_b200_embedding_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def residual_prepare(hidden, projection, norm_weight, eps, inp, inv_rms, gate=None, stream=None):
    """hidden (bf16 bits, [M][cols], updated), projection (f32 or None), norm_weight (bf16
    bits [cols]) -> inp (f32 [M][cols]), inv_rms (f32 [M]), gate (bf16 bits or None)."""
    check(lib().yskn_b200_residual_prepare(_ptr(hidden), _ptr(projection), _ptr(norm_weight), hidden.shape[0],
                                           hidden.shape[1], eps, _ptr(inp), _ptr(inv_rms), _ptr(gate),
                                           _stream(stream)), "residual_prepare")


def gated_product(gate, up, out, stream=None):
    """out = bf16(bf16(silu(bf16(gate))) * bf16(up)) as f32, for f32 [M][n] gate and up."""
    check(lib().yskn_b200_gated_product(_ptr(gate), _ptr(up), gate.shape[0], gate.shape[1], _ptr(out),
                                        _stream(stream)), "gated_product")


def head_select(logits, token=None, top_logits=None, top_ids=None, stream=None):
    """Greedy token (int32 [M]) and top-8 (f32 / int32 [M][8]) of f32 logits [M][n]."""
    check(lib().yskn_b200_head_select(_ptr(logits), logits.shape[0], logits.shape[1], _ptr(token), _ptr(top_logits),
                                      _ptr(top_ids), _stream(stream)), "head_select")


def attention_prep(q, k, v, q_norm, k_norm, positions, eps, query, gate, k_rot, v_rot, stream=None):
    """q f32 [M][n_qh][512], k, v f32 [M][n_kvh][256], norms bf16 bits [256], positions
    int32 [M] -> query, gate (bf16 bits [M][n_qh][256]), k_rot, v_rot (f32 [M][n_kvh][256])."""
    check(lib().yskn_b200_attention_prep(_ptr(q), _ptr(k), _ptr(v), _ptr(q_norm), _ptr(k_norm), _ptr(positions), eps,
                                         q.shape[0], q.shape[1], k.shape[1], _ptr(query), _ptr(gate), _ptr(k_rot),
                                         _ptr(v_rot), _stream(stream)), "attention_prep")


def widen_bf16(src, out, stream=None):
    """out (f32) = the bf16 values of src (16-bit tensor), element count of src."""
    check(lib().yskn_b200_widen_bf16(_ptr(src), src.numel(), _ptr(out), _stream(stream)), "widen_bf16")


def gdn_gates(hidden, inv_rms, wb, wa, gates, stream=None):
    check(lib().yskn_b200_gdn_gates(_ptr(hidden), _ptr(inv_rms), _ptr(wb), _ptr(wa), hidden.shape[0], hidden.shape[1],
                                    _ptr(gates), _stream(stream)), "gdn_gates")


def gdn_gates_heads(hidden, inv_rms, wb, wa, gates, stream=None):
    """yskn_b200_gdn_gates_heads: the gates of the value heads whose rows wb, wa hold."""
    check(lib().yskn_b200_gdn_gates_heads(_ptr(hidden), _ptr(inv_rms), _ptr(wb), _ptr(wa), wb.shape[0],
                                          hidden.shape[0], hidden.shape[1], _ptr(gates), _stream(stream)),
          "gdn_gates_heads")


def gdn_step_heads(qkv, z, gates, conv_w, a_log, dt_bias, norm_w, eps, state, history, out, v_head0, qk_head0,
                   qk_channels, n_commit=None, stream=None):
    """yskn_b200_gdn_step_heads: the step of state.shape[0] value heads from v_head0, with
    the query/key channels of key heads from qk_head0 (qk_channels each)."""
    n_commit = qkv.shape[0] if n_commit is None else n_commit
    check(lib().yskn_b200_gdn_step_heads(_ptr(qkv), _ptr(z), _ptr(gates), _ptr(conv_w), _ptr(a_log), _ptr(dt_bias),
                                         _ptr(norm_w), eps, qkv.shape[0], n_commit, state.shape[0], v_head0,
                                         qk_head0, qk_channels, _ptr(state), _ptr(history), _ptr(out),
                                         _stream(stream)), "gdn_step_heads")


def head_merge(part_logits, part_ids, offsets, token=None, top_logits=None, top_ids=None, stream=None):
    """yskn_b200_head_merge: part_logits f32 / part_ids int32 [n_parts][M][8] (views whose
    first dimension may be strided, the other two dense), offsets the parts' first ids."""
    n_parts, M = part_logits.shape[0], part_logits.shape[1]
    assert part_logits.stride(0) == part_ids.stride(0) and part_logits.stride(1) == 8 and part_ids.stride(1) == 8
    offs = (C.c_int32 * n_parts)(*[int(o) for o in offsets])
    check(lib().yskn_b200_head_merge(_ptr(part_logits), _ptr(part_ids), part_logits.stride(0), offs, n_parts, M,
                                     _ptr(token), _ptr(top_logits), _ptr(top_ids), _stream(stream)), "head_merge")


def gdn_step(qkv, z, gates, conv_w, a_log, dt_bias, norm_w, eps, state, history, out, n_commit=None, stream=None):
    """One Gated DeltaNet pass over qkv.shape[0] rows, committing after n_commit rows
    (default: all of them; 0 = provisional, state and history unchanged)."""
    n_commit = qkv.shape[0] if n_commit is None else n_commit
    check(lib().yskn_b200_gdn_step(_ptr(qkv), _ptr(z), _ptr(gates), _ptr(conv_w), _ptr(a_log), _ptr(dt_bias),
                                   _ptr(norm_w), eps, qkv.shape[0], n_commit, _ptr(state), _ptr(history), _ptr(out),
                                   _stream(stream)), "gdn_step")


def gdn_mixer(hidden, inv_rms, wb, wa, qkv, z, conv_w, a_log, dt_bias, norm_w, eps, state, history, out,
              n_commit=None, stream=None):
    """yskn_b200_gdn_mixer: gdn_gates then gdn_step (with the history) in one launch."""
    n_commit = qkv.shape[0] if n_commit is None else n_commit
    check(lib().yskn_b200_gdn_mixer(_ptr(hidden), _ptr(inv_rms), _ptr(wb), _ptr(wa), hidden.shape[1], _ptr(qkv),
                                    _ptr(z), _ptr(conv_w), _ptr(a_log), _ptr(dt_bias), _ptr(norm_w), eps,
                                    qkv.shape[0], n_commit, _ptr(state), _ptr(history), _ptr(out), _stream(stream)),
          "gdn_mixer")


def gdn_mixer_heads(hidden, inv_rms, wb, wa, qkv, z, conv_w, a_log, dt_bias, norm_w, eps, state, history, out,
                    v_head0, qk_head0, qk_channels, n_commit=None, stream=None):
    """yskn_b200_gdn_mixer_heads: gdn_gates_heads then gdn_step_heads in one launch."""
    n_commit = qkv.shape[0] if n_commit is None else n_commit
    check(lib().yskn_b200_gdn_mixer_heads(_ptr(hidden), _ptr(inv_rms), _ptr(wb), _ptr(wa), hidden.shape[1],
                                          _ptr(qkv), _ptr(z), _ptr(conv_w), _ptr(a_log), _ptr(dt_bias), _ptr(norm_w),
                                          eps, qkv.shape[0], n_commit, state.shape[0], v_head0, qk_head0,
                                          qk_channels, _ptr(state), _ptr(history), _ptr(out), _stream(stream)),
          "gdn_mixer_heads")


def _handles(mats):
    arr = (C.c_void_p * len(mats))(*[m.handle for m in mats])
    return arr


def weighted_sums(mats, act, scales, outs, stream=None):
    """int64 [M][physical_rows] per matrix (yskn_b200_weighted_sums)."""
    M = act.shape[0]
    outp = (C.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    check(lib().yskn_b200_weighted_sums(_handles(mats), len(mats), _ptr(act), _ptr(scales), M, outp, _stream(stream)),
          "weighted_sums")


def weighted_sums_noalloc(mats, act, scales, outs, stream=None):
    """yskn_b200_weighted_sums_noalloc: the same sums with the library allocating nothing
    (scratch in a static device array; M <= 64; calls on one device must not overlap)."""
    M = act.shape[0]
    outp = (C.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    check(lib().yskn_b200_weighted_sums_noalloc(_handles(mats), len(mats), _ptr(act), _ptr(scales), M, outp,
                                                _stream(stream)), "weighted_sums_noalloc")


def weighted_sums_prefix(mat, act, scales, n_rows, out, stream=None):
    check(lib().yskn_b200_weighted_sums_prefix(mat.handle, _ptr(act), _ptr(scales), act.shape[0], n_rows, _ptr(out),
                                               _stream(stream)), "weighted_sums_prefix")


def quantize(x, signs_dev_ptr, act, alpha, scales, row_quantum, stream=None):
    M, K = x.shape
    check(lib().yskn_b200_quantize(_ptr(x), signs_dev_ptr, M, K, _ptr(act), _ptr(alpha), _ptr(scales),
                                   _ptr(row_quantum), _stream(stream)), "quantize")


def rescale(alpha, row_max, scales, row_quantum, stream=None):
    """yskn_b200_rescale: the rows' integer grids from given row maxima of the group scales."""
    M, G = alpha.shape
    check(lib().yskn_b200_rescale(_ptr(alpha), _ptr(row_max), M, G, _ptr(scales), _ptr(row_quantum),
                                  _stream(stream)), "rescale")


TP_HANDLE_BYTES = 64


class TpExchange:
    """This rank's side of the row-parallel exchange (yskn_b200_tp_create / _connect):
    create, swap the handles between ranks (`connect(handles)` takes all of them in rank
    order), then pass it to linear_rowpar."""

    def __init__(self, world, rank, max_physical_rows):
        self._handle_buf = C.create_string_buffer(TP_HANDLE_BYTES)
        self.handle = lib().yskn_b200_tp_create(world, rank, max_physical_rows, self._handle_buf)
        if not self.handle:
            raise YsknError(-1, "tp_create: " + last_error())
        self.world, self.rank = world, rank

    @property
    def ipc_handle(self):
        return self._handle_buf.raw

    def connect(self, handles):
        blob = b"".join(handles)
        if len(blob) != TP_HANDLE_BYTES * self.world:
            raise ValueError("one %d-byte handle per rank expected" % TP_HANDLE_BYTES)
        check(lib().yskn_b200_tp_connect(self.handle, blob), "tp_connect")

    @property
    def area(self):
        """This rank's exchange area as a device address (yskn_b200_tp_area)."""
        return lib().yskn_b200_tp_area(self.handle)

    def connect_peers(self, areas):
        """Connect with the peers' areas given as device addresses in rank order (one
        process driving several devices); this rank's own entry is ignored."""
        if len(areas) != self.world:
            raise ValueError("one area per rank expected")
        arr = (C.c_void_p * self.world)(*[a or 0 for a in areas])
        check(lib().yskn_b200_tp_connect_peers(self.handle, arr), "tp_connect_peers")

    def set_wait(self, seconds):
        """Limit of each wait phase on the peers (yskn_b200_tp_set_wait)."""
        check(lib().yskn_b200_tp_set_wait(self.handle, float(seconds)), "tp_set_wait")

    def close(self):
        if self.handle:
            lib().yskn_b200_tp_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def linear_rowpar(exchange, mat, x_local, y, inv_rms=None, stream=None):
    """yskn_b200_linear_rowpar: the whole output of a row-parallel shard, on every rank."""
    check(lib().yskn_b200_linear_rowpar(exchange.handle, mat.handle, _ptr(x_local), x_local.shape[0], _ptr(inv_rms),
                                        _ptr(y), _stream(stream)), "linear_rowpar")


def linear_rowpar_q8(exchange, mat, act_local, alpha_local, y, stream=None):
    """yskn_b200_linear_rowpar_q8: the whole output of a row-parallel shard from this rank's
    int8 input columns, on every rank."""
    check(lib().yskn_b200_linear_rowpar_q8(exchange.handle, mat.handle, _ptr(act_local), _ptr(alpha_local),
                                           act_local.shape[0], _ptr(y), _stream(stream)), "linear_rowpar_q8")


def linear_rowpar_residual(exchange, mat, hidden, norm_weight, next_signs, act_out, alpha_out, bss_out, x=None,
                           act=None, alpha=None, gate_out=None, stream=None):
    """yskn_b200_linear_rowpar_residual: the row-parallel operator from this rank's input
    columns (x f32, or act/alpha int8) into the whole residual stream and next input."""
    M = (x if x is not None else act).shape[0]
    check(lib().yskn_b200_linear_rowpar_residual(exchange.handle, mat.handle, _ptr(x), _ptr(act), _ptr(alpha), M,
                                                 _ptr(hidden), _ptr(norm_weight), _ptr(next_signs), _ptr(act_out),
                                                 _ptr(alpha_out), _ptr(bss_out), _ptr(gate_out), _stream(stream)),
          "linear_rowpar_residual")


def restore(ws, row_quantum, inv_rms, mat, rotate_out, n_rows, clear_ws, y, stream=None):
    check(lib().yskn_b200_restore(_ptr(ws), _ptr(row_quantum), _ptr(inv_rms), mat.handle, ws.shape[0],
                                  int(rotate_out), n_rows, int(clear_ws), _ptr(y), _stream(stream)), "restore")


def linear_work_bytes(mats, M):
    return lib().yskn_b200_linear_work_bytes(_handles(mats), len(mats), M)


def linear(mats, x, work, ys, inv_rms=None, stream=None):
    yp = (C.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
    check(lib().yskn_b200_linear(_handles(mats), len(mats), _ptr(x), x.shape[0], _ptr(inv_rms), _ptr(work), yp,
                                 _stream(stream)), "linear")


def linear_residual(mat, hidden, norm_weight, next_signs, act_out, alpha_out, bss_out, x=None, act=None,
                    alpha=None, gate_out=None, stream=None):
    """yskn_b200_linear_residual: restore `mat` from x (f32) or act/alpha (int8) into the
    residual stream `hidden` (bf16 as int16) and write the next operator's int8 input."""
    M = (x if x is not None else act).shape[0]
    check(lib().yskn_b200_linear_residual(mat.handle, _ptr(x), _ptr(act), _ptr(alpha), M, _ptr(hidden),
                                          _ptr(norm_weight), _ptr(next_signs), _ptr(act_out), _ptr(alpha_out),
                                          _ptr(bss_out), _ptr(gate_out), _stream(stream)), "linear_residual")


def linear_q8(mats, act, alpha, ys, bss=None, eps=0.0, inv_rms_out=None, stream=None):
    """yskn_b200_linear_q8: the operator from an int8 input (and block sums of squares)."""
    yp = (C.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
    check(lib().yskn_b200_linear_q8(_handles(mats), len(mats), _ptr(act), _ptr(alpha), _ptr(bss), float(eps),
                                    act.shape[0], _ptr(inv_rms_out), yp, _stream(stream)), "linear_q8")


def linear_from_residual(mats, y_prev, hidden_in, hidden_out, norm_weight, eps, ys, gate_out=None, inv_rms_out=None,
                         stream=None):
    """yskn_b200_linear_from_residual: the operator whose input is the residual stream
    hidden_in plus the previous projection's rows y_prev, normalised (norm_weight, eps) and
    quantised in the launch; the updated stream goes to hidden_out."""
    yp = (C.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
    check(lib().yskn_b200_linear_from_residual(_handles(mats), len(mats), _ptr(y_prev), _ptr(hidden_in),
                                               _ptr(hidden_out), _ptr(norm_weight), float(eps), y_prev.shape[0],
                                               _ptr(gate_out), _ptr(inv_rms_out), yp, _stream(stream)),
          "linear_from_residual")


def gated_product_q8(gate, up, signs, act, alpha, stream=None):
    """yskn_b200_gated_product_q8: the MLP product quantised for the down projection."""
    M, n = gate.shape
    check(lib().yskn_b200_gated_product_q8(_ptr(gate), _ptr(up), M, n, _ptr(signs), _ptr(act), _ptr(alpha),
                                           _stream(stream)), "gated_product_q8")


PORTABLE_FN = {"exp": 0, "exp2": 1, "log": 2, "log1p": 3, "sigmoid": 4, "silu": 5, "softplus": 6, "rsqrt": 7,
               "sincos": 8}


def portable_math(name, x, y, y2=None, stream=None):
    """yskn_b200_portable_math: the device portable function `name` over the f32 tensor x
    into y (sincos: cosine into y, sine into y2)."""
    check(lib().yskn_b200_portable_math(PORTABLE_FN[name], _ptr(x), x.numel(), _ptr(y), _ptr(y2), _stream(stream)),
          "portable_math")


def status(stream=None):
    return lib().yskn_b200_status(_stream(stream))


def repack_warp_to_frag(words, frag, rows, seqs, wps, stream=None):
    return lib().yskn_repack_warp_to_frag(_ptr(words), _ptr(frag), rows, seqs, wps, _stream(stream))


def pack(words, layout, physical_rows, cols, bits, out, stream=None):
    check(lib().yskn_b200_pack(_ptr(words), LAYOUTS.get(layout, layout), physical_rows, cols, bits, _ptr(out),
                               _stream(stream)), "pack")


def kv4_attention_work_bytes(M, n_query_heads, length, n_splits=0):
    return lib().yskn_b200_kv4_attention_work_bytes(M, n_query_heads, length, n_splits)


def kv4_attention(q, k_rows, k_scales, v_rows, v_scales, k_codebook, v_codebook, length, work, out, gate=None,
                  v_mean=None, attended=None, n_splits=0, kb=4, stream=None):
    """q, gate, out: bf16 [M][n_qh][256] (passed as int16/bfloat16 tensors); k_rows/v_rows:
    int32 [n_kvh][capacity][8*kb]; scales f32 [n_kvh][capacity]; codebooks bf16 [n_kvh][256]."""
    M, n_qh = q.shape[0], q.shape[1]
    n_kvh, capacity = k_rows.shape[0], k_rows.shape[1]
    check(lib().yskn_b200_kv4_attention(_ptr(q), _ptr(gate), _ptr(k_rows), _ptr(k_scales), _ptr(v_rows),
                                        _ptr(v_scales), _ptr(k_codebook), _ptr(v_codebook), _ptr(v_mean), M, n_qh,
                                        n_kvh, length, capacity, kb, n_splits, _ptr(work), _ptr(attended),
                                        _ptr(out), _stream(stream)), "kv4_attention")


def kv_encode(rows, row_group, tables, gains, mults, kb, vit2, words, scales, means=None, has_mean=None, dest=None,
              stream=None):
    """rows f32 [n][256]; row_group int32 [n]; tables int16 [groups][256]; gains f32 [groups];
    mults f32 [n_mult]; words int32 [*][8*kb]; scales f32 [*]; dest int64 [n] or None."""
    check(lib().yskn_b200_kv_encode(_ptr(rows), _ptr(row_group), rows.shape[0], _ptr(tables), _ptr(gains),
                                    _ptr(means), _ptr(has_mean), _ptr(mults), mults.shape[0], kb, int(vit2),
                                    _ptr(dest), _ptr(words), _ptr(scales), _stream(stream)), "kv_encode")
