"""TEST INFRASTRUCTURE ONLY: ctypes front end of the C oracle (oracle/yskn_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module, as the checker. Each function names the reference code it restates.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libyskn_oracle.so")
RULES = {"splitmix64": 0, "mulberry32_7919_13": 1}
LAYOUTS = {"row": 0, "warp": 1}
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(HERE, f) for f in ("yskn_oracle.c", "kv_oracle.c", "portable_math.c", "Makefile")]
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
            build()
        _lib = C.CDLL(LIB_PATH)
        _lib.orc_f16_to_f32.restype = C.c_float
        _lib.orc_f16_to_f32.argtypes = [C.c_uint16]
        _lib.orc_f32_to_f16.restype = C.c_uint16
        _lib.orc_f32_to_f16.argtypes = [C.c_float]
        _lib.orc_f32_to_bf16.restype = C.c_uint16
        _lib.orc_f32_to_bf16.argtypes = [C.c_float]
        _lib.orc_state.restype = C.c_uint16
        _lib.orc_state.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int, C.c_int64, C.c_int64, C.c_int]
        _lib.orc_hadamard512.argtypes = [C.c_void_p]
        for name in ("exp", "exp2", "log", "log1p", "sigmoid", "silu", "softplus", "rsqrt", "sqrt_rn"):
            f = getattr(_lib, "orc_pm_" + name)
            f.restype = C.c_float
            f.argtypes = [C.c_float]
        for name in ("exp_d", "log_d"):
            f = getattr(_lib, "orc_pm_" + name)
            f.restype = C.c_double
            f.argtypes = [C.c_double]
        _lib.orc_pm_sincos.argtypes = [C.c_float, C.c_void_p, C.c_void_p]
        _lib.orc_pm_map.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64]
        _lib.orc_pm_sincos_map.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]
    return _lib


def _p(a):
    return C.c_void_p(a.ctypes.data)


class OracleError(RuntimeError):
    pass


def _check(rc, what):
    if rc == -2:
        raise OverflowError("%s: compressed integer accumulation exceeds i64" % what)
    if rc != 0:
        raise OracleError("%s failed (%d)" % (what, rc))


# ---------------------------------------------------------------- portable math --
# crates/yskn-ref/src/portable_math.rs restated in portable_math.c: the scalar
# reference computes every exponential, logarithm, inverse square root and rotary
# sine/cosine with these functions, so the layer oracles below call them too.
_PM_FN = {"exp": 0, "exp2": 1, "log": 2, "log1p": 3, "sigmoid": 4, "silu": 5, "softplus": 6, "rsqrt": 7,
          "sqrt_rn": 8}


def pm(name, x):
    """Elementwise portable function `name` over float32 values (same shape out)."""
    shape = np.shape(x)
    a = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1))
    out = np.empty_like(a)
    _check(lib().orc_pm_map(_PM_FN[name], _p(a), _p(out), C.c_int64(a.size)), "portable " + name)
    return out.reshape(shape) if shape else np.float32(out[0])


def pm_scalar(name, x):
    """One portable binary32 function value (portable_math.rs), or exp_d / log_d in binary64."""
    return getattr(lib(), "orc_pm_" + name)(x)


def pm_sincos(angle):
    """portable_math.rs:406-434 over float32 angles -> (cos, sin) float32 arrays."""
    shape = np.shape(angle)
    a = np.ascontiguousarray(np.asarray(angle, np.float32).reshape(-1))
    c, s = np.empty_like(a), np.empty_like(a)
    _check(lib().orc_pm_sincos_map(_p(a), _p(c), _p(s), C.c_int64(a.size)), "portable sincos")
    return c.reshape(shape), s.reshape(shape)


def signs(rule, seed, offset, n):
    """crates/yskn-format/src/signs.rs:12-38."""
    out = np.empty(n, np.int8)
    _check(lib().orc_signs(C.c_int(RULES[rule]), C.c_uint64(seed), C.c_uint64(offset), C.c_int64(n), _p(out)), "signs")
    return out


def tensor_signs(rot, n):
    return None if rot is None else signs(rot["rule"], rot["seed"], rot["offset"], n)


def f16_to_f32(bits):
    return lib().orc_f16_to_f32(int(bits))


def f32_to_f16(value):
    return lib().orc_f32_to_f16(float(value))


def f32_to_bf16(value):
    return lib().orc_f32_to_bf16(float(value))


def states(words, layout, phys_rows, cols, bits):
    """tensor.rs:385-428: uint16 [phys_rows, cols/256, 128]."""
    words = np.ascontiguousarray(words, np.uint32)
    out = np.empty((phys_rows, cols // 256, 128), np.uint16)
    _check(lib().orc_states_all(_p(words), C.c_int(LAYOUTS[layout]), C.c_int64(phys_rows), C.c_int64(cols),
                                C.c_int(bits), _p(out)), "states")
    return out


def quantize_weight_table(lut16, scale16):
    """compressed_linear.rs:138-158 -> (int8 lut8[8192], f32 tau[N])."""
    lut16 = np.ascontiguousarray(lut16, np.uint16)
    scale16 = np.ascontiguousarray(scale16, np.uint16)
    lut8 = np.empty(8192, np.int8)
    tau = np.empty(scale16.size, np.float32)
    _check(lib().orc_quantize_weight_table(_p(lut16), _p(scale16), C.c_int64(scale16.size), _p(lut8), _p(tau)),
           "quantize_weight_table")
    return lut8, tau


def hadamard512(v):
    v = np.array(v, np.float32).copy()
    lib().orc_hadamard512(_p(v))
    return v


def embedding_rows(parts, tokens, signs_in):
    """docs/spec/02_COMPRESSED_LINEAR.md:271-303 (src/q35_kernels.cu:1501-1574): the
    bf16 bits [len(tokens), cols] of coded embedding rows. parts: the main table and up
    to two residual tables, each (words, layout, physical_rows, cols, bits, lut16,
    scale16); every part is decoded with its own table and row scale, the parts are
    added in order, then per 512 columns H512 (ascending strides), * 1/sqrt(512) and the
    main table's input signs, one rounding to bf16. Every float32 operation rounds once
    (numpy float32 arithmetic, no fused multiply-add)."""
    signs = np.asarray(signs_in, np.int8).astype(np.float32)
    cols = signs.size
    decoded = []
    for words, layout, phys, pcols, bits, lut16, scale16 in parts:
        assert pcols == cols
        st = states(words, layout, phys, cols, bits).reshape(phys, cols // 2)
        table = np.asarray(lut16, np.uint16).view("<f2").astype(np.float32).reshape(4096, 2)
        scale = np.asarray(scale16, np.uint16).view("<f2").astype(np.float32)
        decoded.append((st, table, scale))
    out = np.empty((len(tokens), cols), np.uint16)
    for m, t in enumerate(tokens):
        v = None
        for st, table, scale in decoded:
            part = table[st[t]].reshape(cols) * scale[t]
            v = part if v is None else v + part
        for b in range(0, cols, 512):
            h = hadamard512(v[b:b + 512])
            y = (h * np.float32(0.044194173824159216)) * signs[b:b + 512]
            out[m, b:b + 512] = [f32_to_bf16(x) for x in y]
    return out


def bf16_bits(x):
    """Round-to-nearest-even float32 -> bf16 bits, vectorised (finite values; NaN stays NaN)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    return np.where(nan, np.uint16(0x7FC0), r)


def bf16_float(bits):
    return (np.asarray(bits, np.uint32) << np.uint32(16)).view(np.float32)


def block_sum_squares(values):
    """docs/spec/05_RESIDUAL_NORM_MLP.md:70-101 (src/q35_kernels.cu:1447-1458): 128 partial
    sums over four elements 128 apart, an XOR reduction with offsets 16..1 in each group
    of 32, the four group sums added in order from +0."""
    v = np.asarray(values, np.float32)
    partial = np.zeros(128, np.float32)
    for j in range(4):
        x = v[128 * j:128 * j + 128]
        partial = partial + x * x
    result = np.float32(0.0)
    for g in range(4):
        lanes = partial[32 * g:32 * g + 32].copy()
        for off in (16, 8, 4, 2, 1):
            lanes = lanes + lanes[np.arange(32) ^ off]
        result = np.float32(result + lanes[0])
    return result


def residual_prepare(hidden_bits, projection, norm_bits, eps):
    """docs/spec/05_RESIDUAL_NORM_MLP.md:53-141, residual_norm_mlp.rs:14-61,120-135 for one
    row: hidden = bf16(hidden + bf16(projection)) (no addition when projection is None),
    the exact sum of squares, inverse RMS = rsqrt(total/cols + eps) with the portable
    rsqrt (rounded square root, rounded division), input = hidden * (1 + norm weight) in
    float32, and the gate copy bf16(input). Returns (hidden_bits, input_f32, inv_rms,
    gate_bits)."""
    h = bf16_float(hidden_bits)
    if projection is not None:
        h = bf16_float(bf16_bits(h + bf16_float(bf16_bits(projection))))
    cols = h.size
    total = np.float32(0.0)
    for b in range(0, cols, 512):
        total = np.float32(total + block_sum_squares(h[b:b + 512]))
    mean = np.float32(np.float32(total / np.float32(cols)) + np.float32(eps))
    inv_rms = pm("rsqrt", mean)
    gain = np.float32(1.0) + bf16_float(norm_bits)
    x = h * gain
    return bf16_bits(h), x, inv_rms, bf16_bits(x)


def gated_product(gate, up):
    """docs/spec/05_RESIDUAL_NORM_MLP.md:156-176, residual_norm_mlp.rs:137-156:
    bf16(bf16(silu(g)) * u) with g = bf16(gate), u = bf16(up) and the portable silu
    g / (1 + exp(-g)), float32 arithmetic."""
    g = bf16_float(bf16_bits(gate))
    u = bf16_float(bf16_bits(up))
    silu = bf16_float(bf16_bits(pm("silu", g)))
    return bf16_float(bf16_bits(silu * u))


def head_select(logits, k=8):
    """docs/spec/06_OUTPUT_HEAD_SAMPLER.md:31-64,240-250: the first k of the order (larger
    logit, smaller id) among logits that beat the starting point (-FLT_MAX, INT_MAX)
    (NaN and -inf never do), padded with that starting point. Returns (token, values, ids)."""
    l = np.asarray(logits, np.float32)
    ids = np.arange(l.size)
    ok = ~np.isnan(l) & (l >= np.float32(-3.4028234663852886e38))
    vals, idx = l[ok], ids[ok]
    order = np.lexsort((idx, -vals))[:k]
    top_v = np.full(k, np.float32(-3.4028234663852886e38), np.float32)
    top_i = np.full(k, 2**31 - 1, np.int64)
    top_v[:order.size] = vals[order]
    top_i[:order.size] = idx[order]
    return int(top_i[0]), top_v, top_i


ROPE_FREQ_BITS = [  # docs/spec/04_ATTENTION.md:42-52
    0x3f800000, 0x3f1ab32b, 0x3ebaf81b, 0x3e61f835, 0x3e088d77, 0x3da50956, 0x3d47763f, 0x3cf11177,
    0x3c91ad39, 0x3c301052, 0x3bd4ca15, 0x3b80967d, 0x3b1b690d, 0x3abbd3ed, 0x3a6301e2, 0x3a092e02,
    0x39a5cb60, 0x394860c1, 0x38f22ce2, 0x3892587e, 0x3830df52, 0x37d5c441, 0x37812dab, 0x371c1fc4,
    0x36bcb0c1, 0x36640cc6, 0x3609cf4a, 0x35a68e4c, 0x35494c57, 0x34f3499d, 0x3493048e, 0x3431af44]


def cache_signs():
    """docs/spec/04_ATTENTION.md:80-88: the sign of each of the 256 cache channels."""
    x = np.arange(1, 257, dtype=np.uint64)
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & np.uint64(0xFFFFFFFF)
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & np.uint64(0xFFFFFFFF)
    x ^= x >> np.uint64(16)
    return np.where(x & np.uint64(1), np.float32(-1.0), np.float32(1.0)).astype(np.float32)


def rotate_cache(x):
    """docs/spec/04_ATTENTION.md:90-100: signs, H256 with distances 1..128, * 1/16."""
    a = np.asarray(x, np.float32) * cache_signs()
    idx = np.arange(256)
    for d in (1, 2, 4, 8, 16, 32, 64, 128):
        o = a[idx ^ d]
        a = np.where((idx & d) != 0, o - a, a + o).astype(np.float32)
    return a * np.float32(0.0625)


def _xor_sum32(v):
    a = np.asarray(v, np.float32).copy()
    for off in (16, 8, 4, 2, 1):
        a = a + a[np.arange(32) ^ off]
    return a[0]


def normalize_head(y, weight_bits, eps):
    """docs/spec/04_ATTENTION.md:27-37; attention.rs:732-755 (the portable rsqrt:
    the rounded square root, then a rounded division)."""
    y = np.asarray(y, np.float32)
    total = np.float32(0.0)
    for g in range(8):
        total = np.float32(total + _xor_sum32(y[32 * g:32 * g + 32] * y[32 * g:32 * g + 32]))
    inv = pm("rsqrt", np.float32(np.float32(total / np.float32(256.0)) + np.float32(eps)))
    return bf16_float(bf16_bits((y * inv) * (np.float32(1.0) + bf16_float(weight_bits))))


def rope(n, position):
    """docs/spec/04_ATTENTION.md:54-66; attention.rs:757-775 (the portable sincos)."""
    freq = np.array(ROPE_FREQ_BITS, np.uint32).view(np.float32)
    arg = np.float32(position) * freq
    cos, sin = pm_sincos(arg)
    c = bf16_float(bf16_bits(cos))
    s = bf16_float(bf16_bits(sin))
    r = np.asarray(n, np.float32).copy()
    a, b = r[:32].copy(), r[32:64].copy()
    r[:32] = bf16_float(bf16_bits(bf16_float(bf16_bits(a * c)) + bf16_float(bf16_bits(-b * s))))
    r[32:64] = bf16_float(bf16_bits(bf16_float(bf16_bits(b * c)) + bf16_float(bf16_bits(a * s))))
    return r


def attention_prep(q, k, v, q_norm_bits, k_norm_bits, position, eps):
    """One row (docs/spec/04_ATTENTION.md:15-106): q [n_qh][512] (query then gate channels
    per head), k, v [n_kvh][256] -> (query bf16 bits, gate bf16 bits, k f32, v f32)."""
    q = np.asarray(q, np.float32)
    query = np.empty((q.shape[0], 256), np.uint16)
    gate = bf16_bits(q[:, 256:])
    for h in range(q.shape[0]):
        n = rope(normalize_head(bf16_float(bf16_bits(q[h, :256])), q_norm_bits, eps), position)
        query[h] = bf16_bits(rotate_cache(n))
    k_out = np.stack([rotate_cache(rope(normalize_head(bf16_float(bf16_bits(x)), k_norm_bits, eps), position))
                      for x in np.asarray(k, np.float32)])
    v_out = np.stack([rotate_cache(bf16_float(bf16_bits(x))) for x in np.asarray(v, np.float32)])
    return query, gate, k_out, v_out


def _sum4(v):
    return np.float32(np.float32(np.float32(v[0] + v[1]) + v[2]) + v[3])


def _squares128(x):
    x = np.asarray(x, np.float32)
    return _sum4([_xor_sum32(x[32 * g:32 * g + 32] * x[32 * g:32 * g + 32]) for g in range(4)])


def _silu(x):
    """portable_math.rs:201-203: x / (1 + exp(-x)) with the portable exp."""
    return pm("silu", x)


def gdn_gates(x_bits, inv_rms, wb_bits, wa_bits):
    """docs/spec/03_GATED_DELTANET.md:57-76, gated_deltanet.rs:612-644 for one row: the
    gates of wb's rows, then wa's (96 at the 27B shape). Partition p of 128 sums elements
    8p + 1024c + e (e < 8) over ceil(hidden / 1024) chunks, skipping indices past the end."""
    x = bf16_float(x_bits)
    w = np.concatenate([bf16_float(wb_bits), bf16_float(wa_bits)])
    out = np.empty(w.shape[0], np.float32)
    p = np.arange(128)
    n = x.size
    for o in range(w.shape[0]):
        partial = np.zeros(128, np.float32)
        for chunk in range(-(-n // 1024)):
            for e in range(8):
                i = 8 * p + 1024 * chunk + e
                ok = i < n
                j = np.minimum(i, n - 1)
                partial = np.where(ok, partial + w[o, j] * x[j], partial).astype(np.float32)
        out[o] = bf16_float(bf16_bits(_sum4([_xor_sum32(partial[32 * g:32 * g + 32]) for g in range(4)]) *
                                      np.float32(inv_rms)))
    return out


def gdn_step(qkv, z, gates, conv_bits, a_log_bits, dt_bias_bits, norm_bits, eps, state, history_bits,
             n_commit=None):
    """docs/spec/03_GATED_DELTANET.md:78-186 and gated_deltanet.rs:332-577, ordinary
    causal rows, numpy float32 with the reference's portable rsqrt/exp/sigmoid/softplus/
    silu. Commits after n_commit rows (default all; 0 = provisional). Returns (out
    [M][6144], the committed state [48][128][128], the committed history bits [3][10240])."""
    qkv = np.asarray(qkv, np.float32)
    M = qkv.shape[0]
    proj = bf16_float(bf16_bits(qkv))
    hist = bf16_float(history_bits)
    cw = bf16_float(conv_bits).reshape(-1, 4)
    past = lambda r: hist[3 + r] if r < 0 else proj[r]
    n_commit = M if n_commit is None else n_commit
    state = np.array(state, np.float32)
    saved = state.copy()
    out = np.empty((M, 48 * 128), np.float32)
    a_log, dt_bias, norm_w = bf16_float(a_log_bits), bf16_float(dt_bias_bits), bf16_float(norm_bits)
    for row in range(M):
        a = cw[:, 0] * past(row - 3)
        a = a + cw[:, 1] * past(row - 2)
        a = a + cw[:, 2] * past(row - 1)
        a = a + cw[:, 3] * past(row)
        conv = bf16_float(bf16_bits(_silu(bf16_float(bf16_bits(a)))))
        for vh in range(48):
            kh = vh // 3
            q = conv[128 * kh:128 * kh + 128]
            k = conv[2048 + 128 * kh:2048 + 128 * kh + 128]
            v = conv[4096 + 128 * vh:4096 + 128 * vh + 128]
            rq = pm("rsqrt", np.float32(_squares128(q) + np.float32(1e-6)))
            rk = pm("rsqrt", np.float32(_squares128(k) + np.float32(1e-6)))
            query = (q * rq) * np.float32(0.08838834764831845)
            key = k * rk
            g = np.asarray(gates[row], np.float32)
            beta = bf16_float(bf16_bits(pm("sigmoid", g[vh])))
            x = np.float32(g[48 + vh] + dt_bias[vh])
            sp = pm("softplus", x)
            decay = pm("exp", np.float32(-pm("exp", a_log[vh]) * sp))
            R = state[vh]
            parts = []
            for grp in range(4):
                acc = np.zeros(128, np.float32)
                for r in range(32):
                    i = 32 * grp + r
                    R[i] = R[i] * decay
                    acc = acc + R[i] * key[i]
                parts.append(acc)
            correction = (v - _sum4(parts)) * beta
            parts = []
            for grp in range(4):
                acc = np.zeros(128, np.float32)
                for r in range(32):
                    i = 32 * grp + r
                    R[i] = R[i] + key[i] * correction
                    acc = acc + R[i] * query[i]
                parts.append(acc)
            core = bf16_float(bf16_bits(_sum4(parts)))
            inv = pm("rsqrt", np.float32(np.float32(_squares128(core) / np.float32(128.0)) + np.float32(eps)))
            normalized = bf16_float(bf16_bits(norm_w * bf16_float(bf16_bits(core * inv))))
            out[row, 128 * vh:128 * vh + 128] = bf16_float(bf16_bits(normalized *
                                                                     _silu(z[row, 128 * vh:128 * vh + 128])))
        if row + 1 == n_commit:
            saved = state.copy()
    if n_commit == 0:
        return out, saved, np.asarray(history_bits, np.uint16).copy()
    rows = [past(n_commit - 3 + a) for a in range(3)]
    return out, saved, bf16_bits(np.stack(rows))


def quantize_activation(x, signs_in):
    """compressed_linear.rs:57-135 for each row of x [M, Kc] -> (act8, alpha, A, row_quantum)."""
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    signs_in = np.ascontiguousarray(signs_in, np.int8)
    M, K = x.shape
    G = K // 512
    act8 = np.empty((M, K), np.int8)
    alpha = np.empty((M, G), np.float32)
    A = np.empty((M, G), np.int32)
    rq = np.empty(M, np.float32)
    _check(lib().orc_quantize_activation(_p(x), _p(signs_in), C.c_int64(M), C.c_int64(K), _p(act8), _p(alpha),
                                         _p(A), _p(rq)), "quantize_activation")
    return act8, alpha, A, rq


def weighted_sums(words, layout, phys_rows, cols, bits, lut8, act8, A, rows=None):
    """compressed_linear.rs:205-252 (scalar, checked) -> int64 [M, rows]."""
    words = np.ascontiguousarray(words, np.uint32)
    act8 = np.ascontiguousarray(np.atleast_2d(act8), np.int8)
    A = np.ascontiguousarray(np.atleast_2d(A), np.int32)
    lut8 = np.ascontiguousarray(lut8, np.int8)
    rows = phys_rows if rows is None else rows
    M = act8.shape[0]
    out = np.empty((M, rows), np.int64)
    _check(lib().orc_weighted_sums(_p(words), C.c_int(LAYOUTS[layout]), C.c_int64(phys_rows), C.c_int64(cols),
                                   C.c_int(bits), _p(lut8), _p(act8), _p(A), C.c_int64(M), C.c_int64(rows), _p(out)),
           "weighted_sums")
    return out


def fast_weighted_sums(words, layout, phys_rows, cols, bits, lut8, act8, A, rows=None, threads=None):
    """crates/yskn-engine/src/kernel.rs:92-233 + pool.rs:248-344 restated with pthreads."""
    words = np.ascontiguousarray(words, np.uint32)
    act8 = np.ascontiguousarray(np.atleast_2d(act8), np.int8)
    A = np.ascontiguousarray(np.atleast_2d(A), np.int32)
    lut8 = np.ascontiguousarray(lut8, np.int8)
    rows = phys_rows if rows is None else rows
    threads = threads or os.cpu_count() or 1
    M = act8.shape[0]
    out = np.empty((M, rows), np.int64)
    _check(lib().orc_fast_weighted_sums(_p(words), C.c_int(LAYOUTS[layout]), C.c_int64(phys_rows), C.c_int64(cols),
                                        C.c_int(bits), _p(lut8), _p(act8), _p(A), C.c_int64(M), C.c_int64(rows),
                                        _p(out), C.c_int(threads)), "fast_weighted_sums")
    return out


def restore(ws, row_quantum, tau, signs_out=None, inv_rms=None, rows=None):
    """compressed_linear.rs:288-370 -> float32 [M, rows]."""
    ws = np.ascontiguousarray(np.atleast_2d(ws), np.int64)
    M, N = ws.shape
    rows = N if rows is None else rows
    rq = np.ascontiguousarray(row_quantum, np.float32).reshape(M)
    tau = np.ascontiguousarray(tau, np.float32)
    so = None if signs_out is None else np.ascontiguousarray(signs_out, np.int8)
    if so is not None and so.size != N:
        raise OracleError("restore: output signs must have one entry per physical row")
    if tau.size != N:
        raise OracleError("restore: one row scale per physical row")
    ir = None if inv_rms is None else np.ascontiguousarray(inv_rms, np.float32).reshape(M)
    out = np.empty((M, rows), np.float32)
    _check(lib().orc_restore(_p(ws), C.c_int64(M), C.c_int64(N), _p(rq), None if ir is None else _p(ir), _p(tau),
                             None if so is None else _p(so), C.c_int64(rows), _p(out)), "restore")
    return out


def repack_warp_to_frag(words, rows, seqs, wps):
    """src/repack.cu:10-18."""
    words = np.ascontiguousarray(words, np.uint32)
    out = np.empty_like(words)
    _check(lib().orc_repack_warp_to_frag(_p(words), _p(out), C.c_int(rows), C.c_int(seqs), C.c_int(wps)), "repack")
    return out


def linear(words, layout, phys_rows, cols, bits, lut16, scale16, x, signs_in, signs_out=None, inv_rms=None,
           rows=None):
    """The whole operator y = D_out H (M (H D_in x)) as CompressedLinear::project
    (compressed_linear.rs:254-285) runs it."""
    lut8, tau = quantize_weight_table(lut16, scale16)
    act8, _, A, rq = quantize_activation(x, signs_in)
    ws = weighted_sums(words, layout, phys_rows, cols, bits, lut8, act8, A)
    return restore(ws, rq, tau, signs_out, inv_rms, rows)
