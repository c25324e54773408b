"""Seeded synthetic inputs of the benchmark workloads (no weights or caches are
shipped with the reference; every bit string is a valid code, docs/FORMAT.md:137-138).

* `model_matrix()`: a 27B-shape compressed matrix: uniformly random warp-layout code
  words, an N(0,1)-shaped fp16 value table and fp16 row scales near 0.02 (so scale *
  table has a standard deviation near 0.02).
* `normal()`: N(0,1) activations.
* `kv_cache()`: packed 4-bit KV rows (uniformly random fields), row scales and the
  BF16 codebook of the synthetic KVQP profile of the reference's tests
  (crates/yskn-ref/tests/support/kv_profile.rs:19-79: table codes
  (s*73 + 19) % 2049 - 1024, gain 257/256).
All streams are splitmix64 (tools/yskn_fixture.py and the reference's test fixtures
use the same generator).
"""
import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def _mix(z):
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def stream64(seed, n, first=1):
    """Outputs first..first+n-1 of the splitmix64 sequence started at `seed`."""
    k = np.arange(first, first + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix(np.uint64(seed) + k * GOLDEN)


def f16_bits(values):
    return np.asarray(values, np.float32).astype("<f2").view("<u2")


def _unit(seed, n):
    return (stream64(seed, n) >> np.uint64(11)).astype(np.float64) / 2.0 ** 53


def model_tables(physical_rows, seed):
    """(fp16 table bits [8192], fp16 row scale bits [physical_rows]) of model_matrix."""
    r = np.sqrt(-2.0 * np.log(np.maximum(_unit(seed + 1, 4096), 1e-300)))
    u2 = _unit(seed + 2, 4096)
    table = np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)]).astype(np.float32)
    scales = (0.02 * (1.0 + 0.2 * (_unit(seed + 3, physical_rows) - 0.5))).astype(np.float32)
    return f16_bits(table), f16_bits(scales)


def model_matrix(rows, cols, bits, seed, physical_rows=None):
    """(warp-layout code words u32, fp16 table bits [8192], fp16 row scale bits [phys])."""
    phys = physical_rows or rows
    n_words = phys * (cols // 256) * 4 * bits
    words = (stream64(seed, n_words) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    return (words,) + model_tables(phys, seed)


def normal(seed, n):
    """Deterministic N(0,1) float32 samples (Box-Muller on splitmix uniforms)."""
    half = (n + 1) // 2
    r = np.sqrt(-2.0 * np.log(np.maximum(_unit(seed, half), 1e-300)))
    u2 = (stream64(seed ^ 0x5555, half) >> np.uint64(11)).astype(np.float64) / 2.0 ** 53
    return np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)])[:n].astype(np.float32)


def kv_codebook_bf16():
    """bfloat(reconstruction(state)) of the synthetic profile's table, 256 entries."""
    codes = ((np.arange(256) * 73 + 19) % 2049 - 1024).astype(np.float32)
    rec = (codes * np.float32(0.00390625)) * np.float32(257.0 / 256.0)
    u = rec.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def kv_cache(n_kv_heads, ctx, seed):
    """One layer's packed 4-bit cache: (K words, K scales, V words, V scales), words
    [n_kv_heads][ctx][32] u32, scales [n_kv_heads][ctx] f32 uniform in [0.02, 0.2] (keys)
    and [0.01, 0.1] (values)."""
    n = n_kv_heads * ctx * 32
    kw = (stream64(seed, n) & np.uint64(0xFFFFFFFF)).astype(np.uint32).reshape(n_kv_heads, ctx, 32)
    vw = (stream64(seed + 1, n) & np.uint64(0xFFFFFFFF)).astype(np.uint32).reshape(n_kv_heads, ctx, 32)
    ks = (0.02 + 0.18 * _unit(seed + 2, n_kv_heads * ctx)).astype(np.float32).reshape(n_kv_heads, ctx)
    vs = (0.01 + 0.09 * _unit(seed + 3, n_kv_heads * ctx)).astype(np.float32).reshape(n_kv_heads, ctx)
    return kw, ks, vw, vs
