"""TEST INFRASTRUCTURE ONLY: seeded synthetic `.yskn` containers.

* `tiny_container()` writes the reference's small test file again, byte for byte,
  restating the generator of tools/yskn_fixture.py:31-93 (splitmix64 streams,
  1/4096-step uniforms, four tensors). Its SHA-256 is pinned by docs/FORMAT.md:252
  (3f4a4886...), which is how tests know this writer is exact.
* `synthetic()` restates the single-matrix fixture of the reference's kernel tests,
  crates/yskn-engine/tests/fixture/mod.rs:47-114 (seed 0x31875bde0219faff; table
  values (r % 2049)/1024 - 1; row scales (row - P/2)/128).
* `model_matrix()` / `normal()` (the benchmark's 27B-shape matrices and activations)
  are the package's own generators (yskn_b200/synthetic.py), re-exported here.
"""
import numpy as np

from container import write_container
from yskn_b200.synthetic import GOLDEN, model_matrix, normal, stream64  # noqa: F401


def uniform(seed, n, lo, hi):
    u = (stream64(seed, n) >> np.uint64(52)).astype(np.float64) / 4096.0
    return lo + (hi - lo) * u


def bf16_bits(x):
    return (np.asarray(x, np.float32).view("<u4") >> np.uint32(16)).astype("<u2")


TINY_TENSORS = [  # name, role, rows, cols, bits, layout, rule, seed, output rotation
    ("tiny.body6", "body", 512, 512, 6, "warp", "mulberry32_7919_13", 7, True),
    ("tiny.body8", "body", 512, 1024, 8, "warp", "splitmix64", 11, True),
    ("tiny.head", "head", 64, 512, 8, "warp", "mulberry32_7919_13", 7, False),
    ("tiny.embed", "embedding", 96, 512, 6, "row", "mulberry32_7919_13", 7, False),
]


def tiny_container():
    blobs, tensors, vectors = [], [], []

    def blob(b):
        blobs.append(b)
        return {"$blob": len(blobs) - 1}

    for i, (name, role, rows, cols, bits, layout, rule, seed, out_rot) in enumerate(TINY_TENSORS):
        n_words = rows * (cols // 256) * 4 * bits
        words = (stream64(1000 + i, n_words) & np.uint64(0xFFFFFFFF)).astype("<u4")
        lut = uniform(2000 + i, 8192, -3.0, 3.0).astype("<f2")
        scale = uniform(3000 + i, rows, 0.01, 0.03).astype("<f2")
        d = dict(name=name, role=role, rows=rows, cols=cols, physical_rows=rows, l=12, d=2, t=256, bits=bits,
                 start="zero", layout=layout,
                 rot_in=dict(kind="H512", m=cols // 512, sign_seed=seed, sign_offset=0, qm_off=0, rule=rule),
                 rot_out=(dict(kind="H512", m=rows // 512, sign_seed=seed, sign_offset=cols, qm_off=0, rule=rule)
                          if out_rot else None),
                 rar=None, bias_off=0, proxy=0.0, encoder="test data (pseudo-random, not a model)")
        d["stream_off"] = blob(words.tobytes())
        d["stream_bytes"] = 4 * n_words
        d["lut_off"] = blob(lut.tobytes())
        d["scale_off"] = blob(scale.tobytes())
        tensors.append(d)
    v = uniform(4000, 512, -2.0, 2.0).astype(np.float32)
    vectors.append(dict(name="tiny.norm", off=blob(bf16_bits(v).tobytes()), n=512, dtype="bf16"))
    h = uniform(4001, 8, -2.0, 2.0).astype("<f2")
    vectors.append(dict(name="tiny.half", off=blob(h.tobytes()), n=8, dtype="f16"))
    model = dict(arch="test", layers=0, hidden=512, ffn=512, heads=1, kv_heads=1, head_dim=512, vocab=96, eps=1e-6,
                 rope_theta=10000.0, tie_embeddings=False, source="test data of tools/yskn_fixture.py (not a model)")
    return write_container(model, tensors, vectors, blobs, 4096, 64)


def embedding_container(rows, cols, parts):
    """A container of coded embedding tables (role embedding, row layout, no output
    rotation): parts = [(name, bits, seed, rot_in)], rot_in = (rule, sign_seed, offset).
    Codes are seeded random words (every bit string is a valid code, docs/FORMAT.md:
    137-138), tables uniform in [-3, 3] and row scales in [0.01, 0.03], as binary16."""
    blobs, tensors = [], []

    def blob(b):
        blobs.append(b)
        return {"$blob": len(blobs) - 1}

    for name, bits, seed, (rule, sign_seed, offset) in parts:
        n_words = rows * (cols // 256) * 4 * bits
        words = (stream64(seed, n_words) & np.uint64(0xFFFFFFFF)).astype("<u4")
        lut = uniform(seed + 1, 8192, -3.0, 3.0).astype("<f2")
        scale = uniform(seed + 2, rows, 0.01, 0.03).astype("<f2")
        tensors.append(dict(name=name, role="embedding", rows=rows, cols=cols, bits=bits, layout="row",
                            rot_in=dict(kind="H512", m=cols // 512, sign_seed=sign_seed, sign_offset=offset,
                                        rule=rule),
                            rot_out=None, stream_off=blob(words.tobytes()), stream_bytes=4 * n_words,
                            lut_off=blob(lut.tobytes()), scale_off=blob(scale.tobytes())))
    return write_container(dict(arch="test"), tensors, [], blobs, 4096, 256)


TINY_SHA256 = "3f4a48866f6a1751beabc3b9a8d06088672a3db0aa0a4c3f96e1877cb448d393"


class FixtureRandom:
    """tests/fixture/mod.rs:47-53: add the golden gamma, then mix; low 32 bits."""

    def __init__(self, seed):
        self.state = np.uint64(seed)

    def take(self, n):
        out = stream64(self.state, n)
        with np.errstate(over="ignore"):
            self.state = self.state + np.uint64(n) * GOLDEN
        return (out & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def _f16_bits(values):
    return np.asarray(values, np.float32).astype("<f2").view("<u2")


def synthetic(bits, layout, rows, physical_rows, cols, output_rotation, stream_offset_pad=0):
    """tests/fixture/mod.rs:57-114 (one tensor named `linear`)."""
    data_offset = 4096
    stream_bytes = physical_rows * (cols // 256) * bits * 16
    rnd = FixtureRandom(0x31875BDE0219FAFF)
    stream = rnd.take(stream_bytes).astype(np.uint8)
    table = (rnd.take(8192) % 2049).astype(np.float32) / np.float32(1024.0) - np.float32(1.0)
    scales = (np.arange(physical_rows, dtype=np.float32) - np.float32(physical_rows / 2.0)) / np.float32(128.0)
    blobs = [stream.tobytes(), _f16_bits(table).tobytes(), _f16_bits(scales).tobytes()]
    t = {"name": "linear", "role": "body" if output_rotation else "head", "rows": rows,
         "physical_rows": physical_rows, "cols": cols, "bits": bits, "layout": layout,
         "stream_off": {"$blob": 0}, "stream_bytes": stream_bytes, "lut_off": {"$blob": 1},
         "scale_off": {"$blob": 2},
         "rot_in": {"kind": "H512", "m": cols // 512, "sign_seed": 91, "sign_offset": 13, "rule": "splitmix64"},
         "rot_out": ({"kind": "H512", "m": rows // 512, "sign_seed": 7, "sign_offset": cols,
                      "rule": "mulberry32_7919_13"} if output_rotation else None)}
    model = {"source": "synthetic integration test; no model weights"}
    return write_container(model, [t], [], blobs, data_offset, 1)
