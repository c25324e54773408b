"""Regenerate the golden fixtures in this folder from the reference project.

    python tests/golden/make_golden.py /path/to/reference

Run in a container that has the reference checkout; the GPU box never runs it.
It writes:
  tiny_expected.json      the values the reference pins for its test file
                          (tools/testdata/tiny_expected.json), copied as data;
  synthetic_decode.json   for every (bits, layout, shape) of the reference's kernel
                          tests (crates/yskn-engine/tests/linear.rs:11-16), the
                          SHA-256 of the trellis states and of the engine's int8
                          table, computed by the reference's own Python reader
                          tools/yskn_decode.py (states(), value_table(engine_table=True))
                          on the containers oracle/fixtures.py::synthetic() writes.
"""
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import fixtures  # noqa: E402

SHAPES = [(17, 32, 512), (65, 96, 1024), (17, 32, 5120), (13, 16, 512), (9, 11, 512)]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref):
    with open(os.path.join(ref, "tools", "testdata", "tiny_expected.json")) as f:
        tiny = json.load(f)
    with open(os.path.join(HERE, "tiny_expected.json"), "w") as f:
        json.dump(tiny, f, indent=1)
        f.write("\n")
    spec = importlib.util.spec_from_file_location("yskn_decode", os.path.join(ref, "tools", "yskn_decode.py"))
    Y = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(Y)
    out = {}
    tmp = os.path.join(HERE, "_tmp.yskn")
    try:
        for bits in range(4, 9):
            for layout in ("row", "warp"):
                for rows, phys, cols in SHAPES:
                    if layout == "warp" and (phys * (cols // 256)) % 32:
                        continue
                    data = fixtures.synthetic(bits, layout, rows, phys, cols, False)
                    with open(tmp, "wb") as f:
                        f.write(data)
                    c = Y.Container(tmp)
                    t = Y.checked(c.tensors["linear"])
                    states = Y.states(Y.unit_words(c, t), t["bits"]).astype("<u2")
                    lut = Y.value_table(c, t)
                    gamma = np.abs(lut).max() / np.float32(127)
                    lut8 = np.clip(np.rint(lut / gamma), -127, 127).astype(np.int8)
                    out["%d/%s/%d/%d/%d" % (bits, layout, rows, phys, cols)] = dict(
                        states_sha256=sha(states), lut8_sha256=sha(lut8.reshape(-1)),
                        container_sha256=hashlib.sha256(data).hexdigest())
                    del c
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)
    with open(os.path.join(HERE, "synthetic_decode.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print("wrote %d synthetic cases" % len(out))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
