"""Generates tests/golden/small_cases.npz from the CPU restatement (oracle/).

The reference (Mojo, osx-arm64) cannot run in this environment and its
tests keep no output vectors, so these fixtures are the oracle's own
outputs on seeded inputs: they pin the restatement against regressions and
give the GPU tests fixed expected values. Run from the repo root:
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "trellis2-mojo_b200")]

from oracle import oracle as O  # noqa: E402
from t2sc import synth  # noqa: E402


def main():
    O.build()
    out = {}
    cases = {
        "shell16": (synth.shell(16, 6.0, 1.0, seed=3), 1, 24, 16),
        "blob4d2": (synth.blob(4), 2, 8, 12),
    }
    for name, (c, dil, ci, co) in cases.items():
        src, tgt, kidx = O.neighbor_map(c, dilation=dil)
        x = synth.normal(11, (len(c), ci))
        w = synth.normal(12, (co, 3, 3, 3, ci), std=(1.0 / (27 * ci)) ** 0.5)
        b = synth.normal(13, (co,), std=0.1)
        y = O.conv(x, w, b, (src, tgt, kidx))
        out.update({f"{name}_coords": c, f"{name}_dil": np.int64(dil), f"{name}_src": src, f"{name}_tgt": tgt,
                    f"{name}_kidx": kidx, f"{name}_x": x, f"{name}_w": w, f"{name}_b": b, f"{name}_y": y})
    pc = synth.shell(12, 4.0, 0.8, seed=5)
    mask = synth.bernoulli(21, (len(pc), 8))
    idx, sidx, nc = O.subdivide(pc, mask)
    out.update({"sub_coords": pc, "sub_mask": mask, "sub_idx": idx, "sub_subidx": sidx, "sub_out_coords": nc})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "small_cases.npz")
    np.savez_compressed(path, **out)
    print(path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
