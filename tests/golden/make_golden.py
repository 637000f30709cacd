"""Regenerate tests/golden/*.npz from the reference's own fixtures.

Reads the torch-generated text fixtures of TokenVector.Inference
(tv/tests/fixtures/g2_*.txt: reduced GPT-2, vocab 256, n_embd 64, 4 heads,
2 layers, 8 tokens, layer_norm_epsilon 1e-6, erf GELU; written by
tools/gen_gpt2_fixture.py in that repository) and stores them as one
compressed npz, so that the tests never need the reference tree at run time.

Usage:  python tests/golden/make_golden.py <path-to-TokenVector.Inference>
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def read_fixture(path):
    with open(path, "r", encoding="utf-8") as f:
        header = f.readline()
        assert header.startswith("# n="), path
        n = int(header.split()[1][2:])
        vals = np.array(f.read().split(), dtype=np.float64)
    assert vals.size == n, (path, vals.size, n)
    return vals


def main(ref_root):
    fx = os.path.join(ref_root, "tv", "tests", "fixtures")
    names = sorted(f[3:-4] for f in os.listdir(fx)
                   if f.startswith("g2_") and f.endswith(".txt") and not f.startswith("g2_m_")
                   and not f.startswith("g2_grad"))
    out = {}
    for nm in names:
        v = read_fixture(os.path.join(fx, "g2_" + nm + ".txt"))
        if nm in ("ids", "pos"):
            out[nm] = v.astype(np.int64)
        else:
            out[nm] = v.astype(np.float32)
    dst = os.path.join(HERE, "g2_reduced.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, "arrays:", len(out))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TVQ_REFERENCE_ROOT", ""))
