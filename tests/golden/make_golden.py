"""Generates tests/golden/q4_0_ref.npz from the reference's own C kernel.

Run in a container that has the reference tree (it builds
oracle/_ref/libq4dot_ref.so from crates/larql-compute/csrc/q4_dot.c with the
reference's x86 flags):

    python tests/golden/make_golden.py

Inputs are the reference tests' LCG (tests/test_q4_x86_correctness.rs:73-79,
seeds 0xC0FFEE / 0xBEEF / 0xDEADBEEF / 0xFEEDFACE) and numpy PCG64 normals.
Q4_0 weights and Q8 x are produced by the restated quantizers, whose bytes are
themselves pinned by tests/test_oracle.py; the outputs are what the
reference's q4_0_matvec_c / q4_0_vecmat_c return for them (bit patterns).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(HERE))

import oracle as O  # noqa: E402
from conftest import lcg_synth, normal  # noqa: E402


def main():
    O.build()
    assert O.ref_lib() is not None, "reference q4_dot.c was not built (needs the reference tree)"
    cases = {}
    # reference test shapes (4 x 64 matvec, 8 x 64 vecmat) and a larger seeded case
    for name, rows, hidden, wseed, xseed, gen in [
        ("x86_matvec", 4, 64, 0xC0FFEE, 0xBEEF, "lcg"),
        ("normal_matvec", 96, 1024, 11, 12, "normal"),
    ]:
        if gen == "lcg":
            w = lcg_synth(rows * hidden, wseed)
            x = lcg_synth(hidden, xseed)
        else:
            w = normal(wseed, rows * hidden, 0.02)
            x = normal(xseed, hidden)
        q4 = O.quantize_q4_0(w)
        q8, q8s = O.quantize_to_q8(x)
        y = O.ref_q4_0_matvec_c(q4, q8, q8s, rows, hidden)
        cases[name] = dict(rows=rows, hidden=hidden, wseed=wseed, xseed=xseed, x=x, q4=q4, q8=q8, q8s=q8s, y=y)
    for name, inter, hidden, aseed, wseed in [("x86_vecmat", 8, 64, 0xDEADBEEF, 0xFEEDFACE)]:
        act = lcg_synth(inter, aseed)
        w = lcg_synth(inter * hidden, wseed)
        q4 = O.quantize_q4_0(w)
        out = O.ref_q4_0_vecmat_c(act, q4, inter, hidden)
        cases[name] = dict(rows=inter, hidden=hidden, x=act, q4=q4, y=out)
    flat = {}
    for name, c in cases.items():
        for k, v in c.items():
            flat[f"{name}.{k}"] = np.asarray(v)
    path = os.path.join(HERE, "q4_0_ref.npz")
    np.savez_compressed(path, **flat)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
