"""Writes reference_kats.json: the known-answer tests of the reference for the decode path.

The reference's own tests for this path (crates/gguf/src/dequant.rs:254-270 and
crates/engine/src/q8_gemv.rs:257-314) build their inputs from simple rules and assert fixed
answers. This script records those rules and the answers they imply, computed exactly in
integer arithmetic (every value involved is an exact small integer or half-integer, so the
f32 results of a correct implementation are exact too):

  q8_0_dequant   d = f16(0.5), q = 2 for all 32 lanes      -> 1.0 (dequant.rs:255-269)
  q8_gemv_ident  m=4, n=32, d = 1, q[r][r] = 1, x[i] = i   -> y[i] = i (q8_gemv.rs:258-281)
  q8_gemv_par    m=256, n=1024, d = 0.5, q = (row+i)%256 as i8, x[i] = i % 100
                 -> y equal to the scalar row loop (q8_gemv.rs:284-314); recorded exactly

Run: python tests/golden/make_golden.py
"""
import json
import os

import numpy as np


def q8_par_expected():
    m, n = 256, 1024
    i = np.arange(32)
    x = (np.arange(n) % 100).astype(np.int64)
    y = []
    for row in range(m):
        q = ((row + i) % 256).astype(np.uint8).view(np.int8).astype(np.int64)
        tot = 0
        for b in range(n // 32):
            tot += int((q * x[b * 32:(b + 1) * 32]).sum())
        y.append(tot * 0.5)
    return y


def main():
    kats = {
        "source": "thebasedcapital/ane-infer crates/gguf/src/dequant.rs:254-270, crates/engine/src/q8_gemv.rs:257-314",
        "q8_0_dequant": {"d": 0.5, "q": 2, "expected": 1.0},
        "q8_gemv_ident": {"m": 4, "n": 32, "d": 1.0, "expected": [0.0, 1.0, 2.0, 3.0]},
        "q8_gemv_par": {"m": 256, "n": 1024, "d": 0.5, "x_mod": 100, "expected": q8_par_expected()},
    }
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(out, "w") as f:
        json.dump(kats, f, indent=1)
    print(out)


if __name__ == "__main__":
    main()
