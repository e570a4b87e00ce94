"""Writes the committed golden fixtures under tests/golden/.

w8a8_cfg1_slice.npz: a 64 x 256 -> 96 slice of the seeded single-linear
workload (same draw order as the full 512 x 4096 x 4096 case: X ~ N(0,1) with
1% outlier channels x20, W ~ N(0, 0.02), bias 0), pushed through the oracle:
x, w, bias (bf16 bits), xq, sx, wq, sw, acc, y.

Run from the repo root: ``python tests/golden/make_golden.py``.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def main():
    x, w, b = O.cfg1_inputs(seed=0, M=64, K=256, N=96)
    xb, wb, bb = (O.torch_bf16_to_bits(t) for t in (x, w, b))
    out = O.w8a8_linear_ref(xb, wb, bb)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "w8a8_cfg1_slice.npz")
    np.savez_compressed(path, x=xb, w=wb, bias=bb, **out)
    print("wrote", path)


if __name__ == "__main__":
    main()
