"""Writes tests/golden/chunked_attention.npz from the reference's own chunked
causal attention.

Run from the repo root with the reference's ``src`` directory as the argument:

    python tests/golden/make_golden_attention.py <reference>/src

It draws seeded bf16 q [B, H, S, D] and k, v [B, Hkv, S, D] (GQA: H = 2 Hkv),
expands k and v to all heads as the reference's RoPE adapter does
(src/lema/adapters/_chunked_rope.py:82-84), and runs, for every query chunk,
``chunked_attention`` (src/lema/_tensorstore.py:565-608) over key chunks 0..c
with ``causal=True``, as ``rope_chunked_forward_layer`` does
(src/lema/adapters/_chunked_rope.py:100-110). It stores the inputs and the
output (bf16 as uint16 bit patterns) for two cases: a ragged sequence (the
last chunk shorter than the others) and a single chunk. The script is the
only place that reads the reference; tests read the .npz.
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

CASES = {"ragged": (1, 4, 2, 160, 32, 64), "one_chunk": (2, 2, 1, 48, 64, 64)}


def main(ref_src: str):
    sys.path.insert(0, ref_src)
    from lema._tensorstore import chunked_attention

    out = {}
    g = torch.Generator().manual_seed(11)
    for name, (B, H, Hkv, S, D, chunk) in CASES.items():
        q = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
        rep = H // Hkv
        ke = k.repeat_interleave(rep, dim=1)
        ve = v.repeat_interleave(rep, dim=1)
        parts = []
        for s in range(0, S, chunk):
            e = min(s + chunk, S)
            kv = [(ke[:, :, c0:min(c0 + chunk, S)], ve[:, :, c0:min(c0 + chunk, S)])
                  for c0 in range(0, e, chunk)]
            parts.append(chunked_attention(q[:, :, s:e], kv, D ** -0.5, query_start=s,
                                           kv_chunk_size=chunk, causal=True))
        o = torch.cat(parts, dim=2)
        for key, t in (("q", q), ("k", k), ("v", v), ("o", o)):
            out[f"{name}/{key}"] = O.torch_bf16_to_bits(t).copy()
        out[f"{name}/meta"] = np.array([B, H, Hkv, S, D, chunk])
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "chunked_attention.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_attention.py <reference>/src")
    main(sys.argv[1])
