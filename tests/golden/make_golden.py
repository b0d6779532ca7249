"""Generate the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

Two kinds of fixture:

* ``quant_kat.json`` -- known answers for the quantiser derived BY HAND from
  the reference formula (src/layers/quantization.jl:35-44): rows whose scale
  max|w|/127 is exactly representable (1, 2, 0.5) so every w/scale is exact
  and the expected Int8 follows from round-half-to-even (Julia's default
  RoundNearest) and the clamp.  These do not come from any program.
* ``linear_*.npz`` -- seeded inputs and the CPU oracle's fp64-accumulated
  outputs (forward Y, backward dX/dA/dB) for small shapes.  They pin the
  oracle and the GPU path to fixed numbers across runs; they are NOT
  reference-produced (Julia is unavailable), see oracle/__init__.py.

Inputs: numpy Generator(PCG64(seed)); X, dY ~ N(0, 1); W ~ N(0, 0.02);
A ~ N(0, 1/sqrt(K)) (lora.jl:23); B ~ N(0, 0.01).  16-bit cases store inputs
already rounded to bf16 with the reference rule (interface.jl:19-25).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

# Hand-derived known answers: (row of w, expected scale, expected q row).
QUANT_KAT = [
    {"w": [127.0, 2.5, -2.5, 3.5, 0.5, -0.5, 1.5, -126.5],
     "scale": 1.0, "q": [127, 2, -2, 4, 0, 0, 2, -126],
     "why": "max 127 -> scale 1; .5 ties go to the even neighbour"},
    {"w": [-254.0, 5.0, -3.0, 1.0, 0.999, 253.0, 127.0, 0.0],
     "scale": 2.0, "q": [-127, 2, -2, 0, 0, 126, 64, 0],
     "why": "max 254 -> scale 2; 2.5->2, -1.5->-2, 0.5->0, 126.5->126, 63.5->64"},
    {"w": [0.0, -63.5, 31.75, 15.875, 0.25, -0.75, 0.0, 0.0],
     "scale": 0.5, "q": [0, -127, 64, 32, 0, -2, 0, 0],
     "why": "max 63.5 -> scale 0.5; 63.5->64, 31.75->32, 0.5->0, -1.5->-2"},
    {"w": [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
     "scale": 1.0, "q": [0, 0, 0, 0, 0, 0, 0, 0],
     "why": "all-zero row -> scale forced to 1"},
    {"w": [-0.0, 0.0, -0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
     "scale": 1.0, "q": [0, 0, 0, 0, 0, 0, 0, 0],
     "why": "negative zeros count as zero maxima"},
]

LINEAR_CASES = [
    # name, M, K, N, r, alpha, dtype, layout, seed
    ("linear_refdims_f32", 4, 5, 7, 2, 2.0, "f32", 0, 950),
    ("linear_rank3_f32", 4, 5, 7, 3, 6.0, "f32", 1, 41),
    ("linear_ragged_bf16", 37, 80, 48, 3, 6.0, "bf16", 0, 7),
    ("linear_mid_bf16", 48, 128, 192, 8, 8.0, "bf16", 1, 11),
    ("linear_mid_f16", 40, 192, 128, 16, 16.0, "f16", 0, 12),
]


def _round(x, dtype):
    x = np.asarray(x, np.float32)
    if dtype == "bf16":
        return oracle.bf16_round(x)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def make_linear(name, M, K, N, r, alpha, dtype, layout, seed):
    g = np.random.Generator(np.random.PCG64(seed))
    X = _round(g.standard_normal((M, K)), dtype)
    W = (0.02 * g.standard_normal((N, K))).astype(np.float32)     # logical (out, in)
    A = _round(g.standard_normal((K, r)) / np.sqrt(K), dtype)    # memory of (rank, in) column-major
    B = _round(0.01 * g.standard_normal((r, N)), dtype)          # memory of (out, rank) column-major
    dY = _round(g.standard_normal((M, N)), dtype)
    Wmem = np.ascontiguousarray(W.T) if layout == 0 else W
    q, s = oracle.quantize(Wmem, layout)
    Y = oracle.lora_forward(X, q, s, layout, A, B, alpha)
    dX, dA, dB = oracle.lora_backward(X, dY, q, s, layout, A, B, alpha)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), X=X, W=Wmem, q=q, s=s, A=A, B=B, dY=dY, Y=Y, dX=dX,
                        dA=dA, dB=dB, meta=json.dumps({"M": M, "K": K, "N": N, "r": r, "alpha": alpha,
                                                      "dtype": dtype, "layout": layout, "seed": seed}))


def main():
    with open(os.path.join(HERE, "quant_kat.json"), "w") as f:
        json.dump({"source": "hand-derived from src/layers/quantization.jl:35-44", "rows": QUANT_KAT}, f, indent=1)
    for case in LINEAR_CASES:
        make_linear(*case)
    print("wrote", len(LINEAR_CASES) + 1, "fixtures to", HERE)


if __name__ == "__main__":
    main()
