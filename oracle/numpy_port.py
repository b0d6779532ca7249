"""The reference's CPU code path for the quantised LoRA linear, in numpy.

TEST / CPU-BASELINE INFRASTRUCTURE ONLY (imported by tests/ and by bench.py's
CPU-baseline leg).  This is what Reels.jl executes when the layer runs on the
CPU in fp32 (the only CPU precision it allows, src/models/interface.jl:38-41):

* `_materialize_weight` (src/layers/quantization.jl:54-64) materialises the
  whole dequantised fp32 matrix ``Float32.(values) .* scales``;
* `_weight_mul` (quantization.jl:73-74) is an fp32 GEMM, which Julia's
  LinearAlgebra sends to OpenBLAS sgemm; numpy calls the same OpenBLAS here;
* the LoRA branch is ``B * (A * x)`` scaled by alpha/r (src/layers/lora.jl:86-94);
* the backward follows `lora_backward` (lora.jl:106-118) operation by operation,
  materialising the dequantised weight again for ``Wdq' * dy``
  (quantization.jl:75-76).

Arrays use the row-major form of the reference's column-major layouts:
X [M][K], Y/dY [M][N], Wq [K][N] (layout 0) or [N][K] (layout 1), A [K][r],
B [r][N].
"""
from __future__ import annotations

import numpy as np


def _dequant(q, scales, layout):
    # quantization.jl:63-64, materialised in the weight's own layout.
    if layout == 0:
        return q.astype(np.float32) * scales[None, :]      # [K][N]
    return q.astype(np.float32) * scales[:, None]          # [N][K]


def _w_mul(Wd, X, layout):
    # y = Wdq * x  ->  Y[M][N] = X @ Wdq^T
    return X @ Wd if layout == 0 else X @ Wd.T


def _wt_mul(Wd, dY, layout):
    # dx = Wdq' * dy  ->  dX[M][K] = dY @ Wdq
    return dY @ Wd.T if layout == 0 else dY @ Wd


def lora_forward(X, q, scales, layout, A, B, alpha):
    """lora.jl:56-95 (training=false, no bias): Y [M][N] in fp32."""
    r = A.shape[1]
    s = np.float32(alpha / r)
    Wd = _dequant(q, scales, layout)
    y = _w_mul(Wd, X, layout)
    t = X @ A                      # (A * x)ᵀ  [M][r]
    adapter = t @ B                # (B * (A * x))ᵀ  [M][N]
    return y + s * adapter


def lora_backward(X, dY, q, scales, layout, A, B, alpha):
    """lora.jl:106-118: returns (dX, dA [K][r], dB [r][N]) in fp32."""
    r = A.shape[1]
    s = np.float32(alpha / r)
    ax = X @ A                     # [M][r]
    g = dY @ B.T                   # (B' * dy)ᵀ  [M][r]
    dA = s * (X.T @ g)             # [K][r]
    dB = s * (ax.T @ dY)           # [r][N]
    Wd = _dequant(q, scales, layout)
    dX = _wt_mul(Wd, dY, layout) + s * (g @ A.T)
    return dX, dA, dB


def lora_step(X, dY, q, scales, layout, A, B, alpha):
    """One forward + backward of the layer, as a training step runs it."""
    Y = lora_forward(X, q, scales, layout, A, B, alpha)
    dX, dA, dB = lora_backward(X, dY, q, scales, layout, A, B, alpha)
    return Y, dX, dA, dB
