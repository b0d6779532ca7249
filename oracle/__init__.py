"""CPU oracle for the Int8-weight LoRA linear -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this package.  The product path (``reels_b200``) never calls it and
fails loudly when its CUDA library is missing.

Two restatements of the reference arithmetic live here:

* ``reels_oracle.c`` (wrapped below): bit-exact quantiser
  (src/layers/quantization.jl:35-44), fp32/fp16/bf16 materialisation
  (quantization.jl:54-64, src/models/interface.jl:13-25), the forward /
  backward of lora.jl:56-95 / lora.jl:106-118 with fp64 accumulation,
  gelu_tanh with its derivative (src/layers/linear.jl:61-68), the LoRA
  dropout forms of both with the library's counter-based mask, and the AdamW
  step with the gradient-norm clip (src/training/optimizer.jl:48-73,
  wan_runner.jl:213-221): the gold standard the CUDA results are compared
  against.
* ``numpy_port.py``: the reference CPU code path in fp32 through OpenBLAS
  (what Julia's LinearAlgebra calls), used as the timed CPU baseline.

Parity status: no reference-produced vectors exist (Julia is not installed and
the reference ships no golden files for this path), so parity against the
reference's own outputs is UNPINNED.  The oracle is pinned by hand-derived
known answers and by the reference tests' properties (tests/test_oracle.py).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_LIB = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64

LAYOUT_OUT_CONTIGUOUS = 0  # Julia (out, in) column-major == row-major [K][N]
LAYOUT_IN_CONTIGUOUS = 1   # PyTorch nn.Linear == row-major [N][K]


def lib():
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        L.oracle_quantize.argtypes = [_f32p, ctypes.c_int, _i64, _i64, _i8p, _f32p]
        L.oracle_quantize.restype = ctypes.c_int
        L.oracle_dequantize_f32.argtypes = [_i8p, _f32p, ctypes.c_int, _i64, _i64, _f32p]
        L.oracle_dequantize_f16.argtypes = [_i8p, _f32p, ctypes.c_int, _i64, _i64, _u16p]
        L.oracle_bf16_materialise_array.argtypes = [_i8p, _f32p, ctypes.c_int, _i64, _i64, _u16p]
        L.oracle_bf16_round_array.argtypes = [_f32p, _i64, _u16p]
        vp = ctypes.c_void_p
        L.oracle_lora_forward.argtypes = [_f32p, _i8p, _f32p, ctypes.c_int, _f32p, _f32p, vp,
                                          _i64, _i64, _i64, _i64, ctypes.c_float, _f32p, vp]
        L.oracle_lora_backward.argtypes = [_f32p, _f32p, _i8p, _f32p, ctypes.c_int, _f32p, _f32p,
                                           _i64, _i64, _i64, _i64, ctypes.c_float, vp, vp, vp]
        L.oracle_gelu_tanh.argtypes = [_f32p, _i64, _f32p]
        L.oracle_gelu_tanh_grad.argtypes = [_f32p, _i64, _f32p]
        f = ctypes.c_float
        L.oracle_adamw_update.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, f, f, f, f, f, f, f, f, ctypes.c_int, f]
        L.oracle_sumsq.argtypes = [_f32p, _i64, ctypes.c_float]
        L.oracle_sumsq.restype = ctypes.c_double
        L.oracle_lora_forward_z.argtypes = [_f32p, vp, _i8p, _f32p, ctypes.c_int, _f32p, _f32p, vp,
                                            _i64, _i64, _i64, _i64, ctypes.c_float, _f32p, vp]
        L.oracle_lora_backward_z.argtypes = [_f32p, vp, vp, _f32p, _i8p, _f32p, ctypes.c_int, _f32p, _f32p,
                                             _i64, _i64, _i64, _i64, ctypes.c_float, vp, vp, vp]
        L.oracle_dropout_keep.argtypes = [_i64, ctypes.c_float, ctypes.c_uint64, ctypes.c_uint64,
                                          np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")]
        L.oracle_layernorm.argtypes = [_f32p, _i64, _i64, ctypes.c_float, vp, vp, _f32p]
        L.oracle_modulate.argtypes = [_f32p, _i64, _i64, _i64, vp, vp, _f32p]
        L.oracle_layernorm_backward.argtypes = [_f32p, _f32p, _i64, _i64, ctypes.c_float, vp, _f32p]
        L.oracle_rel_l2.argtypes = [_f32p, _f32p, _i64]
        L.oracle_rel_l2.restype = ctypes.c_double
        _LIB = L
    return _LIB


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _wshape(layout, N, K):
    return (K, N) if layout == LAYOUT_OUT_CONTIGUOUS else (N, K)


def quantize(w: np.ndarray, layout: int = LAYOUT_OUT_CONTIGUOUS):
    """Bit-exact restatement of quantization.jl:35-44.  ``w`` is given in
    ``layout`` ([K][N] for the Julia layout, [N][K] for the PyTorch layout).
    Returns (q int8 same shape as w, scales fp32 [N]).  Raises ValueError on
    non-finite weights and on a row whose scale underflows to 0 while it
    holds a zero (0/0 = NaN), where the reference raises InexactError."""
    w = _c(w, np.float32)
    if layout == LAYOUT_OUT_CONTIGUOUS:
        K, N = w.shape
    else:
        N, K = w.shape
    q = np.empty(w.shape, np.int8)
    s = np.empty((N,), np.float32)
    rc = lib().oracle_quantize(w, layout, N, K, q, s)
    if rc == -1:
        raise ValueError("frozen weight contains non-finite values")
    if rc == -2:
        raise ValueError("a row's max|w| / 127 underflows to 0 while the row holds a zero: 0/0 is NaN")
    return q, s


def dequantize_f32(q, scales, layout=LAYOUT_OUT_CONTIGUOUS):
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    N = scales.shape[0]
    K = q.size // max(N, 1)
    out = np.empty(q.shape, np.float32)
    lib().oracle_dequantize_f32(q, scales, layout, N, K, out)
    return out


def dequantize_f16_bits(q, scales, layout=LAYOUT_OUT_CONTIGUOUS):
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    N = scales.shape[0]
    K = q.size // max(N, 1)
    out = np.empty(q.shape, np.uint16)
    lib().oracle_dequantize_f16(q, scales, layout, N, K, out)
    return out


def dequantize_bf16_bits(q, scales, layout=LAYOUT_OUT_CONTIGUOUS):
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    N = scales.shape[0]
    K = q.size // max(N, 1)
    out = np.empty(q.shape, np.uint16)
    lib().oracle_bf16_materialise_array(q, scales, layout, N, K, out)
    return out


def bf16_bits(x):
    """interface.jl:19-25 rounding of fp32 to bf16 (returns uint16 bits)."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_bf16_round_array(x, x.size, out)
    return out


def bf16_to_f32(bits):
    """interface.jl:13-17: widen bf16 bits to fp32 exactly."""
    bits = np.asarray(bits, np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x):
    return bf16_to_f32(bf16_bits(x))


def lora_forward(X, q, scales, layout, A, B, alpha, bias=None, want_T=False):
    """Forward of lora.jl:56-95 on Wdq = Float32(q)*scale, fp64 accumulate.
    X [M][K], A [K][r], B [r][N] -> Y [M][N] (and T [M][r] if want_T)."""
    X = _c(X, np.float32)
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    M, K = X.shape
    r = A.shape[1]
    N = scales.shape[0]
    Y = np.empty((M, N), np.float32)
    T = np.empty((M, r), np.float32) if want_T else None
    b = _c(bias, np.float32) if bias is not None else None
    lib().oracle_lora_forward(X, q, scales, layout, A, B,
                              b.ctypes.data if b is not None else None,
                              M, K, N, r, float(alpha), Y,
                              T.ctypes.data if T is not None else None)
    return (Y, T) if want_T else Y


def lora_backward(X, dY, q, scales, layout, A, B, alpha):
    """lora.jl:106-118, fp64 accumulate.  Returns (dX [M][K], dA [K][r], dB [r][N])."""
    X = _c(X, np.float32)
    dY = _c(dY, np.float32)
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    M, K = X.shape
    r = A.shape[1]
    N = scales.shape[0]
    dX = np.empty((M, K), np.float32)
    dA = np.empty((K, r), np.float32)
    dB = np.empty((r, N), np.float32)
    lib().oracle_lora_backward(X, dY, q, scales, layout, A, B, M, K, N, r, float(alpha),
                               dX.ctypes.data, dA.ctypes.data, dB.ctypes.data)
    return dX, dA, dB


def gelu_tanh(h):
    """gelu_tanh (src/layers/linear.jl:61-68) in fp32, elementwise."""
    h = _c(h, np.float32)
    out = np.empty_like(h)
    lib().oracle_gelu_tanh(h.ravel(), h.size, out.ravel())
    return out


def gelu_tanh_grad(h):
    """d gelu_tanh / dh in fp32, elementwise (the pullback's factor)."""
    h = _c(h, np.float32)
    out = np.empty_like(h)
    lib().oracle_gelu_tanh_grad(h.ravel(), h.size, out.ravel())
    return out


def adamw_update(g, m, v, w, lr, beta1, beta2, eps, decay, c1, c2, grad_scale=1.0, clip_scale=None):
    """update! (src/training/optimizer.jl:63-71) on copies of m, v, w (fp32),
    with the gradient clipped by ``clip_scale`` first when given
    (wan_runner.jl:218-221).  Returns the new (m, v, w)."""
    g = _c(g, np.float32).ravel()
    m = np.array(m, np.float32).ravel()
    v = np.array(v, np.float32).ravel()
    w = np.array(w, np.float32).ravel()
    lib().oracle_adamw_update(g, m, v, w, g.size, lr, beta1, beta2, eps, decay, c1, c2, grad_scale,
                              0 if clip_scale is None else 1, 0.0 if clip_scale is None else clip_scale)
    return m, v, w


def sumsq(grads, grad_scale=1.0) -> float:
    """Sum over every array of (grad_scale*g)^2, in fp64."""
    return float(sum(lib().oracle_sumsq(_c(g, np.float32).ravel(), np.asarray(g).size, grad_scale)
                     for g in grads))


def dropout_keep(n, p, seed, stream=0):
    """The library's LoRA dropout mask (uint8, 1 = kept) for n elements."""
    keep = np.empty(n, np.uint8)
    lib().oracle_dropout_keep(n, p, seed & 0xFFFFFFFFFFFFFFFF, stream & 0xFFFFFFFFFFFFFFFF, keep)
    return keep


def lora_dropout(X, Z, dY, q, scales, layout, A, B, alpha, dscale, bias=None):
    """Forward and backward with LoRA dropout (lora.jl:71-85): the adapter's
    input is Z, its part of dX is scaled per element by dscale.  Returns
    (Y, dX, dA, dB), fp64 accumulation."""
    X = _c(X, np.float32)
    Z = _c(Z, np.float32)
    dY = _c(dY, np.float32)
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    dscale = _c(dscale, np.float32)
    M, K = X.shape
    r = A.shape[1]
    N = scales.shape[0]
    Y = np.empty((M, N), np.float32)
    b = _c(bias, np.float32) if bias is not None else None
    lib().oracle_lora_forward_z(X, Z.ctypes.data, q, scales, layout, A, B, b.ctypes.data if b is not None else None,
                                M, K, N, r, float(alpha), Y, None)
    dX = np.empty((M, K), np.float32)
    dA = np.empty((K, r), np.float32)
    dB = np.empty((r, N), np.float32)
    lib().oracle_lora_backward_z(X, Z.ctypes.data, dscale.ctypes.data, dY, q, scales, layout, A, B, M, K, N, r,
                                 float(alpha), dX.ctypes.data, dA.ctypes.data, dB.ctypes.data)
    return Y, dX, dA, dB


def _ptr_or_none(a):
    return None if a is None else _c(a, np.float32).ctypes.data


def layernorm(X, eps, w=None, b=None):
    """layernorm (src/layers/linear.jl:49-59) in fp32, unrounded."""
    X = _c(X, np.float32)
    M, K = X.shape
    Y = np.empty_like(X)
    w = None if w is None else _c(w, np.float32)
    b = None if b is None else _c(b, np.float32)
    lib().oracle_layernorm(X, M, K, eps, _ptr_or_none(w), _ptr_or_none(b), Y)
    return Y


def modulate(LN, tps, scale=None, shift=None):
    """mixed_affine's fp32 part (linear.jl:26-36), unrounded; scale/shift [batch][K]."""
    LN = _c(LN, np.float32)
    M, K = LN.shape
    out = np.empty_like(LN)
    scale = None if scale is None else _c(scale, np.float32)
    shift = None if shift is None else _c(shift, np.float32)
    lib().oracle_modulate(LN, M, K, tps, _ptr_or_none(scale), _ptr_or_none(shift), out)
    return out


def layernorm_backward(X, G, eps, w=None):
    """The LayerNorm's pullback (fp64) for the gradient G at its output."""
    X = _c(X, np.float32)
    G = _c(G, np.float32)
    M, K = X.shape
    DX = np.empty_like(X)
    w = None if w is None else _c(w, np.float32)
    lib().oracle_layernorm_backward(X, G, M, K, eps, _ptr_or_none(w), DX)
    return DX


def rel_l2(a, b) -> float:
    a = _c(a, np.float32).ravel()
    b = _c(b, np.float32).ravel()
    return float(lib().oracle_rel_l2(a, b, a.size))
