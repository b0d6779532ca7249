"""Python mirror of Reels.jl's quantised frozen-weight / LoRA layer API.

Names, argument meaning and error behaviour follow the reference:

==============================  ===============================================
reference (src/...)             here
==============================  ===============================================
QuantizedMatrix                 :class:`QuantizedMatrix` (layers/quantization.jl:5-9)
quantize_frozen_matrix          :func:`quantize_frozen_matrix` (quantization.jl:35-44)
_materialize_weight             :func:`materialize_weight` (quantization.jl:54-64)
_weight_mul                     :func:`weight_mul` (quantization.jl:73-74)
_weight_transpose_mul           :func:`weight_transpose_mul` (quantization.jl:75-76)
DenseLayer / linear             :class:`DenseLayer`, :func:`linear` (layers/linear.jl:1-46)
LoRALinear                      :class:`LoRALinear` (layers/lora.jl:1-35)
lora_parameters                 :func:`lora_parameters` (lora.jl:36-37)
frozen_weight_transfer          :func:`frozen_weight_transfer` (quantization.jl:78-140)
lora_forward                    :func:`lora_forward` (lora.jl:56-95)
lora_backward                   :func:`lora_backward` (lora.jl:106-118)
merged_weight                   :func:`merged_weight` (lora.jl:120-122)
rrule(linear)                   :class:`FrozenLinearFunction` (training/ad_rules.jl:55-68)
rrule(_weight_mul) / Zygote     :class:`LoRALinearFunction` (training/ad_rules.jl:70-80)
_projection + gelu_tanh         :func:`lora_forward_gelu` (models/wan21/transformer.jl:289-291,
                                layers/linear.jl:61-68)
feed-forward pair               :class:`GeluFeedForwardFunction` (transformer.jl:287-292)
==============================  ===============================================

Shapes: parameters keep the reference's logical shapes (weight (out, in),
A (rank, in), B (out, rank)); activations are tokens-first, ``x`` (..., in),
which is the same memory as the reference's feature-first column-major
``(in, tokens...)``.  The reference stores parameters column-major; a tensor
here may be either column-major (a transposed view, zero-copy) or row-major.

All arithmetic runs in libreels_lowvram.so on the GPU.  Tensors must be CUDA
tensors; there is no CPU execution path (the reference's own CPU path is
restated only in the test oracle).
"""
from __future__ import annotations

from collections import namedtuple
from dataclasses import dataclass
from typing import Optional

import torch

from . import _native as nat

_DT = {torch.float32: nat.F32, torch.float16: nat.F16, torch.bfloat16: nat.BF16}


def _dt(dtype) -> int:
    try:
        return _DT[dtype]
    except KeyError:
        raise ValueError(f"unsupported compute precision: {dtype}") from None


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("low-VRAM int8 kernels require CUDA tensors (no CPU path)")


def _check_numel(t: Optional[torch.Tensor], n: int, what: str, device=None):
    """The kernels read exactly ``n`` entries of ``t``: a mismatch is a
    DimensionMismatch in the reference's broadcasts, and an out-of-bounds
    read here, so it is refused before any launch."""
    if t is None:
        return
    if t.numel() != n:
        raise ValueError(f"{what} must have {n} entries, found {t.numel()} (shape {tuple(t.shape)})")
    if device is not None and t.device != device:
        raise ValueError(f"{what} is on {t.device}, the input on {device}")


class _Workspace:
    """Scratch buffer per (device, stream), grown on demand by the caller
    side (the native library itself never allocates).  One buffer per stream:
    calls on different streams may run concurrently, and the caching
    allocator only orders a replaced buffer's reuse after work on its own
    stream."""

    def __init__(self):
        self._bufs = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.type, device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WS = _Workspace()


def _workspace(device, M, K, N, r, dt, which):
    n = nat.lib().reels_q8lora_workspace_bytes(M, K, N, r, dt, which)
    buf = _WS.get(device, n)
    return buf.data_ptr(), buf.numel()


# ------------------------------------------------------------- QuantizedMatrix
@dataclass
class QuantizedMatrix:
    """Per-output-channel symmetric Int8 storage of a frozen linear weight
    (quantization.jl:5-9).  ``values`` has logical shape (out, in) and is
    either column-major (the reference's layout: out-contiguous) or
    row-major; ``scales`` is fp32 (out,).  ``dtype`` is the compute dtype
    produced when the weight is materialised."""

    values: torch.Tensor
    scales: torch.Tensor
    dtype: torch.dtype = torch.float32

    @property
    def shape(self):
        return tuple(self.values.shape)

    def size(self, dim=None):
        return self.values.shape if dim is None else self.values.shape[dim]

    @property
    def layout(self) -> int:
        return _weight_layout(self.values)

    def __getitem__(self, idx):
        # quantization.jl:18-19: T(values[i, j]) * T(scales[i]), the product
        # taken in T (for 16-bit T the scale is rounded to T first)
        i, j = idx
        return self.values[i, j].to(self.dtype) * self.scales[i].to(self.dtype)


def _weight_layout(values: torch.Tensor) -> int:
    N, K = values.shape
    if values.stride() == (1, N) or (K == 1 and values.stride()[0] == 1):
        return nat.W_OUT_CONTIGUOUS
    if values.is_contiguous():
        return nat.W_IN_CONTIGUOUS
    raise ValueError("QuantizedMatrix values must be row- or column-major")


def _wmem(values: torch.Tensor) -> int:
    _weight_layout(values)
    return values.data_ptr()


def quantize_frozen_matrix(weight: torch.Tensor, dtype: Optional[torch.dtype] = None,
                           layout: Optional[int] = None) -> QuantizedMatrix:
    """Bit-exact per-row Int8 quantisation (quantization.jl:35-44).

    ``weight`` has logical shape (out, in); its memory layout (column-major as
    in the reference, or row-major) is kept for the int8 values unless
    ``layout`` asks for the other one.  Raises ValueError where the
    reference raises InexactError: on non-finite weights, and on a row whose
    max|w| / 127 underflows to a zero scale while it holds a zero element
    (0 / 0 is NaN)."""
    _require_cuda(weight)
    if weight.dim() != 2:
        raise ValueError("frozen weight must be a matrix")
    N, K = weight.shape
    if dtype is None:
        dtype = weight.dtype
    src_layout = _weight_layout(weight) if (weight.stride() == (1, N) or weight.is_contiguous()) else nat.W_IN_CONTIGUOUS
    if layout is None:
        layout = src_layout
    if layout == nat.W_OUT_CONTIGUOUS:
        w_mem = weight.t().contiguous()           # [K][N]
        values = torch.empty((K, N), dtype=torch.int8, device=weight.device).t()
    else:
        w_mem = weight.contiguous()                # [N][K]
        values = torch.empty((N, K), dtype=torch.int8, device=weight.device)
    scales = torch.empty((N,), dtype=torch.float32, device=weight.device)
    code = nat.lib().reels_q8_quantize(w_mem.data_ptr(), _dt(w_mem.dtype), layout, N, K, values.data_ptr(),
                                       scales.data_ptr(), _stream(weight.device))
    nat.check("quantize_frozen_matrix", code)
    return QuantizedMatrix(values, scales, dtype)


def materialize_weight(weight: QuantizedMatrix, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """_materialize_weight / _dequantize_for_compute (quantization.jl:54-64);
    returns a dense (out, in) tensor in the values' memory layout."""
    dtype = dtype or weight.dtype
    v = weight.values
    _require_cuda(v)
    N, K = v.shape
    layout = weight.layout
    if layout == nat.W_OUT_CONTIGUOUS:
        out = torch.empty((K, N), dtype=dtype, device=v.device).t()
    else:
        out = torch.empty((N, K), dtype=dtype, device=v.device)
    code = nat.lib().reels_q8_materialize(v.data_ptr(), weight.scales.data_ptr(), layout, N, K, _dt(dtype),
                                          out.data_ptr(), _stream(v.device))
    nat.check("materialize_weight", code)
    return out


def _flat(x: torch.Tensor, feat: int):
    if x.shape[-1] != feat:
        raise ValueError("input and weight dimensions differ")  # DimensionMismatch in the reference
    return x.reshape(-1, feat).contiguous()


def weight_mul(weight: QuantizedMatrix, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """_weight_mul (quantization.jl:73-74): y = dequant(W) x (+ bias)."""
    N, K = weight.shape
    _require_cuda(x, weight.values)
    xf = _flat(x, K)
    M = xf.shape[0]
    _check_numel(bias, N, "bias", x.device)
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    dt = _dt(x.dtype)
    ws, wsn = _workspace(x.device, M, K, N, 0, dt, nat.PASS_FORWARD)
    b = bias.contiguous().to(x.dtype) if bias is not None else None
    code = nat.lib().reels_q8_weight_mul(xf.data_ptr(), _wmem(weight.values), weight.scales.data_ptr(),
                                         weight.layout, _ptr(b), M, K, N, dt, y.data_ptr(), ws, wsn,
                                         _stream(x.device))
    nat.check("weight_mul", code)
    return y.reshape(*x.shape[:-1], N)


def weight_transpose_mul(weight: QuantizedMatrix, dy: torch.Tensor) -> torch.Tensor:
    """_weight_transpose_mul (quantization.jl:75-76): dx = dequant(W)' dy."""
    N, K = weight.shape
    _require_cuda(dy, weight.values)
    dyf = _flat(dy, N)
    M = dyf.shape[0]
    dx = torch.empty((M, K), dtype=dy.dtype, device=dy.device)
    dt = _dt(dy.dtype)
    ws, wsn = _workspace(dy.device, M, K, N, 0, dt, nat.PASS_BACKWARD)
    code = nat.lib().reels_q8_weight_transpose_mul(dyf.data_ptr(), _wmem(weight.values), weight.scales.data_ptr(),
                                                   weight.layout, M, K, N, dt, dx.data_ptr(), ws, wsn,
                                                   _stream(dy.device))
    nat.check("weight_transpose_mul", code)
    return dx.reshape(*dy.shape[:-1], K)


# ------------------------------------------------------------------- layers
@dataclass
class DenseLayer:
    """Frozen dense layer (linear.jl:1-4) over a QuantizedMatrix."""

    weight: QuantizedMatrix
    bias: Optional[torch.Tensor] = None


def linear(layer: DenseLayer, x: torch.Tensor) -> torch.Tensor:
    """linear (linear.jl:38-46)."""
    return weight_mul(layer.weight, x, layer.bias)


class LoRALinear:
    """LoRA adapter over a frozen (Int8) weight (lora.jl:1-35).

    ``A`` (rank, in) and ``B`` (out, rank) are stored column-major, as in the
    reference; ``alpha``/``rank`` is the adapter scale."""

    def __init__(self, weight: QuantizedMatrix, bias=None, A=None, B=None, alpha=None, dropout=0.0,
                 enabled=True, train_bias=False, rank=None, generator=None):
        N, K = weight.shape
        if A is None:
            # lora.jl:13-28: A ~ randn / sqrt(in), B = 0
            if rank is None or rank <= 0:
                raise ValueError("rank must be positive")
            dev = weight.values.device
            A = (torch.randn((K, rank), generator=generator, device=dev, dtype=torch.float32)
                 * (1.0 / K ** 0.5)).to(weight.dtype).t()
            B = torch.zeros((rank, N), device=dev, dtype=weight.dtype).t()
        r = A.shape[0]
        if alpha is None:
            alpha = float(r)
        if not (torch.isfinite(torch.tensor(float(alpha))) and alpha > 0):
            raise ValueError("alpha must be finite and positive")
        if not (0 <= dropout < 1):
            raise ValueError("dropout must be in [0, 1)")
        if train_bias and bias is None:
            raise ValueError("cannot train a missing linear bias")
        if tuple(A.shape) != (r, K) or tuple(B.shape) != (N, r):
            raise ValueError("LoRA A must be (rank, in) and B (out, rank)")
        self.weight = weight
        self.bias = bias.clone() if (train_bias and bias is not None) else bias
        self.base_bias = bias
        self.A = A
        self.B = B
        # alpha and dropout are Float32 fields in the reference (lora.jl:6-7)
        self.alpha = _f32(alpha)
        self.dropout = _f32(dropout)
        self.enabled = bool(enabled)
        self.train_bias = bool(train_bias)

    @property
    def rank(self) -> int:
        return self.A.shape[0]

    def __call__(self, x, **kw):
        return lora_forward(self, x, **kw)


def _f32(v) -> float:
    return torch.tensor(float(v), dtype=torch.float32).item()


def set_adapter_enabled(layer: LoRALinear, enabled: bool) -> LoRALinear:
    layer.enabled = bool(enabled)
    return layer


def lora_parameters(layer: LoRALinear) -> dict:
    """The trainable tensors of a layer (lora.jl:36-37): A and B, plus the
    bias when it is trained."""
    return dict(A=layer.A, B=layer.B, bias=layer.bias) if layer.train_bias else dict(A=layer.A, B=layer.B)


_PRECISIONS = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


class FrozenWeightTransfer:
    """Moves frozen weights to their compute form (quantization.jl:78-85,
    111-140): with ``quantization="int8"`` a floating-point weight becomes a
    :class:`QuantizedMatrix` on the device through the GPU quantiser (the
    weight's memory layout is kept), and a QuantizedMatrix is moved as is;
    otherwise the weight is cast to the compute precision."""

    def __init__(self, device, precision: str, quantization: str = "none"):
        self.device = torch.device(device)
        self.precision = precision
        self.dtype = _PRECISIONS[precision]
        self.quantization = quantization

    def __call__(self, weight):
        if self.quantization == "int8":
            if isinstance(weight, QuantizedMatrix):
                return QuantizedMatrix(weight.values.to(self.device), weight.scales.to(self.device), self.dtype)
            return quantize_frozen_matrix(weight.to(self.device), self.dtype)
        if isinstance(weight, QuantizedMatrix):
            return materialize_weight(QuantizedMatrix(weight.values.to(self.device), weight.scales.to(self.device),
                                                      weight.dtype), self.dtype)
        return weight.to(self.device, self.dtype)


def frozen_weight_transfer(device, precision: str, quantization: str = "none",
                           cpu_offload: bool = False) -> FrozenWeightTransfer:
    """frozen_weight_transfer (quantization.jl:87-101), with the reference's
    argument errors.  Two differences: bf16 compute is accepted with Int8
    weights (the reference rejects it; these kernels support it), and CPU
    weight offload is not provided (it is outside this path)."""
    if quantization not in ("none", "int8"):
        raise ValueError("frozen weight quantization must be none or int8")
    if precision not in _PRECISIONS:
        raise ValueError(f"unknown precision {precision}")
    if cpu_offload:
        if torch.device(device).type != "cuda":
            raise ValueError("CPU weight offloading requires device=cuda")
        raise NotImplementedError("CPU weight offloading is not provided by the native int8 path")
    if quantization == "int8" and torch.device(device).type != "cuda":
        raise ValueError("int8 frozen weights run on the GPU path (device=cuda)")
    return FrozenWeightTransfer(device, precision, quantization)


def _colmajor(t: torch.Tensor, dtype) -> torch.Tensor:
    """Memory of logical (a, b) tensor `t` as the reference's column-major
    [b][a] contiguous array."""
    return t.t().contiguous().to(dtype)


def lora_forward(layer: LoRALinear, x: torch.Tensor, training: bool = False, dropout_seed=None,
                 dropout_stream: int = 0, saved: Optional[torch.Tensor] = None) -> torch.Tensor:
    """lora_forward (lora.jl:56-95).  ``saved`` (optional uint8 buffer of
    reels_q8lora_saved_bytes) receives A*x for :func:`lora_backward`.

    With ``training`` and ``layer.dropout > 0`` the adapter sees the dropped
    out input (lora.jl:71-85).  The mask is a function of ``dropout_seed``
    and ``dropout_stream`` (the reference's _dropout_seed); the backward
    recomputes it from the same pair.  ``dropout_seed=None`` draws a seed
    from torch's default generator, as the reference then uses its global
    RNG; pass an explicit seed to be able to call :func:`lora_backward`."""
    if training and layer.dropout > 0 and layer.enabled:
        if dropout_seed is None:
            dropout_seed = int(torch.randint(0, 2 ** 63 - 1, (1,)).item())
        return _lora_forward_dropout(layer, x, saved, int(dropout_seed), int(dropout_stream))
    return _lora_forward(layer, x, False, saved, nat.ACT_NONE, False)[0]


def _u64(v: int) -> int:
    return int(v) & 0xFFFFFFFFFFFFFFFF


def _lora_forward_dropout(layer, x, saved, seed, stream):
    N, K = layer.weight.shape
    _require_cuda(x, layer.weight.values)
    xf = _flat(x, K)
    M = xf.shape[0]
    dt = _dt(x.dtype)
    _check_numel(layer.bias, N, "bias", x.device)
    b = layer.bias.contiguous().to(x.dtype) if layer.bias is not None else None
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    r = layer.rank
    ws, wsn = _workspace(x.device, M, K, N, r, dt, nat.PASS_FORWARD | nat.PASS_DROPOUT)
    A_mem = _colmajor(layer.A, x.dtype)
    B_mem = _colmajor(layer.B, x.dtype)
    code = nat.lib().reels_q8lora_forward_dropout(
        xf.data_ptr(), _wmem(layer.weight.values), layer.weight.scales.data_ptr(), layer.weight.layout,
        A_mem.data_ptr(), B_mem.data_ptr(), _ptr(b), M, K, N, r, layer.alpha, dt, float(layer.dropout), _u64(seed),
        _u64(stream), y.data_ptr(), _ptr(saved), ws, wsn, _stream(x.device))
    nat.check("lora_forward", code)
    return y.reshape(*x.shape[:-1], N)


def dropout_mask(n: int, dropout: float, seed: int, stream: int = 0, device=None) -> torch.Tensor:
    """The keep mask (uint8, 1 = kept) of the first ``n`` elements of an
    adapter input for (seed, stream): the mask lora_forward applies."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    keep = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
    nat.check("dropout_mask", nat.lib().reels_dropout_mask(n, float(dropout), _u64(seed), _u64(stream),
                                                           keep.data_ptr(), _stream(dev)))
    return keep[:n]


def lora_forward_gelu(layer: LoRALinear, x: torch.Tensor, training: bool = False,
                      saved: Optional[torch.Tensor] = None, keep_pre: bool = True):
    """``gelu_tanh(lora_forward(layer, x))`` in one pass (the feed-forward
    input projection and activation of transformer.jl:289-291).  Returns
    ``(y, pre)``: y = gelu_tanh(pre), pre = the linear's output rounded to the
    activation type (None unless ``keep_pre``; the backward of the next linear
    needs it, see :func:`lora_backward`'s ``x_pre``)."""
    return _lora_forward(layer, x, training, saved, nat.ACT_GELU_TANH, keep_pre)


def _lora_forward(layer, x, training, saved, act, keep_pre):
    if training and layer.dropout > 0 and layer.enabled:
        raise NotImplementedError("LoRA dropout is not combined with the fused activation")
    N, K = layer.weight.shape
    _require_cuda(x, layer.weight.values)
    xf = _flat(x, K)
    M = xf.shape[0]
    dt = _dt(x.dtype)
    active_bias = layer.base_bias if (layer.train_bias and not layer.enabled) else layer.bias
    _check_numel(active_bias, N, "bias", x.device)
    b = active_bias.contiguous().to(x.dtype) if active_bias is not None else None
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    pre = torch.empty((M, N), dtype=x.dtype, device=x.device) if keep_pre else None
    r = layer.rank if layer.enabled else 0
    ws, wsn = _workspace(x.device, M, K, N, r, dt, nat.PASS_FORWARD)
    if act != nat.ACT_NONE:
        A_mem = _colmajor(layer.A, x.dtype) if r > 0 else None
        B_mem = _colmajor(layer.B, x.dtype) if r > 0 else None
        code = nat.lib().reels_q8lora_forward_act(xf.data_ptr(), _wmem(layer.weight.values),
                                                  layer.weight.scales.data_ptr(), layer.weight.layout,
                                                  _ptr(A_mem), _ptr(B_mem), _ptr(b), M, K, N, r,
                                                  float(layer.alpha) if r > 0 else 1.0, dt, act, y.data_ptr(), _ptr(pre),
                                                  _ptr(saved), ws, wsn, _stream(x.device))
    elif r > 0:
        A_mem = _colmajor(layer.A, x.dtype)   # [K][r]
        B_mem = _colmajor(layer.B, x.dtype)   # [r][N]
        code = nat.lib().reels_q8lora_forward(xf.data_ptr(), _wmem(layer.weight.values),
                                              layer.weight.scales.data_ptr(), layer.weight.layout,
                                              A_mem.data_ptr(), B_mem.data_ptr(), _ptr(b), M, K, N, r,
                                              layer.alpha, dt, y.data_ptr(), _ptr(saved), ws, wsn,
                                              _stream(x.device))
    else:
        code = nat.lib().reels_q8_weight_mul(xf.data_ptr(), _wmem(layer.weight.values),
                                             layer.weight.scales.data_ptr(), layer.weight.layout, _ptr(b), M, K,
                                             N, dt, y.data_ptr(), ws, wsn, _stream(x.device))
    nat.check("lora_forward", code)
    shape = (*x.shape[:-1], N)
    return y.reshape(shape), (pre.reshape(shape) if pre is not None else None)


LoRAGradients = namedtuple("LoRAGradients", ["dx", "A", "B"])


def lora_backward(layer: LoRALinear, x: torch.Tensor, dy: torch.Tensor, saved: Optional[torch.Tensor] = None,
                  grad_scale: float = 1.0, dA_acc: Optional[torch.Tensor] = None,
                  dB_acc: Optional[torch.Tensor] = None, need_dx: bool = True,
                  x_pre: Optional[torch.Tensor] = None, dropout_seed: Optional[int] = None,
                  dropout_stream: int = 0) -> LoRAGradients:
    """lora_backward (lora.jl:106-118) -> (dx, A=dA, B=dB).

    dA/dB are fp32 with the logical shapes of A and B (column-major).  With
    ``dA_acc``/``dB_acc`` given (fp32 accumulators of that memory layout) the
    gradients times ``grad_scale`` are added into them instead.

    ``x_pre``: when the input is an activation's output, x = gelu_tanh(x_pre)
    (the feed-forward output projection), the gradient is carried through the
    activation in the same pass and ``dx`` is the gradient with respect to
    ``x_pre`` (Zygote's pullback of gelu_tanh, linear.jl:61-68).

    ``dropout_seed``: the gradients of a training forward with LoRA dropout
    (``layer.dropout > 0``) run with that seed and ``dropout_stream``."""
    if tuple(x.shape[:-1]) != tuple(dy.shape[:-1]):
        raise ValueError("LoRA input and output trailing dimensions differ")
    N, K = layer.weight.shape
    _require_cuda(x, dy, layer.weight.values)
    xf = _flat(x, K)
    dyf = _flat(dy, N)
    M = xf.shape[0]
    r = layer.rank
    dt = _dt(x.dtype)
    A_mem = _colmajor(layer.A, x.dtype)
    B_mem = _colmajor(layer.B, x.dtype)
    accumulate = dA_acc is not None
    if accumulate:
        if dB_acc is None:
            raise ValueError("dA_acc and dB_acc are given together")
        if tuple(dA_acc.shape) != (r, K) or tuple(dB_acc.shape) != (N, r):
            raise ValueError("gradient accumulators must have the shapes of A (rank, in) and B (out, rank)")
        if dA_acc.dtype != torch.float32 or dB_acc.dtype != torch.float32:
            raise ValueError("gradient accumulators must be column-major fp32")
        if dA_acc.device != x.device or dB_acc.device != x.device:
            raise ValueError("gradient accumulators must be on the input's device")
        dA_mem, dB_mem = dA_acc.t(), dB_acc.t()
        if not (dA_mem.is_contiguous() and dB_mem.is_contiguous()):
            raise ValueError("gradient accumulators must be column-major fp32")
    else:
        dA_mem = torch.empty((K, r), dtype=torch.float32, device=x.device)
        dB_mem = torch.empty((r, N), dtype=torch.float32, device=x.device)
    dx = torch.empty((M, K), dtype=x.dtype, device=x.device) if need_dx else None
    ws, wsn = _workspace(x.device, M, K, N, r, dt, nat.PASS_BACKWARD)
    drop = dropout_seed is not None and layer.dropout > 0
    if drop and x_pre is not None:
        raise ValueError("dropout is not combined with a fused activation")
    if drop:
        ws, wsn = _workspace(x.device, M, K, N, r, dt, nat.PASS_BACKWARD | nat.PASS_DROPOUT)
        code = nat.lib().reels_q8lora_backward_dropout(
            xf.data_ptr(), dyf.data_ptr(), _wmem(layer.weight.values), layer.weight.scales.data_ptr(),
            layer.weight.layout, A_mem.data_ptr(), B_mem.data_ptr(), _ptr(saved), M, K, N, r, layer.alpha,
            float(grad_scale), dt, float(layer.dropout), _u64(dropout_seed), _u64(dropout_stream), _ptr(dx),
            dA_mem.data_ptr(), dB_mem.data_ptr(), 1 if accumulate else 0, ws, wsn, _stream(x.device))
    elif x_pre is not None:
        if tuple(x_pre.shape) != tuple(x.shape) or x_pre.dtype != x.dtype:
            raise ValueError("x_pre must have the shape and dtype of x")
        xp = _flat(x_pre, K)
        code = nat.lib().reels_q8lora_backward_act(
            xf.data_ptr(), dyf.data_ptr(), _wmem(layer.weight.values), layer.weight.scales.data_ptr(),
            layer.weight.layout, A_mem.data_ptr(), B_mem.data_ptr(), _ptr(saved), M, K, N, r, layer.alpha,
            float(grad_scale), dt, nat.ACT_GELU_TANH, xp.data_ptr(), _ptr(dx), dA_mem.data_ptr(),
            dB_mem.data_ptr(), 1 if accumulate else 0, ws, wsn, _stream(x.device))
    else:
        code = nat.lib().reels_q8lora_backward(xf.data_ptr(), dyf.data_ptr(), _wmem(layer.weight.values),
                                               layer.weight.scales.data_ptr(), layer.weight.layout,
                                               A_mem.data_ptr(), B_mem.data_ptr(), _ptr(saved), M, K, N, r,
                                               layer.alpha, float(grad_scale), dt, _ptr(dx), dA_mem.data_ptr(),
                                               dB_mem.data_ptr(), 1 if accumulate else 0, ws, wsn,
                                               _stream(x.device))
    nat.check("lora_backward", code)
    return LoRAGradients(dx.reshape(x.shape) if dx is not None else None, dA_mem.t(), dB_mem.t())


def saved_buffer(layer: LoRALinear, x: torch.Tensor) -> torch.Tensor:
    """Allocate the buffer that carries A*x from the forward to the backward."""
    M = x.numel() // x.shape[-1]
    n = nat.lib().reels_q8lora_saved_bytes(M, layer.rank, _dt(x.dtype))
    return torch.empty((max(n, 16),), dtype=torch.uint8, device=x.device)


def merged_weight(layer: LoRALinear) -> torch.Tensor:
    """merged_weight (lora.jl:120-122), fp32 (out, in) on the layer's device."""
    w = materialize_weight(layer.weight, torch.float32)
    s = torch.tensor(layer.alpha, dtype=torch.float32, device=w.device) / layer.rank   # Float32 / Int
    return w + s * (layer.B.float() @ layer.A.float())


def check_device_status(device=None) -> None:
    """Synchronise and raise if a kernel's bounded pipeline wait gave up."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    nat.check("device status", nat.lib().reels_lowvram_check_device_status(_stream(dev)))


class FrozenLinearFunction(torch.autograd.Function):
    """Autograd rule of ``linear`` over a frozen DenseLayer (ad_rules.jl:55-68):
    the pullback transmits the activation gradient, dequant(W)' * dy, and
    produces no tangents for the frozen weight or bias."""

    @staticmethod
    def forward(ctx, x, layer):
        ctx.layer = layer
        return linear(layer, x)

    @staticmethod
    def backward(ctx, dy):
        return weight_transpose_mul(ctx.layer.weight, dy.contiguous()), None


class LoRALinearFunction(torch.autograd.Function):
    """Autograd rule for a quantised LoRALinear: the forward saves A*x, the
    backward is the fused native backward.  The counterpart of the rrule that
    routes the frozen weight's pullback to _weight_transpose_mul
    (ad_rules.jl:70-80) plus Zygote's adjoints of B*(A*x)."""

    @staticmethod
    def forward(ctx, x, A, B, layer, training=False, dropout_seed=None, dropout_stream=0):
        saved = saved_buffer(layer, x)
        drop = training and layer.dropout > 0 and layer.enabled
        if drop and dropout_seed is None:
            dropout_seed = int(torch.randint(0, 2 ** 63 - 1, (1,)).item())
        y = lora_forward(layer, x, training=training, dropout_seed=dropout_seed, dropout_stream=dropout_stream,
                         saved=saved)
        ctx.layer = layer
        ctx.dropout = (dropout_seed, dropout_stream) if drop else (None, 0)
        ctx.save_for_backward(x, saved)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, saved = ctx.saved_tensors
        seed, stream = ctx.dropout
        g = lora_backward(ctx.layer, x, dy.contiguous(), saved=saved, dropout_seed=seed, dropout_stream=stream)
        return g.dx, g.A.to(ctx.layer.A.dtype), g.B.to(ctx.layer.B.dtype), None, None, None, None


class GeluFeedForwardFunction(torch.autograd.Function):
    """The feed-forward pair of the Wan block, ``ffn_out(gelu_tanh(ffn_in(x)))``
    (transformer.jl:287-292), with gelu_tanh fused into ffn_in's output tile
    and its derivative into ffn_out's dx tile.  Gradients flow to x and to
    both adapters' A and B."""

    @staticmethod
    def forward(ctx, x, A_in, B_in, A_out, B_out, ffn_in, ffn_out):
        saved_in = saved_buffer(ffn_in, x)
        act, hidden = lora_forward_gelu(ffn_in, x, saved=saved_in)
        saved_out = saved_buffer(ffn_out, act)
        y = lora_forward(ffn_out, act, saved=saved_out)
        ctx.layers = (ffn_in, ffn_out)
        ctx.save_for_backward(x, act, hidden, saved_in, saved_out)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, act, hidden, saved_in, saved_out = ctx.saved_tensors
        ffn_in, ffn_out = ctx.layers
        g_out = lora_backward(ffn_out, act, dy.contiguous(), saved=saved_out, x_pre=hidden)
        g_in = lora_backward(ffn_in, x, g_out.dx, saved=saved_in)
        return (g_in.dx, g_in.A.to(ffn_in.A.dtype), g_in.B.to(ffn_in.B.dtype), g_out.A.to(ffn_out.A.dtype),
                g_out.B.to(ffn_out.B.dtype), None, None)


# ------------------------------------------------------- norm + modulation
def layernorm_modulate(x: torch.Tensor, scale: Optional[torch.Tensor] = None, shift: Optional[torch.Tensor] = None,
                       epsilon: float = 1e-6, weight: Optional[torch.Tensor] = None,
                       bias: Optional[torch.Tensor] = None, tokens_per_sample: Optional[int] = None) -> torch.Tensor:
    """``mixed_affine(layernorm(x; epsilon, weight, bias), scale, shift)``
    (linear.jl:26-36,49-59) in one pass per token: the input of the Wan
    block's linears (transformer.jl:287-289).  ``x`` is (..., K); ``scale``
    and ``shift`` are (batch, K), sample b covering ``tokens_per_sample``
    consecutive tokens (default: all tokens, batch 1)."""
    K = x.shape[-1]
    _require_cuda(x)
    xf = _flat(x, K)
    M = xf.shape[0]
    tps = M if tokens_per_sample is None else int(tokens_per_sample)
    if tps <= 0 and M > 0:
        raise ValueError("tokens_per_sample must be positive")
    batch = max((M + max(tps, 1) - 1) // max(tps, 1), 1)
    for t, n, what in ((scale, batch * K, "scale"), (shift, batch * K, "shift"), (weight, K, "LayerNorm weight"),
                       (bias, K, "LayerNorm bias")):
        if M > 0:
            _check_numel(t, n, what, x.device)
    out = torch.empty_like(xf)
    args = [t.contiguous().to(x.dtype) if t is not None else None for t in (scale, shift, weight, bias)]
    code = nat.lib().reels_layernorm_modulate(xf.data_ptr(), M, K, max(tps, 1), *[_ptr(t) for t in args],
                                              float(epsilon), _dt(x.dtype), out.data_ptr(), _stream(x.device))
    nat.check("layernorm_modulate", code)
    return out.reshape(x.shape)


def layernorm_modulate_backward(x: torch.Tensor, dout: torch.Tensor, scale: Optional[torch.Tensor] = None,
                                epsilon: float = 1e-6, weight: Optional[torch.Tensor] = None,
                                bias: Optional[torch.Tensor] = None, tokens_per_sample: Optional[int] = None,
                                param_grads: bool = False):
    """Pullback of :func:`layernorm_modulate`: ``dx``, and with
    ``param_grads`` the fp32 gradients of ``scale`` and ``shift``
    (modulation.jl:13-22), as ``(dx, dscale, dshift)``."""
    K = x.shape[-1]
    _require_cuda(x, dout)
    if dout.shape != x.shape:
        raise ValueError("dout must have the shape of x")
    xf = _flat(x, K)
    df = _flat(dout, K)
    M = xf.shape[0]
    tps = max(M if tokens_per_sample is None else int(tokens_per_sample), 1)
    batch = max((M + tps - 1) // tps, 1)
    if M == 0:
        # no tokens: the parameter gradients are sums over nothing
        rows = scale.numel() // K if scale is not None else 1
        z = (lambda: torch.zeros((rows, K), dtype=torch.float32, device=x.device)) if param_grads else (lambda: None)
        return torch.empty_like(x), z(), z()
    for t, n, what in ((scale, batch * K, "scale"), (weight, K, "LayerNorm weight"), (bias, K, "LayerNorm bias")):
        _check_numel(t, n, what, x.device)
    dx = torch.empty_like(xf)
    dscale = dshift = None
    ws, wsn = None, 0
    if param_grads:
        dscale = torch.empty((batch, K), dtype=torch.float32, device=x.device)
        dshift = torch.empty((batch, K), dtype=torch.float32, device=x.device)
        wsn = nat.lib().reels_layernorm_modulate_workspace_bytes(M, K, tps)
        ws = _WS.get(x.device, wsn).data_ptr()
    args = [t.contiguous().to(x.dtype) if t is not None else None for t in (scale, weight, bias)]
    code = nat.lib().reels_layernorm_modulate_backward(xf.data_ptr(), df.data_ptr(), M, K, tps, *[_ptr(t) for t in args],
                                                       float(epsilon), _dt(x.dtype), dx.data_ptr(), _ptr(dscale),
                                                       _ptr(dshift), 0, ws, wsn, _stream(x.device))
    nat.check("layernorm_modulate_backward", code)
    return dx.reshape(x.shape), dscale, dshift


class LayerNormModulateFunction(torch.autograd.Function):
    """Autograd rule for :func:`layernorm_modulate`: gradients for x, scale
    and shift (the LayerNorm's own weight and bias are frozen)."""

    @staticmethod
    def forward(ctx, x, scale, shift, epsilon=1e-6, weight=None, bias=None, tokens_per_sample=None):
        ctx.save_for_backward(x, scale, weight, bias)
        ctx.args = (epsilon, tokens_per_sample, shift is not None)
        return layernorm_modulate(x, scale, shift, epsilon, weight, bias, tokens_per_sample)

    @staticmethod
    def backward(ctx, dout):
        x, scale, weight, bias = ctx.saved_tensors
        epsilon, tps, has_shift = ctx.args
        want = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        dx, dscale, dshift = layernorm_modulate_backward(x, dout.contiguous(), scale, epsilon, weight, bias, tps,
                                                         param_grads=want)
        gs = dscale.to(scale.dtype) if (dscale is not None and scale is not None) else None
        gh = dshift.to(x.dtype) if (dshift is not None and has_shift) else None
        return dx, gs, gh, None, None, None, None


# ---------------------------------------------------------- gated residual
def gated_residual(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor, tokens_per_sample: Optional[int] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``mixed_add(x, mixed_mul(y, gate))`` (transformer.jl:272,293) in one
    pass; ``gate`` is (batch, N), sample b covering ``tokens_per_sample``
    tokens.  ``out=x`` updates the residual stream in place."""
    N = x.shape[-1]
    _require_cuda(x, y, gate)
    if y.shape != x.shape or y.dtype != x.dtype:
        raise ValueError("x and y must have the same shape and dtype")
    xf, yf = _flat(x, N), _flat(y, N)
    M = xf.shape[0]
    tps = max(M if tokens_per_sample is None else int(tokens_per_sample), 1)
    if M > 0:
        _check_numel(gate, max((M + tps - 1) // tps, 1) * N, "gate", x.device)
    if out is not None and (out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous()
                            or out.device != x.device):
        raise ValueError("out must be a contiguous tensor of x's shape, dtype and device")
    o = torch.empty_like(xf) if out is None else out.view(-1, N)
    g = gate.contiguous().to(x.dtype)
    nat.check("gated_residual", nat.lib().reels_gated_residual(xf.data_ptr(), yf.data_ptr(), g.data_ptr(), M, N, tps,
                                                               _dt(x.dtype), o.data_ptr(), _stream(x.device)))
    return o.reshape(x.shape) if out is None else out


def gated_residual_backward(dout: torch.Tensor, y: torch.Tensor, gate: torch.Tensor,
                            tokens_per_sample: Optional[int] = None, gate_grad: bool = True):
    """Pullback of :func:`gated_residual`: ``(dy, dgate)`` (the residual's
    gradient is ``dout``); dgate is fp32 (batch, N)."""
    N = dout.shape[-1]
    _require_cuda(dout, y, gate)
    if y.shape != dout.shape or y.dtype != dout.dtype:
        raise ValueError("y and dout must have the same shape and dtype")
    df, yf = _flat(dout, N), _flat(y, N)
    M = df.shape[0]
    tps = max(M if tokens_per_sample is None else int(tokens_per_sample), 1)
    batch = max((M + tps - 1) // tps, 1)
    if M == 0:
        rows = gate.numel() // N
        return torch.empty_like(dout), (torch.zeros((rows, N), dtype=torch.float32, device=dout.device)
                                        if gate_grad else None)
    _check_numel(gate, batch * N, "gate", dout.device)
    dy = torch.empty_like(df)
    dgate, ws, wsn = None, None, 0
    if gate_grad:
        dgate = torch.empty((batch, N), dtype=torch.float32, device=dout.device)
        wsn = nat.lib().reels_gated_residual_workspace_bytes(M, N, tps)
        ws = _WS.get(dout.device, wsn).data_ptr()
    g = gate.contiguous().to(dout.dtype)
    nat.check("gated_residual_backward", nat.lib().reels_gated_residual_backward(
        df.data_ptr(), yf.data_ptr(), g.data_ptr(), M, N, tps, _dt(dout.dtype), dy.data_ptr(), _ptr(dgate), 0, ws,
        wsn, _stream(dout.device)))
    return dy.reshape(dout.shape), dgate
