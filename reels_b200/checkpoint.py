"""Prequantised Int8 checkpoints in the SafeTensors format.

The reference stores frozen Int8 linears on disk so that they load without a
host quantisation pass (src/models/wan21/text_encoder.jl:296-355, over the
SafeTensors reader/writer of src/checkpoints/safetensors.jl:15-124).  This
module reads and writes the same files:

* file layout: a little-endian u64 header length, a JSON header mapping each
  tensor name to ``{"dtype", "shape", "data_offsets"}`` plus an optional
  ``"__metadata__"`` map of strings, padded with spaces to a multiple of 8
  bytes, then the tensor bytes in name order.  Shapes are row-major.
* an Int8 linear ``key`` is two tensors: ``"{key}.weight"``, I8 of shape
  ``[out, in]`` (row-major, so the input features are contiguous), and
  ``"{key}.weight.scale"``, F32 of shape ``[out]``; the file's metadata names
  the quantisation ``"int8-per-output-channel"``.

``load_quantized_linear`` returns a :class:`QuantizedMatrix` whose values keep
the file's row-major layout, which the library consumes directly
(``REELS_W_IN_CONTIGUOUS``): one host-to-device copy, no quantise pass and no
transpose.  ``quantize_checkpoint`` converts a floating-point checkpoint on the
GPU with the library's bit-exact quantiser (quantization.jl:35-44).

The header checks follow ``inspect_safetensors`` (safetensors.jl:15-49): a
truncated file, an oversized header, offsets that overlap or leave the file,
and byte lengths that disagree with the shape are errors.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Iterable, Mapping, Optional, Tuple

import torch

from . import _native as nat
from .lowvram import QuantizedMatrix, quantize_frozen_matrix

MAX_HEADER_BYTES = 100_000_000
INT8_QUANTIZATION = "int8-per-output-channel"

# SafeTensors dtype codes and their torch types (safetensors.jl:51-57).
DTYPES: Dict[str, torch.dtype] = {
    "F32": torch.float32, "F64": torch.float64, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8,
    "U8": torch.uint8, "BOOL": torch.bool,
}
CODES: Dict[torch.dtype, str] = {v: k for k, v in DTYPES.items()}


@dataclass(frozen=True)
class TensorInfo:
    dtype: str
    shape: Tuple[int, ...]
    data_offsets: Tuple[int, int]


@dataclass(frozen=True)
class SafeTensorHeader:
    metadata: Dict[str, str]
    tensors: Dict[str, TensorInfo]
    data_start: int


def inspect_safetensors(path: str) -> SafeTensorHeader:
    """Parse and validate the header of a SafeTensors file."""
    size = os.path.getsize(path)
    if size < 8:
        raise ValueError("truncated SafeTensors file")
    with open(path, "rb") as f:
        (header_len,) = struct.unpack("<Q", f.read(8))
        if header_len > MAX_HEADER_BYTES:
            raise ValueError(f"unreasonable SafeTensors header length {header_len}")
        if 8 + header_len > size:
            raise ValueError("SafeTensors header exceeds file size")
        raw = json.loads(f.read(header_len).decode("utf-8"))
    if not isinstance(raw, dict):
        raise ValueError("SafeTensors header is not a JSON object")
    metadata: Dict[str, str] = {}
    tensors: Dict[str, TensorInfo] = {}
    for name, value in raw.items():
        try:
            if name == "__metadata__":
                metadata = {str(k): str(v) for k, v in value.items()}
                continue
            offsets = [int(v) for v in value["data_offsets"]]
            shape = tuple(int(v) for v in value["shape"])
            dtype = str(value["dtype"])
        except (AttributeError, KeyError, TypeError, ValueError):
            raise ValueError(f"malformed SafeTensors header entry {name!r}") from None
        if len(offsets) != 2 or not 0 <= offsets[0] <= offsets[1]:
            raise ValueError(f"invalid offsets for tensor {name}")
        if any(d < 0 for d in shape):
            raise ValueError(f"negative dimension for tensor {name}")
        tensors[name] = TensorInfo(dtype, shape, (offsets[0], offsets[1]))
    previous = 0
    for lo, hi, name in sorted((t.data_offsets[0], t.data_offsets[1], n) for n, t in tensors.items()):
        if lo < previous:
            raise ValueError(f"overlapping tensor data at {name}")
        if 8 + header_len + hi > size:
            raise ValueError(f"tensor {name} exceeds file size")
        previous = hi
    return SafeTensorHeader(metadata, tensors, 8 + header_len)


def load_safetensor(path: str, name: str, header: Optional[SafeTensorHeader] = None) -> torch.Tensor:
    """One tensor as a CPU torch tensor of its row-major shape."""
    header = header or inspect_safetensors(path)
    if name not in header.tensors:
        raise KeyError(name)
    info = header.tensors[name]
    if info.dtype not in DTYPES:
        raise ValueError(f"unsupported SafeTensors dtype {info.dtype}")
    dt = DTYPES[info.dtype]
    count = 1
    for d in info.shape:
        count *= d
    nbytes = info.data_offsets[1] - info.data_offsets[0]
    if nbytes != count * torch.empty((), dtype=dt).element_size():
        raise ValueError(f"byte length does not match shape for tensor {name}")
    with open(path, "rb") as f:
        f.seek(header.data_start + info.data_offsets[0])
        buf = bytearray(f.read(nbytes))
    if count == 0:
        return torch.empty(info.shape, dtype=dt)
    return torch.frombuffer(buf, dtype=dt).reshape(info.shape).clone()


def write_safetensors(path: str, tensors: Mapping[str, torch.Tensor],
                      metadata: Optional[Mapping[str, str]] = None) -> str:
    """Write ``tensors`` (any device; written row-major) and ``metadata``.
    The file is written beside ``path`` and renamed into place."""
    names = sorted(tensors)
    header: Dict[str, object] = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in sorted(metadata.items())}
    blobs = []
    offset = 0
    for name in names:
        t = tensors[name].detach().to("cpu").contiguous()
        if t.dtype not in CODES:
            raise ValueError(f"unsupported tensor dtype {t.dtype} for {name}")
        data = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": CODES[t.dtype], "shape": list(t.shape),
                        "data_offsets": [offset, offset + len(data)]}
        offset += len(data)
        blobs.append(data)
    encoded = json.dumps(header, separators=(",", ":")).encode("utf-8")
    encoded += b" " * (-len(encoded) % 8)
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(encoded)))
        f.write(encoded)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)
    return path


def quantized_linear_tensors(key: str, weight: QuantizedMatrix) -> Dict[str, torch.Tensor]:
    """The two on-disk tensors of an Int8 linear: ``{key}.weight`` I8
    ``[out, in]`` and ``{key}.weight.scale`` F32 ``[out]``."""
    return {f"{key}.weight": weight.values.contiguous(),
            f"{key}.weight.scale": weight.scales.to(torch.float32).contiguous()}


def write_quantized_checkpoint(path: str, linears: Mapping[str, QuantizedMatrix],
                               tensors: Optional[Mapping[str, torch.Tensor]] = None,
                               compute_dtype: torch.dtype = torch.float16,
                               metadata: Optional[Mapping[str, str]] = None) -> str:
    """Write Int8 linears (plus any other ``tensors``) with the quantisation
    metadata of the reference's Int8 checkpoints."""
    out: Dict[str, torch.Tensor] = dict(tensors or {})
    for key, qm in linears.items():
        out.update(quantized_linear_tensors(key, qm))
    info = dict(metadata or {})
    info["quantization"] = INT8_QUANTIZATION
    info["compute_dtype"] = {torch.float16: "float16", torch.float32: "float32",
                             torch.bfloat16: "bfloat16"}[compute_dtype]
    return write_safetensors(path, out, info)


def load_quantized_linear(path: str, key: str, out_features: int, in_features: int,
                          device=None, dtype: torch.dtype = torch.float16,
                          header: Optional[SafeTensorHeader] = None) -> QuantizedMatrix:
    """Load ``{key}.weight`` (I8) and ``{key}.weight.scale`` (F32) as a
    QuantizedMatrix on ``device`` (the weight stays row-major: in-features
    contiguous).  Mirrors _load_quantized_t5_dense (text_encoder.jl:337-348):
    a weight stored in any other dtype is an error."""
    header = header or inspect_safetensors(path)
    wname, sname = f"{key}.weight", f"{key}.weight.scale"
    if wname not in header.tensors:
        raise KeyError(wname)
    if header.tensors[wname].dtype != "I8":
        raise ValueError(f"{key}.weight must use SafeTensors I8 storage")
    if header.tensors[wname].shape != (out_features, in_features):
        raise ValueError(f"{wname} has shape {header.tensors[wname].shape}, expected "
                         f"{(out_features, in_features)}")
    if sname not in header.tensors:
        raise KeyError(sname)
    if header.tensors[sname].shape != (out_features,):
        raise ValueError(f"{sname} has shape {header.tensors[sname].shape}, expected {(out_features,)}")
    values = load_safetensor(path, wname, header)
    scales = load_safetensor(path, sname, header).to(torch.float32)
    if device is not None:
        values = values.to(device)
        scales = scales.to(device)
    return QuantizedMatrix(values=values, scales=scales, dtype=dtype)


def cast_unquantized(tensors: Mapping[str, torch.Tensor], compute_dtype: torch.dtype) -> Dict[str, torch.Tensor]:
    """The other tensors of an Int8 checkpoint in the compute type, as
    quantized_umt5_state_dict does (text_encoder.jl:322-326): every
    floating-point tensor except a ``.scale`` is cast; integer tensors and
    the fp32 scales are kept."""
    return {name: (t.to(compute_dtype) if t.is_floating_point() and not name.endswith(".scale") else t)
            for name, t in tensors.items()}


def quantize_checkpoint(src: str, dst: str, keys: Iterable[str], device="cuda",
                        compute_dtype: torch.dtype = torch.float16,
                        metadata: Optional[Mapping[str, str]] = None, cast_others: bool = True) -> str:
    """Convert the floating-point linears ``{key}.weight`` of ``src`` to Int8
    on the GPU (bit-exact quantiser) and write every tensor of ``src`` to
    ``dst``, the listed linears as Int8 with their scales.  With
    ``cast_others`` the remaining floating-point tensors are written in
    ``compute_dtype``, as the reference's Int8 writer does."""
    header = inspect_safetensors(src)
    keys = list(keys)
    wanted = {f"{k}.weight" for k in keys}
    linears: Dict[str, QuantizedMatrix] = {}
    others: Dict[str, torch.Tensor] = {}
    for name in header.tensors:
        t = load_safetensor(src, name, header)
        if name in wanted:
            if t.dim() != 2:
                raise ValueError(f"{name} must be a matrix")
            w = t.to(device)
            linears[name[: -len(".weight")]] = quantize_frozen_matrix(
                w, compute_dtype, layout=nat.W_IN_CONTIGUOUS)
        else:
            others[name] = t
    missing = [k for k in keys if k not in linears]
    if missing:
        raise KeyError(f"missing weights: {missing}")
    if cast_others:
        others = cast_unquantized(others, compute_dtype)
    info = dict(header.metadata)
    info.update(metadata or {})
    return write_quantized_checkpoint(dst, linears, others, compute_dtype, info)
