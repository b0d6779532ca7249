"""Prequantised Int8 checkpoints (SafeTensors), on the CPU.

Checks the file format the reference reads and writes
(src/checkpoints/safetensors.jl:15-124): the u64 little-endian header length,
space padding to 8 bytes, name-ordered contiguous data, row-major shapes, and
the header validation errors; then the Int8 linear convention of
src/models/wan21/text_encoder.jl:296-355 ({key}.weight I8 [out, in] +
{key}.weight.scale F32 [out]), with values and scales from the oracle's
bit-exact quantiser.
"""
import json
import struct

import numpy as np
import pytest
import torch

import oracle
from reels_b200 import QuantizedMatrix
from reels_b200 import checkpoint as ck


def test_round_trip_all_dtypes(tmp_path):
    g = torch.Generator().manual_seed(0)
    tensors = {
        "b.f32": torch.randn(3, 5, generator=g),
        "a.f16": torch.randn(7, generator=g).to(torch.float16),
        "c.bf16": torch.randn(2, 3, 4, generator=g).to(torch.bfloat16),
        "d.i8": torch.randint(-128, 128, (4, 6), generator=g, dtype=torch.int8),
        "e.i32": torch.randint(-1000, 1000, (5,), generator=g, dtype=torch.int32),
        "f.u8": torch.randint(0, 256, (9,), generator=g, dtype=torch.uint8),
        "g.bool": torch.rand(4, generator=g) > 0.5,
        "h.f64": torch.randn(2, 2, generator=g, dtype=torch.float64),
        "i.empty": torch.empty(0, 3),
    }
    p = str(tmp_path / "x.safetensors")
    ck.write_safetensors(p, tensors, {"format": "test", "n": "1"})
    h = ck.inspect_safetensors(p)
    assert h.metadata == {"format": "test", "n": "1"}
    assert set(h.tensors) == set(tensors)
    for name, t in tensors.items():
        back = ck.load_safetensor(p, name, h)
        assert back.dtype == t.dtype and tuple(back.shape) == tuple(t.shape)
        assert torch.equal(back, t), name


def test_file_layout(tmp_path):
    p = str(tmp_path / "y.safetensors")
    ck.write_safetensors(p, {"z": torch.arange(3, dtype=torch.int32), "a": torch.ones(2, 2)}, {"k": "v"})
    raw = open(p, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    header = raw[8:8 + n]
    assert header.rstrip(b" ").endswith(b"}")  # JSON, then space padding only
    h = json.loads(header)
    # tensors in name order, data contiguous from offset 0
    assert h["a"]["data_offsets"] == [0, 16] and h["z"]["data_offsets"] == [16, 28]
    assert h["a"]["dtype"] == "F32" and h["a"]["shape"] == [2, 2]
    assert len(raw) == 8 + n + 28
    assert np.frombuffer(raw[8 + n + 16:], dtype="<i4").tolist() == [0, 1, 2]


def _write_raw(path, header: dict, data: bytes, pad=True):
    enc = json.dumps(header).encode()
    if pad:
        enc += b" " * (-len(enc) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(enc)) + enc + data)


def test_header_validation(tmp_path):
    p = str(tmp_path / "bad.safetensors")
    open(p, "wb").write(b"\x01\x02")
    with pytest.raises(ValueError, match="truncated"):
        ck.inspect_safetensors(p)
    open(p, "wb").write(struct.pack("<Q", 10 ** 9) + b"{}")
    with pytest.raises(ValueError, match="unreasonable"):
        ck.inspect_safetensors(p)
    open(p, "wb").write(struct.pack("<Q", 64) + b"{}")
    with pytest.raises(ValueError, match="exceeds file size"):
        ck.inspect_safetensors(p)
    _write_raw(p, {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
                   "b": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}, b"\0" * 12)
    with pytest.raises(ValueError, match="overlapping"):
        ck.inspect_safetensors(p)
    _write_raw(p, {"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 8)
    with pytest.raises(ValueError, match="exceeds file size"):
        ck.inspect_safetensors(p)
    _write_raw(p, {"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8)
    with pytest.raises(ValueError, match="byte length"):
        ck.load_safetensor(p, "a")
    _write_raw(p, {"a": {"dtype": "C64", "shape": [1], "data_offsets": [0, 8]}}, b"\0" * 8)
    with pytest.raises(ValueError, match="unsupported"):
        ck.load_safetensor(p, "a")
    with pytest.raises(KeyError):
        ck.load_safetensor(p, "missing")


def _oracle_qm(N, K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[3] = 0.0  # an all-zero row: scale 1 (quantization.jl:40)
    q, s = oracle.quantize(w, layout=oracle.LAYOUT_IN_CONTIGUOUS)
    return w, QuantizedMatrix(torch.from_numpy(np.ascontiguousarray(q)), torch.from_numpy(s), torch.float16)


def test_int8_linear_round_trip(tmp_path):
    _, q1 = _oracle_qm(48, 40, 1)
    _, q2 = _oracle_qm(16, 24, 2)
    p = str(tmp_path / "m.safetensors")
    ck.write_quantized_checkpoint(p, {"blocks.0.attn.q": q1, "blocks.0.ffn.fc1": q2},
                                  {"norm.weight": torch.ones(40, dtype=torch.float16)},
                                  compute_dtype=torch.float16, metadata={"format": "reels-test"})
    h = ck.inspect_safetensors(p)
    assert h.metadata["quantization"] == "int8-per-output-channel"
    assert h.metadata["compute_dtype"] == "float16" and h.metadata["format"] == "reels-test"
    assert h.tensors["blocks.0.attn.q.weight"].dtype == "I8"
    assert h.tensors["blocks.0.attn.q.weight"].shape == (48, 40)
    assert h.tensors["blocks.0.attn.q.weight.scale"].dtype == "F32"
    back = ck.load_quantized_linear(p, "blocks.0.attn.q", 48, 40, dtype=torch.float16, header=h)
    assert back.values.is_contiguous() and back.values.dtype == torch.int8
    assert torch.equal(back.values, q1.values) and torch.equal(back.scales, q1.scales)
    assert back.scales[3].item() == 1.0
    assert torch.equal(ck.load_safetensor(p, "norm.weight"), torch.ones(40, dtype=torch.float16))


def test_prequantised_equals_on_load_quantisation(tmp_path):
    # The quantiser is deterministic, so loading a prequantised file gives the
    # bytes an on-load quantisation of the same weights gives.
    w, qm = _oracle_qm(32, 64, 3)
    p = str(tmp_path / "q.safetensors")
    ck.write_quantized_checkpoint(p, {"lin": qm})
    back = ck.load_quantized_linear(p, "lin", 32, 64)
    q_again, s_again = oracle.quantize(w, layout=oracle.LAYOUT_IN_CONTIGUOUS)
    assert np.array_equal(back.values.numpy(), q_again)
    assert np.array_equal(back.scales.numpy().view(np.uint32), s_again.view(np.uint32))


def test_int8_storage_required(tmp_path):
    p = str(tmp_path / "f.safetensors")
    ck.write_safetensors(p, {"lin.weight": torch.zeros(4, 8, dtype=torch.float16),
                             "lin.weight.scale": torch.ones(4)})
    with pytest.raises(ValueError, match="I8 storage"):
        ck.load_quantized_linear(p, "lin", 4, 8)
    ck.write_safetensors(p, {"lin.weight": torch.zeros(4, 8, dtype=torch.int8),
                             "lin.weight.scale": torch.ones(4)})
    with pytest.raises(ValueError, match="shape"):
        ck.load_quantized_linear(p, "lin", 8, 4)
    with pytest.raises(KeyError):
        ck.load_quantized_linear(p, "other", 4, 8)


def test_reference_streaming_io_case(tmp_path):
    """The file test/unit/safetensors.jl:1-13 writes: z = reshape(Float32.(1:6),
    2, 3) and a = Float16[1, 2] under metadata format=reels.  Its writer
    (src/checkpoints/safetensors.jl:101-130) sorts the names, records
    size(z) = [2, 3] and stores z row-major (permutedims of the column-major
    array), so the data section is a's two halves then 1, 3, 5, 2, 4, 6.  The
    bytes are built here as that writer lays them out; loading them gives z
    as the logical 2 x 3 matrix [[1, 3, 5], [2, 4, 6]] and a unchanged, and
    writing the same tensors with this module gives the same data section."""
    header = {"__metadata__": {"format": "reels"},
              "a": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]},
              "z": {"dtype": "F32", "shape": [2, 3], "data_offsets": [4, 28]}}
    data = np.array([1, 2], np.float16).tobytes() + np.array([1, 3, 5, 2, 4, 6], np.float32).tobytes()
    p = str(tmp_path / "adapter.safetensors")
    _write_raw(p, header, data)
    h = ck.inspect_safetensors(p)
    assert h.metadata["format"] == "reels"
    assert sorted(h.tensors) == ["a", "z"]
    z = ck.load_safetensor(p, "z", h)
    assert z.tolist() == [[1, 3, 5], [2, 4, 6]]
    assert ck.load_safetensor(p, "a", h).tolist() == [1.0, 2.0]
    with pytest.raises(KeyError):
        ck.load_safetensor(p, "missing", h)
    q = str(tmp_path / "ours.safetensors")
    ck.write_safetensors(q, {"z": z, "a": torch.tensor([1, 2], dtype=torch.float16)}, {"format": "reels"})
    raw = open(q, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    assert raw[8 + n:] == data


def test_unquantized_tensors_take_the_compute_type():
    """quantized_umt5_state_dict (text_encoder.jl:322-326): floating-point
    tensors other than scales go to the compute type; integers and scales
    are kept."""
    t = {"norm.weight": torch.ones(4, dtype=torch.float32), "lin.weight.scale": torch.ones(4),
         "lin.weight": torch.zeros(4, 4, dtype=torch.int8), "pos": torch.arange(3)}
    out = ck.cast_unquantized(t, torch.float16)
    assert out["norm.weight"].dtype == torch.float16
    assert out["lin.weight.scale"].dtype == torch.float32
    assert out["lin.weight"].dtype == torch.int8 and out["pos"].dtype == torch.int64


def _raw_file(path, header_bytes, payload=b""):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_bytes)))
        f.write(header_bytes)
        f.write(payload)
    return str(path)


@pytest.mark.parametrize("header", [
    b"[1, 2, 3]",                                                   # not an object
    b'{"a": {"dtype": "F32", "shape": [2]}}',                       # no offsets
    b'{"a": {"dtype": "F32", "shape": 3, "data_offsets": [0, 4]}}',  # shape not a list
    b'{"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}',
    b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}',
    b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": "x"}}',
    b'{"__metadata__": [1]}',
    b'{"a": 5}',
    b"\xff\xfe not utf-8",
    b"{not json",
])
def test_malformed_headers_raise_value_errors(tmp_path, header):
    """Every malformed header is a ValueError, as inspect_safetensors
    (safetensors.jl:15-49) throws ArgumentError: never another exception
    type from deep inside the parser."""
    p = _raw_file(tmp_path / "bad.safetensors", header, b"\0" * 8)
    with pytest.raises(ValueError):
        ck.inspect_safetensors(p)


def test_random_bytes_never_crash_the_parser(tmp_path):
    import random
    rng = random.Random(7)
    good = tmp_path / "good.safetensors"
    ck.write_safetensors(str(good), {"w": torch.arange(6, dtype=torch.float32).reshape(2, 3)}, {"k": "v"})
    blob = bytearray(good.read_bytes())
    for trial in range(300):
        b = bytearray(blob)
        for _ in range(rng.randint(1, 6)):
            b[rng.randrange(len(b))] = rng.randrange(256)
        if rng.random() < 0.3:
            b = b[:rng.randrange(len(b))]
        p = tmp_path / f"m{trial}.safetensors"
        p.write_bytes(bytes(b))
        try:
            h = ck.inspect_safetensors(str(p))
            for name in h.tensors:
                try:
                    ck.load_safetensor(str(p), name, h)
                except (KeyError, ValueError):
                    pass
        except ValueError:
            pass
