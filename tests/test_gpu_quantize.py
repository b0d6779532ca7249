"""GPU: the Int8 quantiser must be bit-exact to the reference formula
(src/layers/quantization.jl:35-44) and materialisation must follow
quantization.jl:54-64 bit for bit."""
import json
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    from reels_b200 import build
    build.build()
    return torch


def _to_dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("layout", [0, 1])
def test_known_answers(torch_cuda, layout):
    torch = torch_cuda
    from reels_b200 import quantize_frozen_matrix
    rows = json.load(open(os.path.join(GOLDEN, "quant_kat.json")))["rows"]
    W = np.array([r["w"] for r in rows], np.float32)
    Wt = _to_dev(torch, W)
    if layout == 0:
        Wt = Wt.t().contiguous().t()   # column-major (the reference's storage)
    qm = quantize_frozen_matrix(Wt)
    assert qm.layout == layout
    q = qm.values.cpu().numpy()
    s = qm.scales.cpu().numpy()
    for i, r in enumerate(rows):
        assert s[i] == np.float32(r["scale"]), r["why"]
        assert q[i].tolist() == r["q"], r["why"]


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("wdtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("shape", [(8960, 1536), (37, 11), (1, 5), (300, 1)])
def test_bit_exact_vs_oracle(torch_cuda, layout, wdtype, shape):
    torch = torch_cuda
    from reels_b200 import quantize_frozen_matrix
    N, K = shape
    g = np.random.default_rng(N * 7 + K)
    W = (0.02 * g.standard_normal((N, K))).astype(np.float32)
    W[N // 2] = 0.0                                   # an all-zero row
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[wdtype]
    Wt = _to_dev(torch, W, tdt)
    W_in = Wt.float().cpu().numpy()                     # the exact values the kernel sees
    if layout == 0:
        Wt = Wt.t().contiguous().t()
    qm = quantize_frozen_matrix(Wt)
    q_ref, s_ref = oracle.quantize(W_in, 1)
    assert np.array_equal(qm.scales.cpu().numpy(), s_ref)
    assert np.array_equal(qm.values.cpu().numpy(), q_ref)


@pytest.mark.parametrize("layout", [0, 1])
def test_extreme_rows_bit_exact(torch_cuda, layout):
    """Rows at the ends of fp32 (largest finite values, subnormal maxima and
    scales, a scale that underflows to 0 in a row without zeros, signed
    zeros, scale exactly 1 with .5 ties) and rows spanning 2^-140 .. 2^120:
    the GPU quantiser keeps gradual underflow as the reference's fp32
    division does."""
    torch = torch_cuda
    from reels_b200 import quantize_frozen_matrix
    f = np.float32
    tiny = np.finfo(f).tiny
    u = f(2.0 ** -149)
    rows = [[np.finfo(f).max, -np.finfo(f).max, 1.0, 0.0], [tiny, -tiny / 2, tiny / 8, 0.0],
            [u, -u, 2 * u, -3 * u], [0.0, 0.0, 3.0, 0.0], [-0.0, -0.0, -0.0, -0.0],
            [127.0, 63.5, -0.5, 0.5], [1e30, 1e-30, -1e30, 2.5e29]]
    g = np.random.default_rng(17)
    e = g.integers(-140, 120, size=(40, 1))
    rand = (g.standard_normal((40, 4)) * np.exp2(e)).astype(f)
    W = np.concatenate([np.array(rows, f), rand])
    assert f(1.0) / f(1.0) == 1  # (numpy float32 arithmetic below is IEEE)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        m = np.abs(W).max(axis=1)
        sc = np.where(m == 0, f(1), (m / f(127)).astype(f))
        W = W[~np.isnan(W / sc[:, None]).any(axis=1)]   # rows the reference rejects are tested below
    Wt = _to_dev(torch, W)
    if layout == 0:
        Wt = Wt.t().contiguous().t()
    qm = quantize_frozen_matrix(Wt)
    q_ref, s_ref = oracle.quantize(W, 1)
    assert np.array_equal(qm.scales.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(qm.values.cpu().numpy(), q_ref)


@pytest.mark.parametrize("layout", [0, 1])
def test_underflowed_scale_with_zero_raises(torch_cuda, layout):
    """The rows src/layers/quantization.jl:35-44 rejects (tests/golden/
    quant_kat.json "raises"): a NaN quotient reaches Int8 and throws
    InexactError.  Each row alone and among good rows; the kernel then
    recovers on a good matrix and matches the known answers."""
    torch = torch_cuda
    from reels_b200 import quantize_frozen_matrix
    kat = json.load(open(os.path.join(GOLDEN, "quant_kat.json")))
    good = np.array([r["w"] for r in kat["rows"]], np.float32)
    for r in kat["raises"]:
        row = np.array([r["w"]], np.float32)
        for W in (row, np.concatenate([good, row, good])):
            Wt = _to_dev(torch, W)
            if layout == 0:
                Wt = Wt.t().contiguous().t()
            with pytest.raises(ValueError, match="non-finite|0/0"):
                quantize_frozen_matrix(Wt)
    Wt = _to_dev(torch, good)
    if layout == 0:
        Wt = Wt.t().contiguous().t()
    qm = quantize_frozen_matrix(Wt)
    assert qm.values.cpu().numpy().tolist() == [r["q"] for r in kat["rows"]]


def test_non_finite_weight_raises(torch_cuda):
    torch = torch_cuda
    from reels_b200 import quantize_frozen_matrix
    W = torch.ones((16, 32), device="cuda")
    W[3, 4] = float("nan")
    with pytest.raises(ValueError, match="non-finite"):
        quantize_frozen_matrix(W)
    W[3, 4] = float("inf")
    with pytest.raises(ValueError, match="non-finite"):
        quantize_frozen_matrix(W.t().contiguous().t())
    W[3, 4] = 1.0
    quantize_frozen_matrix(W)   # recovers: the status word is per call


@pytest.mark.parametrize("layout", [0, 1])
def test_materialise_bit_exact(torch_cuda, layout):
    torch = torch_cuda
    from reels_b200 import QuantizedMatrix, materialize_weight
    g = np.random.default_rng(5)
    N, K = 96, 80
    q = g.integers(-127, 128, size=(N, K)).astype(np.int8)
    s = (np.abs(g.standard_normal(N)) * 1e-3 + 1e-6).astype(np.float32)
    qt = _to_dev(torch, q)
    if layout == 0:
        qt = qt.t().contiguous().t()
    qm = QuantizedMatrix(qt, _to_dev(torch, s))
    f32 = materialize_weight(qm, torch.float32).cpu().numpy()
    assert np.array_equal(f32, oracle.dequantize_f32(q, s, 1))
    f16 = materialize_weight(qm, torch.float16).cpu().numpy().view(np.uint16)
    assert np.array_equal(f16, oracle.dequantize_f16_bits(q, s, 1))
    bf = materialize_weight(qm, torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(bf, oracle.dequantize_bf16_bits(q, s, 1))


def test_frozen_weight_transfer_int8(torch_cuda):
    """frozen_weight_transfer (quantization.jl:87-140) with int8: a host fp32
    weight becomes a device QuantizedMatrix equal to the oracle's bytes, and
    moving a QuantizedMatrix keeps its values and scales."""
    torch = torch_cuda
    from reels_b200 import frozen_weight_transfer
    w = (0.02 * np.random.default_rng(4).standard_normal((64, 32))).astype(np.float32)
    transfer = frozen_weight_transfer("cuda", "fp16", quantization="int8")
    qm = transfer(torch.from_numpy(w))
    assert qm.values.is_cuda and qm.values.dtype == torch.int8 and qm.dtype == torch.float16
    q_ref, s_ref = oracle.quantize(w, layout=1)
    assert np.array_equal(qm.values.cpu().numpy(), q_ref)
    assert np.array_equal(qm.scales.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    moved = transfer(qm)
    assert torch.equal(moved.values, qm.values) and torch.equal(moved.scales, qm.scales)
