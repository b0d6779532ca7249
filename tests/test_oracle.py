"""CPU tests of the oracle itself: it must be trustworthy before it judges
the CUDA path.  Pins: hand-derived quantiser known answers, the reference
test properties (test/unit/quantization.jl, test/unit/lora.jl), agreement
with the OpenBLAS restatement, and the committed fixtures."""
import glob
import json
import os

import numpy as np
import pytest

import oracle
from oracle import numpy_port

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _kat():
    with open(os.path.join(GOLDEN, "quant_kat.json")) as f:
        return json.load(f)["rows"]


@pytest.mark.parametrize("layout", [0, 1])
def test_quantizer_known_answers(layout):
    rows = _kat()
    W = np.array([r["w"] for r in rows], np.float32)          # logical (out, in)
    Wmem = np.ascontiguousarray(W.T) if layout == 0 else W
    q, s = oracle.quantize(Wmem, layout)
    qlog = q.T if layout == 0 else q
    for i, r in enumerate(rows):
        assert s[i] == np.float32(r["scale"]), r["why"]
        assert qlog[i].tolist() == r["q"], r["why"]


def test_quantizer_matches_numpy_restatement():
    # The same formula written with numpy's IEEE ops (np.rint = ties-to-even).
    g = np.random.default_rng(3)
    W = (0.02 * g.standard_normal((64, 96))).astype(np.float32)
    W[5] = 0
    W[7, :3] = [0.5, -0.5, 1.5]
    m = np.abs(W).max(axis=1)
    s = (m / np.float32(127)).astype(np.float32)
    s[m == 0] = 1
    qn = np.rint(np.clip(W / s[:, None], -127, 127)).astype(np.int8)
    q, sc = oracle.quantize(W, 1)
    assert np.array_equal(sc, s)
    assert np.array_equal(q, qn)


def _numpy_nan_rows(W):
    """Rows the reference rejects: Julia's clamp keeps a NaN quotient and
    Int8(NaN) throws.  Non-finite weights, or a zero element in a row whose
    max/127 underflowed to a zero scale (0/0)."""
    m = np.abs(W).max(axis=1)
    s = (m / np.float32(127)).astype(np.float32)
    s[m == 0] = 1
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        t = W / s[:, None]
    return np.isnan(t).any(axis=1) | ~np.isfinite(W).all(axis=1)


def _numpy_quantize(W):
    m = np.abs(W).max(axis=1)
    s = (m / np.float32(127)).astype(np.float32)
    s[m == 0] = 1
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        t = W / s[:, None]
    if np.isnan(t).any():
        raise ValueError("NaN quotient: Int8(NaN) throws InexactError")
    qn = np.rint(np.clip(t, -127, 127)).astype(np.int8)
    return qn, s


def test_quantizer_extreme_rows_match_numpy():
    """Rows at the ends of fp32 (largest finite values, subnormals, a lone
    nonzero among zeros, mixed signs of zero) quantise identically in the C
    oracle and the numpy statement; fp32 division with gradual underflow."""
    f = np.float32
    tiny = np.finfo(f).tiny
    rows = [
        [np.finfo(f).max, -np.finfo(f).max, 1.0, 0.0],
        [tiny, -tiny / 2, tiny / 8, 0.0],                 # subnormal maxima and scales
        [np.float32(1e-45), np.float32(-1e-45), np.float32(2e-45), -np.float32(3e-45)],  # scale 0
        [0.0, 0.0, 3.0, 0.0],
        [-0.0, -0.0, -0.0, -0.0],
        [127.0, 63.5, -0.5, 0.5],                         # exact scale 1: ties to even
        [1e30, 1e-30, -1e30, 2.5e29],
    ]
    W = np.array(rows, f)
    q, s = oracle.quantize(W, 1)
    qn, sn = _numpy_quantize(W)
    assert np.array_equal(s.view(np.uint32), sn.view(np.uint32))
    assert np.array_equal(q, qn)
    assert q[5].tolist() == [127, 64, 0, 0] and s[4] == 1
    assert s[2] == 0 and q[2].tolist() == [127, -127, 127, -127]


@pytest.mark.parametrize("layout", [0, 1])
def test_quantizer_rejects_what_the_reference_rejects(layout):
    """The hand-derived rows the reference throws InexactError on (a NaN
    quotient reaching Int8): each alone and inside a matrix of good rows."""
    bad = json.load(open(os.path.join(GOLDEN, "quant_kat.json")))["raises"]
    good = np.array([r["w"] for r in _kat()], np.float32)
    for r in bad:
        row = np.array([r["w"]], np.float32)
        for W in (row, np.concatenate([good, row, good])):
            Wm = np.ascontiguousarray(W.T) if layout == 0 else W
            with pytest.raises(ValueError):
                oracle.quantize(Wm, layout)
            with pytest.raises(ValueError):
                _numpy_quantize(W)
            assert _numpy_nan_rows(W).sum() == 1, r["why"]


def test_quantizer_random_scales_match_numpy():
    """Rows whose magnitudes span 2^-140 .. 2^120, in both layouts."""
    g = np.random.default_rng(17)
    for trial in range(20):
        e = g.integers(-140, 120, size=(32, 1))
        W = (g.standard_normal((32, 48)) * np.exp2(e)).astype(np.float32)
        W[g.random(W.shape) < 0.1] = 0
        bad = _numpy_nan_rows(W)
        if bad.any():
            # rows with a zero scale and a zero element: the whole call raises
            for layout in (0, 1):
                with pytest.raises(ValueError):
                    oracle.quantize(np.ascontiguousarray(W.T) if layout == 0 else W, layout)
            W = W[~bad]
        qn, sn = _numpy_quantize(W)
        for layout in (0, 1):
            Wm = np.ascontiguousarray(W.T) if layout == 0 else W
            q, s = oracle.quantize(Wm, layout)
            assert np.array_equal(s.view(np.uint32), sn.view(np.uint32)), trial
            assert np.array_equal(q.T if layout == 0 else q, qn), trial


def test_quantizer_rejects_non_finite():
    W = np.ones((3, 4), np.float32)
    W[1, 2] = np.nan
    with pytest.raises(ValueError):
        oracle.quantize(W, 1)
    W[1, 2] = np.inf
    with pytest.raises(ValueError):
        oracle.quantize(W, 1)


def test_quantizer_round_trip_and_requantise():
    # test/unit/quantization.jl:8 (rtol = atol = 1e-2) and :50-53 (int8 values
    # stay identical when a quantised weight is moved again).
    g = np.random.default_rng(950)
    W = g.standard_normal((7, 5)).astype(np.float32)
    q, s = oracle.quantize(W, 1)
    Wd = oracle.dequantize_f32(q, s, 1)
    assert np.allclose(Wd, W, rtol=1e-2, atol=1e-2)
    q2, s2 = oracle.quantize(Wd, 1)
    assert np.array_equal(q2, q)
    assert np.allclose(s2, s, rtol=1e-6, atol=0)


def test_materialise_rules():
    q = np.array([[127, -3, 0, 64], [1, -127, 5, 2]], np.int8)
    s = np.array([0.0123, 3.0e-5], np.float32)
    f32 = oracle.dequantize_f32(q, s, 1)
    assert np.array_equal(f32, q.astype(np.float32) * s[:, None])
    f16 = oracle.dequantize_f16_bits(q, s, 1).view(np.float16)
    ref = (q.astype(np.float16) * s.astype(np.float16)[:, None]).astype(np.float16)
    assert np.array_equal(f16, ref)
    b = oracle.dequantize_bf16_bits(q, s, 1)
    assert np.array_equal(b, oracle.bf16_bits(f32))


def test_bf16_rounding_rule():
    # interface.jl:19-25: bits + 0x7fff + lsb, i.e. round-to-nearest-even.
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-39], np.float32)
    bits = oracle.bf16_bits(x)
    u = x.view(np.uint32)
    ref = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    assert np.array_equal(bits, ref)


def _case(M=9, K=24, N=40, r=3, seed=0, layout=0):
    g = np.random.default_rng(seed)
    X = g.standard_normal((M, K)).astype(np.float32)
    W = (0.02 * g.standard_normal((N, K))).astype(np.float32)
    Wmem = np.ascontiguousarray(W.T) if layout == 0 else W
    A = (g.standard_normal((K, r)) / np.sqrt(K)).astype(np.float32)
    B = g.standard_normal((r, N)).astype(np.float32)
    dY = g.standard_normal((M, N)).astype(np.float32)
    q, s = oracle.quantize(Wmem, layout)
    return X, q, s, A, B, dY


@pytest.mark.parametrize("layout", [0, 1])
def test_oracle_matches_blas_port(layout):
    X, q, s, A, B, dY = _case(layout=layout)
    Y = oracle.lora_forward(X, q, s, layout, A, B, 6.0)
    assert oracle.rel_l2(numpy_port.lora_forward(X, q, s, layout, A, B, 6.0), Y) < 1e-5
    for a, b in zip(numpy_port.lora_backward(X, dY, q, s, layout, A, B, 6.0),
                    oracle.lora_backward(X, dY, q, s, layout, A, B, 6.0)):
        assert oracle.rel_l2(a, b) < 1e-5


def test_zero_B_is_exactly_the_base_linear():
    # test/unit/lora.jl:6: B = 0 gives exactly W*x.
    X, q, s, A, B, dY = _case()
    Y = oracle.lora_forward(X, q, s, 0, A, np.zeros_like(B), 2.0)
    Y0 = oracle.lora_forward(X, q, s, 0, A[:, :0].copy(), B[:0].copy(), 2.0)
    assert np.array_equal(Y, Y0)


def test_merged_weight_equivalence():
    # test/unit/lora.jl:8: layer(x) ≈ merged_weight(layer) * x
    X, q, s, A, B, dY = _case(layout=1)
    alpha, r = 6.0, A.shape[1]
    Wd = oracle.dequantize_f32(q, s, 1)                       # [N][K]
    merged = Wd + (alpha / r) * (B.T @ A.T)                   # (out, in)
    Y = oracle.lora_forward(X, q, s, 1, A, B, alpha)
    assert np.allclose(Y, X @ merged.T, rtol=1e-5, atol=1e-5)


def test_backward_finite_differences():
    # test/unit/lora.jl:12-21 (dA[1], eps 1e-3, rtol 2e-2) and the lora_B
    # finite difference of test/unit/wan_training.jl:44-60, in fp64 here.
    X, q, s, A, B, dY = _case(M=5, K=4, N=3, r=2, seed=4)
    alpha = 2.0
    dX, dA, dB = oracle.lora_backward(X, dY, q, s, 0, A, B, alpha)

    def loss(A_, B_, X_):
        return float(np.sum(oracle.lora_forward(X_, q, s, 0, A_, B_, alpha).astype(np.float64) * dY))

    eps = 1e-3
    for (k, j) in [(0, 0), (3, 1)]:
        Ap, Am = A.copy(), A.copy()
        Ap[k, j] += eps
        Am[k, j] -= eps
        fd = (loss(Ap, B, X) - loss(Am, B, X)) / (2 * eps)
        assert fd == pytest.approx(dA[k, j], rel=2e-2, abs=1e-4)
    for (j, n) in [(0, 0), (1, 2)]:
        Bp, Bm = B.copy(), B.copy()
        Bp[j, n] += eps
        Bm[j, n] -= eps
        fd = (loss(A, Bp, X) - loss(A, Bm, X)) / (2 * eps)
        assert fd == pytest.approx(dB[j, n], rel=2e-2, abs=1e-4)
    for (m, k) in [(0, 0), (4, 3)]:
        Xp, Xm = X.copy(), X.copy()
        Xp[m, k] += eps
        Xm[m, k] -= eps
        fd = (loss(A, B, Xp) - loss(A, B, Xm)) / (2 * eps)
        assert fd == pytest.approx(dX[m, k], rel=2e-2, abs=1e-4)


def test_quantised_linear_tracks_fp32():
    # test/unit/quantization.jl:11,22-23: quantised ≈ unquantised within 2e-2.
    g = np.random.default_rng(950)
    W = g.standard_normal((7, 5)).astype(np.float32)
    X = g.standard_normal((4, 5)).astype(np.float32)
    A = g.standard_normal((5, 2)).astype(np.float32)
    B = g.standard_normal((2, 7)).astype(np.float32)
    q, s = oracle.quantize(W, 1)
    Y = oracle.lora_forward(X, q, s, 1, A, B, 2.0)
    ref = X @ W.T + (2.0 / 2) * (X @ A) @ B
    assert np.allclose(Y, ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "linear_*.npz"))))
def test_oracle_reproduces_committed_fixtures(path):
    f = np.load(path)
    meta = json.loads(str(f["meta"]))
    q, s = oracle.quantize(f["W"], meta["layout"])
    assert np.array_equal(q, f["q"]) and np.array_equal(s, f["s"])
    Y = oracle.lora_forward(f["X"], q, s, meta["layout"], f["A"], f["B"], meta["alpha"])
    assert np.array_equal(Y, f["Y"])
    dX, dA, dB = oracle.lora_backward(f["X"], f["dY"], q, s, meta["layout"], f["A"], f["B"], meta["alpha"])
    assert np.array_equal(dX, f["dX"]) and np.array_equal(dA, f["dA"]) and np.array_equal(dB, f["dB"])


def test_gelu_tanh_known_answers():
    """gelu_tanh (src/layers/linear.jl:61-68): fixed points and the published
    values of the tanh approximation, in fp32."""
    x = np.array([0.0, 1.0, -1.0, 2.0, -3.0, 0.5, 10.0, -10.0], np.float32)
    y = oracle.gelu_tanh(x)
    expect = [0.0, 0.8411920, -0.1588080, 1.9545977, -0.0036374, 0.3457140, 10.0, 0.0]
    assert np.allclose(y, expect, rtol=2e-6, atol=2e-7)
    # odd part: gelu(x) - gelu(-x) = x
    z = np.linspace(-6, 6, 1001, dtype=np.float32)
    assert np.allclose(oracle.gelu_tanh(z) - oracle.gelu_tanh(-z), z, atol=2e-6)


def test_gelu_tanh_grad_matches_finite_differences():
    z = np.linspace(-8, 8, 4001)
    k0, k1 = np.sqrt(2 / np.pi), 0.044715
    f = lambda v: 0.5 * v * (1 + np.tanh(k0 * (v + k1 * v ** 3)))
    h = 1e-5
    fd = (f(z + h) - f(z - h)) / (2 * h)
    got = oracle.gelu_tanh_grad(z.astype(np.float32))
    assert np.max(np.abs(got - fd)) < 2e-6


def test_gelu_tanh_float16_reference_case():
    """test/unit/layers.jl:12-18: gelu_tanh of Float16 values, rounded to
    Float16, is within rtol 2e-3 / atol 2e-4 of the Float32 result."""
    v = np.array([-2, -0.5, 0, 0.5, 2], np.float16)
    h = oracle.gelu_tanh(v.astype(np.float32)).astype(np.float16).astype(np.float32)
    ref = oracle.gelu_tanh(v.astype(np.float32))
    assert np.allclose(h, ref, rtol=2e-3, atol=2e-4)


def test_dropout_oracle_matches_numpy():
    """oracle.lora_dropout (the forward and backward with the adapter fed
    Z and its dx part scaled per element) against an fp64 numpy statement."""
    rng = np.random.default_rng(12)
    M, K, N, r, alpha = 9, 24, 16, 4, 8.0
    X = rng.standard_normal((M, K)).astype(np.float32)
    Wm = (0.02 * rng.standard_normal((K, N))).astype(np.float32)
    q, s = oracle.quantize(Wm, 0)
    A = rng.standard_normal((K, r)).astype(np.float32)
    B = rng.standard_normal((r, N)).astype(np.float32)
    dY = rng.standard_normal((M, N)).astype(np.float32)
    keep = (rng.random((M, K)) > 0.3).astype(np.float32)
    Z = (X * keep / np.float32(0.7)).astype(np.float32)
    Y, dX, dA, dB = oracle.lora_dropout(X, Z, dY, q, s, 0, A, B, alpha, keep / np.float32(0.7))
    W = oracle.dequantize_f32(q, s, 0).astype(np.float64)  # [K][N]
    sc = float(np.float32(alpha / r))
    T = Z.astype(np.float64) @ A
    G = dY.astype(np.float64) @ B.T
    assert np.allclose(Y, X @ W + sc * T @ B, rtol=1e-5, atol=1e-5)
    assert np.allclose(dX, dY @ W.T + sc * (G @ A.T) * (keep / np.float32(0.7)), rtol=1e-5, atol=1e-5)
    assert np.allclose(dA, sc * Z.T.astype(np.float64) @ G, rtol=1e-5, atol=1e-5)
    assert np.allclose(dB, sc * T.T @ dY, rtol=1e-5, atol=1e-5)
