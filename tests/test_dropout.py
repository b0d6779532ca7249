"""CPU checks of the LoRA dropout mask restated in the oracle.

The mask's generator is SplitMix64's output function over a Weyl sequence
(Steele, Lea and Flood 2014): with seed 0 and stream 0 its outputs for
elements 0, 1, 2 are SplitMix64's published first outputs for seed 0.  The
reference draws the mask from Xoshiro256++ instead (lora.jl:45-52), so the
agreement asked of the mask is statistical: the kept fraction is 1 - p,
neighbouring elements are independent, and masks of different streams or
seeds are unrelated.
"""
import numpy as np
import pytest

import oracle

SPLITMIX_SEED0 = [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


def _u(bits):
    return (bits >> 40) / 2.0 ** 24


def test_known_answers():
    # u of the first three elements is the top 24 bits of those outputs
    us = [_u(b) for b in SPLITMIX_SEED0]
    for p in (0.0, 0.02, 0.5, 0.9):
        keep = oracle.dropout_keep(3, p, 0, 0)
        assert keep.tolist() == [1 if u >= np.float32(p) else 0 for u in us]
    # the stream enters as seed xor (stream * 0x9e3779b97f4a7c15) (lora.jl:41-43)
    g = 0x9E3779B97F4A7C15
    assert np.array_equal(oracle.dropout_keep(1000, 0.3, 7 ^ ((5 * g) & (2 ** 64 - 1)), 0),
                          oracle.dropout_keep(1000, 0.3, 7, 5))


@pytest.mark.parametrize("p", [0.05, 0.1, 0.25, 0.5, 0.9])
def test_kept_fraction(p):
    n = 1 << 20
    keep = oracle.dropout_keep(n, p, 1234, 2).astype(np.float64)
    sigma = np.sqrt(p * (1 - p) / n)
    assert abs(keep.mean() - (1 - p)) < 5 * sigma


def test_p_zero_keeps_everything():
    assert oracle.dropout_keep(10000, 0.0, 99, 1).all()


def test_independence():
    n, p = 1 << 20, 0.3
    k = oracle.dropout_keep(n, p, 42, 0).astype(np.float64) - (1 - p)
    # lag-1 and lag-K (the next token's same feature, K = 1536) correlations
    for lag in (1, 2, 1536):
        c = (k[:-lag] * k[lag:]).mean() / (p * (1 - p))
        assert abs(c) < 5 / np.sqrt(n), lag
    # other streams / seeds: agreement p^2 + (1-p)^2, as for independent masks
    base = oracle.dropout_keep(n, p, 42, 0)
    for other in (oracle.dropout_keep(n, p, 42, 1), oracle.dropout_keep(n, p, 43, 0)):
        agree = (base == other).mean()
        expect = p * p + (1 - p) * (1 - p)
        assert abs(agree - expect) < 5 * np.sqrt(expect * (1 - expect) / n)


def test_uniform_bins():
    # the kept fraction at 20 thresholds traces the uniform CDF
    n = 1 << 18
    for p in np.linspace(0.05, 0.95, 19):
        keep = oracle.dropout_keep(n, float(p), 5, 9)
        assert abs(keep.mean() - (1 - p)) < 5 * np.sqrt(p * (1 - p) / n)
