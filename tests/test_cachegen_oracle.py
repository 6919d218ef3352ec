"""CPU tests of the CacheGen oracle (oracle/cachegen_ref.c): CDF invariants,
encode -> decode round trips, prefix-sum decoding, overflow reporting and
edge cases. The reference's codec entry points are stubs
(csrc/cachegen_kernels.cpp:7-32), so these properties, not golden vectors,
pin the format."""

import numpy as np
import pytest

from oracle import cachegen as cg


def skewed_symbols(rng, shape, max_bins, conc):
    p = rng.dirichlet(np.full(max_bins, conc))
    return rng.choice(max_bins, size=shape, p=p).astype(np.uint8)


def check_cdf(cdf, max_bins):
    u = cdf.view(np.uint16).astype(np.int64)
    assert (u[..., 0] == 0).all()
    assert (u[..., max_bins] == 1 << 15).all()
    assert (np.diff(u, axis=-1) >= 1).all()


@pytest.mark.parametrize("seed", range(12))
def test_round_trip_random(seed):
    rng = np.random.default_rng(seed)
    L, T, C = int(rng.integers(1, 4)), int(rng.integers(1, 400)), int(rng.integers(1, 70))
    max_bins = int(rng.choice([1, 2, 5, 16, 32, 64, 200, 256]))
    sym = skewed_symbols(rng, (L, T, C), max_bins, float(rng.choice([0.02, 0.3, 3.0])))
    cdf = cg.calculate_cdf(sym, max_bins)
    check_cdf(cdf, max_bins)
    streams, lengths = cg.encode(cdf, sym, 2 * T + 8)
    assert (lengths >= 4).all()
    assert np.array_equal(cg.decode(cdf, streams, lengths, T), sym)
    cat, ends = cg.concat_streams(streams, lengths)
    assert np.array_equal(cg.decode_prefsum(cdf, cat, ends, T), sym)


def test_cdf_matches_definition():
    rng = np.random.default_rng(1)
    sym = skewed_symbols(rng, (2, 300, 3), 16, 0.5)
    cdf = cg.calculate_cdf(sym, 16).view(np.uint16)
    for layer in range(2):
        for c in range(3):
            counts = np.bincount(sym[layer, :, c], minlength=16)
            cum = np.concatenate([[0], np.cumsum(counts)])
            want = cum * ((1 << 15) - 16) // 300 + np.arange(17)
            assert np.array_equal(cdf[layer, c], want)


def test_empty_stream_uses_uniform_cdf():
    sym = np.zeros((1, 0, 2), dtype=np.uint8)
    cdf = cg.calculate_cdf(sym, 8).view(np.uint16)
    assert np.array_equal(cdf[0, 0], (np.arange(9) * (1 << 15)) // 8)
    streams, lengths = cg.encode(cdf.view(np.int16), sym, 16)
    assert (lengths == 4).all()  # only the flush bytes


def test_single_symbol_alphabet_compresses():
    sym = np.full((1, 1000, 4), 3, dtype=np.uint8)
    cdf = cg.calculate_cdf(sym, 8)
    streams, lengths = cg.encode(cdf, sym, 64)
    assert (lengths < 40).all()
    assert np.array_equal(cg.decode(cdf, streams, lengths, 1000), sym)


def test_compression_tracks_entropy():
    rng = np.random.default_rng(2)
    p = np.exp(-np.arange(32) / 3.0)
    p /= p.sum()
    sym = rng.choice(32, size=(1, 4096, 8), p=p).astype(np.uint8)
    cdf = cg.calculate_cdf(sym, 32)
    _, lengths = cg.encode(cdf, sym, 8192)
    entropy_bytes = 4096 * -(p * np.log2(p)).sum() / 8
    assert lengths.max() < entropy_bytes * 1.05 + 8


def test_overflow_is_reported():
    rng = np.random.default_rng(3)
    sym = rng.integers(0, 256, size=(1, 200, 2), dtype=np.uint8)
    cdf = cg.calculate_cdf(sym, 256)
    streams, lengths = cg.encode(cdf, sym, 32)
    assert (lengths == -1).all()


def test_out_of_range_symbols_are_left_out_of_the_cdf():
    sym = np.array([[[0], [1], [9], [1]]], dtype=np.uint8)  # 9 >= max_bins
    cdf = cg.calculate_cdf(sym, 4).view(np.uint16)
    # counts over the 3 in-range symbols: 0 -> 1, 1 -> 2
    cum = np.array([0, 1, 3, 3, 3])
    assert np.array_equal(cdf[0, 0], cum * ((1 << 15) - 4) // 3 + np.arange(5))
