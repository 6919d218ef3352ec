"""GPU parity tests of the CacheGen kernels against the C oracle: identical
CDFs, byte-identical bitstreams and lengths, identical decoded symbols,
through c_ops (calculate_cdf / encode_fast_new / decode_fast_new /
decode_fast_prefsum) and the C ABI."""

import numpy as np
import pytest
import torch

from lmcache_b200 import abi, c_ops
from oracle import cachegen as cg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def symbols(seed, L, T, C, max_bins, conc=0.3):
    rng = np.random.default_rng(seed)
    out = np.empty((L, T, C), dtype=np.uint8)
    for c in range(C):  # a different distribution per channel
        p = rng.dirichlet(np.full(max_bins, conc))
        out[:, :, c] = rng.choice(max_bins, size=(L, T), p=p)
    return out


CASES = [
    # (L, T, C, max_bins): a KV chunk (32 layers x 256 tokens x 1024 channels,
    # 32 bins) plus ragged channel counts, tiny and full alphabets
    (32, 256, 1024, 32),
    (2, 1000, 130, 16),
    (3, 77, 33, 256),
    (1, 5, 1, 1),
    (4, 256, 96, 2),
    # every other power-of-two alphabet (each has its own search shape)
    (2, 300, 40, 4),
    (1, 200, 64, 8),
    (2, 150, 50, 64),
    (1, 100, 20, 128),
    # T >= 65536
    (1, 70000, 40, 16),
    # a ragged last group of channels with a 64-symbol alphabet
    (2, 120, 132, 64),
]


@pytest.mark.parametrize("L,T,C,max_bins", CASES)
def test_codec_matches_oracle(L, T, C, max_bins):
    sym = symbols(L * 7 + C, L, T, C, max_bins)
    sym_dev = torch.from_numpy(sym.view(np.int8)).to(DEV)
    cdf_dev = c_ops.calculate_cdf(sym_dev, max_bins)
    cdf_ref = cg.calculate_cdf(sym, max_bins)
    assert np.array_equal(cdf_dev.cpu().numpy(), cdf_ref)

    cap = 2 * T + 16
    out = torch.zeros((L, C, cap), dtype=torch.uint8, device=DEV)
    lengths = torch.zeros((L, C), dtype=torch.int32, device=DEV)
    c_ops.encode_fast_new(cdf_dev, sym_dev, out, lengths)
    ref_streams, ref_len = cg.encode(cdf_ref, sym, cap)
    assert np.array_equal(lengths.cpu().numpy(), ref_len)
    assert np.array_equal(out.cpu().numpy(), ref_streams)  # bytes past each length stay zero

    dec = torch.zeros_like(sym_dev)
    c_ops.decode_fast_new(cdf_dev, out, lengths, dec)
    assert np.array_equal(dec.cpu().numpy().view(np.uint8), sym)

    cat, ends = cg.concat_streams(ref_streams, ref_len)
    dec2 = torch.zeros_like(sym_dev)
    c_ops.decode_fast_prefsum(cdf_dev, torch.from_numpy(cat).to(DEV),
                              torch.from_numpy(ends).to(DEV), dec2)
    assert np.array_equal(dec2.cpu().numpy().view(np.uint8), sym)
    assert c_ops.device_status(torch.cuda.current_device()) == 0


def test_unaligned_stride_uses_byte_path():
    L, T, C, mb = 2, 300, 40, 32
    sym = symbols(5, L, T, C, mb)
    sym_dev = torch.from_numpy(sym.view(np.int8)).to(DEV)
    cdf = c_ops.calculate_cdf(sym_dev, mb)
    cap = 2 * T + 3  # not a multiple of 4
    out = torch.zeros((L, C, cap), dtype=torch.uint8, device=DEV)
    lengths = torch.zeros((L, C), dtype=torch.int32, device=DEV)
    c_ops.encode_fast_new(cdf, sym_dev, out, lengths)
    ref_streams, ref_len = cg.encode(cdf.cpu().numpy(), sym, cap)
    assert np.array_equal(out.cpu().numpy(), ref_streams)
    assert np.array_equal(lengths.cpu().numpy(), ref_len)


def test_overflow_and_out_of_range_flags():
    L, T, C, mb = 1, 400, 8, 256
    rng = np.random.default_rng(9)
    sym = rng.integers(0, 256, size=(L, T, C), dtype=np.uint8)
    sym_dev = torch.from_numpy(sym.view(np.int8)).to(DEV)
    c_ops.device_status(torch.cuda.current_device())
    cdf = c_ops.calculate_cdf(sym_dev, mb)
    out = torch.zeros((L, C, 64), dtype=torch.uint8, device=DEV)
    lengths = torch.zeros((L, C), dtype=torch.int32, device=DEV)
    c_ops.encode_fast_new(cdf, sym_dev, out, lengths)
    torch.cuda.synchronize()
    assert (lengths.cpu() == -1).all()
    assert c_ops.device_status(torch.cuda.current_device()) & abi.LMCB_DEVICE_FLAG_STREAM_OVERFLOW
    ref_streams, _ = cg.encode(cdf.cpu().numpy(), sym, 64)
    assert np.array_equal(out.cpu().numpy(), ref_streams)  # the first 64 bytes still match
    # symbols >= max_bins are flagged by calculate_cdf
    small = torch.from_numpy(np.array([[[0], [9]]], dtype=np.int8)).to(DEV)
    c_ops.calculate_cdf(small, 4)
    torch.cuda.synchronize()
    assert c_ops.device_status(torch.cuda.current_device()) & abi.LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE
    # several channels: the out-of-range symbol is left out of its channel's counts
    wide = np.zeros((1, 3, 8), dtype=np.uint8)
    wide[0, 1, 5] = 9
    cdf_w = c_ops.calculate_cdf(torch.from_numpy(wide.view(np.int8)).to(DEV), 4)
    torch.cuda.synchronize()
    assert c_ops.device_status(torch.cuda.current_device()) & abi.LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE
    assert np.array_equal(cdf_w.cpu().numpy(), cg.calculate_cdf(wide, 4))


def test_empty_token_axis():
    sym_dev = torch.zeros((2, 0, 5), dtype=torch.int8, device=DEV)
    cdf = c_ops.calculate_cdf(sym_dev, 8)
    assert np.array_equal(cdf.cpu().numpy(), cg.calculate_cdf(np.zeros((2, 0, 5), np.uint8), 8))
    out = torch.zeros((2, 5, 8), dtype=torch.uint8, device=DEV)
    lengths = torch.zeros((2, 5), dtype=torch.int32, device=DEV)
    c_ops.encode_fast_new(cdf, sym_dev, out, lengths)
    assert (lengths.cpu() == 4).all()


@pytest.mark.parametrize("max_bins", [32, 21, 256, 2])
def test_decode_of_arbitrary_bytes_matches_oracle(max_bins):
    """Random bytes decoded with valid CDFs: the decoder's search sees values
    of (code - low) / r at and above 2^15 (the clamp), and every length from
    empty to the full capacity. Symbols must still match the oracle's."""
    L, T, C = 2, 300, 70
    rng = np.random.default_rng(max_bins)
    sym = symbols(max_bins, L, T, C, max_bins)
    cdf = cg.calculate_cdf(sym, max_bins)
    cap = 96
    streams = rng.integers(0, 256, size=(L, C, cap), dtype=np.uint8)
    lengths = rng.integers(0, cap + 1, size=(L, C)).astype(np.int32)
    lengths[0, :3] = [0, cap, 4]
    want = cg.decode(cdf, streams, lengths, T)
    dec = torch.zeros((L, T, C), dtype=torch.int8, device=DEV)
    c_ops.decode_fast_new(torch.from_numpy(cdf).to(DEV), torch.from_numpy(streams).to(DEV),
                          torch.from_numpy(lengths).to(DEV), dec)
    assert np.array_equal(dec.cpu().numpy().view(np.uint8), want)
    cat, ends = cg.concat_streams(streams, lengths)
    want2 = cg.decode_prefsum(cdf, cat, ends, T)
    dec2 = torch.zeros_like(dec)
    c_ops.decode_fast_prefsum(torch.from_numpy(cdf).to(DEV), torch.from_numpy(cat).to(DEV),
                              torch.from_numpy(ends).to(DEV), dec2)
    assert np.array_equal(dec2.cpu().numpy().view(np.uint8), want2)


def wide_cdf(rng, L, C, max_bins):
    """Strictly increasing CDF rows whose values may pass 2^15 (up to 65535):
    probes at and above 2^15 are never accepted, and cdf[a + 1] - cdf[a] may
    be anything from 1 up. Strictly increasing keeps every interval non-empty,
    so the oracle's renormalisation ends."""
    steps = rng.integers(1, 2 * 65535 // max(max_bins, 1) + 2, size=(L, C, max_bins + 1))
    rows = np.cumsum(steps, axis=-1) - steps[..., :1] + rng.integers(0, 50, size=(L, C, 1))
    rows = np.minimum(rows, 65535 - (max_bins - np.arange(max_bins + 1)))
    assert (np.diff(rows, axis=-1) >= 1).all()
    return rows.astype(np.uint16).view(np.int16)  # the int16 bit patterns c_ops takes


@pytest.mark.parametrize("max_bins", [3, 4, 5, 8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("kind", ["valid", "wide"])
def test_decode_search_shapes_match_oracle(max_bins, kind):
    """Random bytes through every search shape (alphabets of 4 to 256 symbols
    search from registers, then in one or two shared-memory rounds; others by
    halving with bounds tests), with CDFs from calculate_cdf or with rows that
    pass 2^15."""
    L, T, C = 2, 200, 67
    rng = np.random.default_rng(1000 + max_bins)
    if kind == "valid":
        cdf = cg.calculate_cdf(symbols(max_bins + 7, L, T, C, max_bins), max_bins)
    else:
        cdf = wide_cdf(rng, L, C, max_bins)
    cap = 80
    streams = rng.integers(0, 256, size=(L, C, cap), dtype=np.uint8)
    lengths = rng.integers(0, cap + 1, size=(L, C)).astype(np.int32)
    want = cg.decode(cdf, streams, lengths, T)
    dec = torch.zeros((L, T, C), dtype=torch.int8, device=DEV)
    c_ops.decode_fast_new(torch.from_numpy(cdf).to(DEV), torch.from_numpy(streams).to(DEV),
                          torch.from_numpy(lengths).to(DEV), dec)
    assert np.array_equal(dec.cpu().numpy().view(np.uint8), want)
