"""Property tests of the oracles (CPU, hypothesis): invariants that hold for
any shape, independent of the golden fixtures.

Transfer: a store followed by a retrieve into empty caches puts back exactly
the rows of valid slots and touches nothing else; a store leaves the object
rows of skipped slots as they were; storing twice changes nothing.
CacheGen: decode(encode(x)) == x for any alphabet size and symbol
distribution that fits the capacity; the concatenated-stream decode equals
the fixed-stride one; the CDF is strictly increasing from 0 to 2^15.
"""

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import cachegen as cg
from oracle import kv_transfer as oracle


@st.composite
def transfer_case(draw):
    L = draw(st.integers(1, 3))
    nb = draw(st.integers(1, 6))
    bs = draw(st.sampled_from([1, 2, 4, 16]))
    H = draw(st.sampled_from([1, 3, 8, 64]))
    pbs = nb * bs
    T = draw(st.integers(0, pbs))
    seed = draw(st.integers(0, 2**31 - 1))
    rng = np.random.default_rng(seed)
    slots = rng.permutation(pbs)[:T].astype(np.int64)
    n_skip = draw(st.integers(0, T))
    if n_skip:
        slots[rng.permutation(T)[:n_skip]] = -1
    layers = [rng.integers(-2**15, 2**15, size=(2, pbs, H), dtype=np.int16) for _ in range(L)]
    return L, pbs, H, slots, layers, rng


@settings(max_examples=60, deadline=None)
@given(transfer_case())
def test_store_then_retrieve_puts_back_exactly_the_valid_rows(case):
    L, pbs, H, slots, layers, rng = case
    T = len(slots)
    sentinel = rng.integers(-2**15, 2**15, size=(2, L, T, H), dtype=np.int16)
    obj = sentinel.copy()
    oracle.multi_layer_kv_transfer(obj, layers, slots, pbs, True, False)
    valid = slots >= 0
    for l in range(L):
        for kv in range(2):
            assert np.array_equal(obj[kv, l, valid], layers[l][kv, slots[valid]])
            # rows of skipped slots keep what the object held
            assert np.array_equal(obj[kv, l, ~valid], sentinel[kv, l, ~valid])
    again = obj.copy()
    oracle.multi_layer_kv_transfer(again, layers, slots, pbs, True, False)
    assert np.array_equal(again, obj)  # idempotent
    new = [np.zeros_like(a) for a in layers]
    oracle.multi_layer_kv_transfer(obj, new, slots, pbs, False, False)
    touched = np.zeros(pbs, dtype=bool)
    touched[slots[valid]] = True
    for l in range(L):
        assert np.array_equal(new[l][:, touched], layers[l][:, touched])
        assert not new[l][:, ~touched].any()


@settings(max_examples=40, deadline=None)
@given(transfer_case(), st.booleans())
def test_single_layer_round_trip(case, token_major):
    _, pbs, H, slots, layers, _ = case
    k, v = layers[0][0], layers[0][1]
    T = len(slots)
    shape = (T, 2, H) if token_major else (2, T, H)
    obj = np.zeros(shape, dtype=np.int16)
    oracle.single_layer_kv_transfer(obj, k, v, slots, True, token_major)
    kn, vn = np.zeros_like(k), np.zeros_like(v)
    oracle.single_layer_kv_transfer(obj, kn, vn, slots, False, token_major)
    valid = slots[slots >= 0]
    assert np.array_equal(kn[valid], k[valid]) and np.array_equal(vn[valid], v[valid])
    rest = np.ones(pbs, dtype=bool)
    rest[valid] = False
    assert not kn[rest].any() and not vn[rest].any()


@st.composite
def codec_case(draw):
    L = draw(st.integers(1, 2))
    T = draw(st.integers(0, 120))
    C = draw(st.integers(1, 9))
    max_bins = draw(st.sampled_from([1, 2, 3, 7, 16, 32, 33, 100, 256]))
    conc = draw(st.sampled_from([0.05, 0.3, 1.0, 10.0]))
    seed = draw(st.integers(0, 2**31 - 1))
    rng = np.random.default_rng(seed)
    p = rng.dirichlet(np.full(max_bins, conc))
    sym = rng.choice(max_bins, size=(L, T, C), p=p).astype(np.uint8)
    return sym, max_bins


@settings(max_examples=60, deadline=None)
@given(codec_case())
def test_codec_round_trip_and_cdf_shape(case):
    sym, max_bins = case
    L, T, C = sym.shape
    cdf = cg.calculate_cdf(sym, max_bins)
    c16 = cdf.view(np.uint16).astype(np.int64)
    assert (c16[..., 0] == 0).all() and (c16[..., -1] == 1 << 15).all()
    assert (np.diff(c16, axis=-1) >= 1).all()  # every symbol keeps a nonzero frequency
    cap = 2 * T + 16  # at most 15 bits a symbol plus the final four bytes
    streams, lengths = cg.encode(cdf, sym, cap)
    assert (lengths >= 4).all() and (lengths <= cap).all()
    assert np.array_equal(cg.decode(cdf, streams, lengths, T), sym)
    cat, ends = cg.concat_streams(streams, lengths)
    assert np.array_equal(cg.decode_prefsum(cdf, cat, ends, T), sym)
