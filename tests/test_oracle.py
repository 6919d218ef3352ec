"""CPU tests of the transfer oracle: pinned to the golden fixtures made with the
reference's own test oracles (tests/golden/make_golden.py), and cross-checked
against those oracle expressions on seeded random cases."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import kv_transfer as oracle
from tests.golden.make_golden import (
    bf16_bits,
    c1_inputs,
    ref_retrieve_kv,
    ref_single_layer,
    ref_store_kv,
    ref_store_mla,
    sha,
    slots_with_skips,
)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def small():
    return dict(np.load(os.path.join(GOLDEN, "kv_small.npz")))


def test_golden_multi_layer_store_and_retrieve(small):
    L, nb, bs, heads, hd = small["kv_meta"].tolist()
    layers = list(small["kv_layers"])
    slots = small["kv_slots"]
    obj = np.zeros((2, L, len(slots), heads * hd), dtype=np.int16)
    oracle.multi_layer_kv_transfer(obj, layers, slots, nb * bs, True, False)
    assert np.array_equal(obj, small["kv_store"])
    new = [np.zeros_like(a) for a in layers]
    oracle.multi_layer_kv_transfer(obj, new, slots, nb * bs, False, False)
    assert np.array_equal(np.stack(new), small["kv_retrieve"])


def test_golden_mla_store(small):
    L, nb, bs, w = small["mla_meta"].tolist()
    slots = small["mla_slots"]
    obj = np.zeros((1, L, len(slots), w), dtype=np.int16)
    oracle.multi_layer_kv_transfer(obj, list(small["mla_layers"]), slots, 0, True, True)
    assert np.array_equal(obj, small["mla_store"])


@pytest.mark.parametrize("token_major", [True, False])
def test_golden_single_layer(small, token_major):
    slots = small["single_slots"]
    k, v = small["single_k"], small["single_v"]
    H = k.shape[-1] * k.shape[-2]
    shape = (len(slots), 2, H) if token_major else (2, len(slots), H)
    out = np.zeros(shape, dtype=np.int16)
    oracle.single_layer_kv_transfer(out, k, v, slots, True, token_major)
    want = small["single_token_major"] if token_major else small["single_kv_major"]
    assert np.array_equal(out, want)
    k2, v2 = np.zeros_like(k), np.zeros_like(v)
    oracle.single_layer_kv_transfer(out, k2, v2, slots, False, token_major)
    ok = slots[slots >= 0]
    assert np.array_equal(k2.reshape(-1, H)[ok], k.reshape(-1, H)[ok])
    assert np.array_equal(v2.reshape(-1, H)[ok], v.reshape(-1, H)[ok])


def test_golden_c1_digest():
    with open(os.path.join(GOLDEN, "c1_digest.json")) as f:
        d = json.load(f)
    spec, layers, slots = c1_inputs()
    assert sha(np.stack(layers)) == d["inputs_sha256"]
    assert sha(slots) == d["slots_sha256"]
    assert int((slots < 0).sum()) == d["skipped_slots"] == 16
    obj = np.zeros(spec.memobj_shape(len(slots)), dtype=np.int16)
    oracle.multi_layer_kv_transfer(obj, layers, slots, spec.page_buffer_size, True, False)
    assert sha(obj) == d["store_sha256"]
    new = [np.zeros_like(a) for a in layers]
    oracle.multi_layer_kv_transfer(obj, new, slots, spec.page_buffer_size, False, False)
    assert sha(np.stack(new)) == d["retrieve_sha256"]


@pytest.mark.parametrize("seed", range(6))
def test_oracle_matches_reference_expressions(seed):
    rng = np.random.default_rng(seed)
    L = int(rng.integers(1, 4))
    nb, bs = int(rng.integers(1, 9)), int(rng.choice([1, 4, 16]))
    heads, hd = int(rng.integers(1, 4)), int(rng.choice([2, 8, 16]))
    shape = (2, nb, bs, heads, hd)
    layers = [bf16_bits(rng, shape) for _ in range(L)]
    n = int(rng.integers(0, nb * bs + 1))
    slots = slots_with_skips(rng, nb * bs, n, int(rng.integers(0, n + 1)) if n else 0)
    want = ref_store_kv(layers, slots, heads, hd)
    got = np.zeros_like(want)
    oracle.multi_layer_kv_transfer(got, layers, slots, nb * bs, True, False)
    assert np.array_equal(got, want)
    new = [np.zeros_like(a) for a in layers]
    oracle.multi_layer_kv_transfer(got, new, slots, nb * bs, False, False)
    assert np.array_equal(np.stack(new), np.stack(ref_retrieve_kv(want, slots, shape, heads, hd)))
    # flash variants on the same data (K and V as separate caches)
    got2 = np.zeros_like(want)
    for layer in range(L):
        oracle.load_and_reshape_flash(got2, layers[layer][0], layers[layer][1], slots, layer)
    assert np.array_equal(got2, want)
    # MLA with the per-token loop
    mla = [bf16_bits(rng, (nb, bs, hd)) for _ in range(L)]
    want_m = ref_store_mla(mla, slots, bs)
    got_m = np.zeros_like(want_m)
    oracle.multi_layer_kv_transfer(got_m, mla, slots, 0, True, True)
    assert np.array_equal(got_m, want_m)
    # single layer both layouts
    for tm in (True, False):
        want_s = ref_single_layer(layers[0][0], layers[0][1], slots, tm)
        got_s = np.zeros_like(want_s)
        oracle.single_layer_kv_transfer(got_s, layers[0][0], layers[0][1], slots, True, tm)
        assert np.array_equal(got_s, want_s)


def test_skipped_and_out_of_range_rows_keep_their_values():
    rng = np.random.default_rng(3)
    layers = [bf16_bits(rng, (2, 4, 4, 1, 8))]
    slots = np.array([-1, 3, 16, 100, 0], dtype=np.int64)  # bound is 16
    obj = np.full((2, 1, 5, 8), 77, dtype=np.int16)
    oracle.multi_layer_kv_transfer(obj, layers, slots, 16, True, False)
    flat = layers[0].reshape(2, 16, 8)
    for t, s in enumerate(slots):
        for k in range(2):
            if 0 <= s < 16:
                assert np.array_equal(obj[k, 0, t], flat[k, s])
            else:
                assert (obj[k, 0, t] == 77).all()


def test_unilateral_oracle_matches_multi_layer():
    rng = np.random.default_rng(4)
    L, rows, H = 3, 40, 16
    k = [bf16_bits(rng, (rows, H)) for _ in range(L)]
    v = [bf16_bits(rng, (rows, H)) for _ in range(L)]
    slots = slots_with_skips(rng, rows, 25, 4)
    a = np.zeros((2, L, 25, H), dtype=np.int16)
    oracle.multi_layer_kv_transfer_unilateral(a, k, v, slots, True)
    b = np.zeros_like(a)
    oracle.multi_layer_kv_transfer(b, [np.stack([kk, vv]) for kk, vv in zip(k, v)], slots, rows,
                                   True, False)
    assert np.array_equal(a, b)


def test_dtype_agnostic_bit_copy():
    """The ops are row copies: fp32 bit patterns (incl. NaN payloads) survive."""
    rng = np.random.default_rng(5)
    raw = rng.integers(-2**31, 2**31 - 1, size=(2, 3, 4, 1, 4), dtype=np.int64).astype(np.int32)
    raw[0, 0, 0, 0, 0] = 0x7FC01234  # a NaN payload
    slots = np.array([0, 5, 11], dtype=np.int64)
    obj = np.zeros((2, 1, 3, 4), dtype=np.int32)
    oracle.multi_layer_kv_transfer(obj, [raw], slots, 12, True, False)
    assert obj[0, 0, 0, 0] == 0x7FC01234
    assert torch.equal(torch.from_numpy(obj[1, 0, 2]), torch.from_numpy(raw.reshape(2, 12, 4)[1, 11]))
