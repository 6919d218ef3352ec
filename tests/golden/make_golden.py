"""Generates the golden fixtures of the transfer ops (tests/golden/kv_small.npz
and tests/golden/c1_digest.json).

The expected outputs are computed with the reference's own test oracles,
restated here in torch: fancy indexing ``cache.reshape(-1, heads, hd)[slots]``
(LMCache-Ascend tests/v1/test_mem_kernels.py:84-101), the per-token MLA loop
``kv_cache[layer][slot // block_size][slot % block_size]`` (:317-327) and
slot-indexed assignment for the write-back direction (the property checked by
tests/v1/utils.py:199-222). Skipped (-1) slots, which no reference test uses,
are masked out before indexing, so their destination rows keep their initial
values. Inputs are drawn from numpy's PCG64 generator, so the fixtures are
reproducible anywhere.

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def bf16_bits(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    """Seeded N(0, std^2) values rounded to bf16; returned as int16 bit patterns."""
    x = torch.from_numpy(rng.standard_normal(shape, dtype=np.float32) * std)
    return x.to(torch.bfloat16).view(torch.int16).numpy()


def slots_with_skips(rng, n_total, n, n_neg):
    s = rng.permutation(n_total)[:n].astype(np.int64)
    if n_neg:
        s[rng.permutation(n)[:n_neg]] = -1
    return s


def ref_store_kv(layers_bits, slots, heads, hd):
    """test_mem_kernels.py:84-101 with -1 slots masked: [2, L, T, H]."""
    T, L, H = len(slots), len(layers_bits), heads * hd
    out = np.zeros((2, L, T, H), dtype=np.int16)
    ok = torch.from_numpy(slots >= 0)
    idx = torch.from_numpy(slots)[ok]
    for layer, kv in enumerate(layers_bits):
        kvt = torch.from_numpy(kv)
        key_cache = kvt[0].reshape(-1, heads, hd)
        value_cache = kvt[1].reshape(-1, heads, hd)
        o = torch.from_numpy(out)
        o[0, layer][ok] = key_cache[idx].reshape(-1, H)
        o[1, layer][ok] = value_cache[idx].reshape(-1, H)
    return out


def ref_retrieve_kv(obj, slots, shape, heads, hd):
    """Write-back into zeroed caches: cache.reshape(-1, heads, hd)[slots] = rows."""
    L = obj.shape[1]
    ok = torch.from_numpy(slots >= 0)
    idx = torch.from_numpy(slots)[ok]
    outs = []
    for layer in range(L):
        new = torch.zeros(shape, dtype=torch.int16)
        for k in range(2):
            new[k].reshape(-1, heads, hd)[idx] = torch.from_numpy(obj[k, layer])[ok].reshape(
                -1, heads, hd)
        outs.append(new.numpy())
    return outs


def ref_store_mla(layers_bits, slots, block_size):
    """test_mem_kernels.py:317-327 per-token loop: [1, L, T, H]."""
    T, L, H = len(slots), len(layers_bits), layers_bits[0].shape[-1]
    out = np.zeros((1, L, T, H), dtype=np.int16)
    for layer in range(L):
        for t, slot in enumerate(slots.tolist()):
            if slot < 0:
                continue
            out[0, layer, t] = layers_bits[layer][slot // block_size][slot % block_size]
    return out


def ref_single_layer(k_bits, v_bits, slots, token_major):
    T, H = len(slots), k_bits.shape[-1] * k_bits.shape[-2]
    out = np.zeros((T, 2, H) if token_major else (2, T, H), dtype=np.int16)
    for k, cache in enumerate((k_bits, v_bits)):
        flat = cache.reshape(-1, H)
        for t, slot in enumerate(slots.tolist()):
            if slot < 0:
                continue
            if token_major:
                out[t, k] = flat[slot]
            else:
                out[k, t] = flat[slot]
    return out


def make_small(rng) -> dict:
    d = {}
    # multi-layer K/V: 2 layers, [2, 6 blocks, 4, 2 heads, 8] -> H = 16
    L, nb, bs, heads, hd = 2, 6, 4, 2, 8
    shape = (2, nb, bs, heads, hd)
    layers = [bf16_bits(rng, shape) for _ in range(L)]
    slots = slots_with_skips(rng, nb * bs, 10, 2)
    obj = ref_store_kv(layers, slots, heads, hd)
    d["kv_layers"] = np.stack(layers)
    d["kv_slots"] = slots
    d["kv_store"] = obj
    d["kv_retrieve"] = np.stack(ref_retrieve_kv(obj, slots, shape, heads, hd))
    d["kv_meta"] = np.array([L, nb, bs, heads, hd], dtype=np.int64)
    # MLA: 2 layers, [5 blocks, 4, 12]
    L2, nb2, bs2, w = 2, 5, 4, 12
    mla = [bf16_bits(rng, (nb2, bs2, w), 0.5) for _ in range(L2)]
    mslots = slots_with_skips(rng, nb2 * bs2, 7, 1)
    d["mla_layers"] = np.stack(mla)
    d["mla_slots"] = mslots
    d["mla_store"] = ref_store_mla(mla, mslots, bs2)
    d["mla_meta"] = np.array([L2, nb2, bs2, w], dtype=np.int64)
    # single layer: K and V caches [4 blocks, 4, 2, 4] -> H = 8
    kc = bf16_bits(rng, (4, 4, 2, 4))
    vc = bf16_bits(rng, (4, 4, 2, 4))
    sslots = slots_with_skips(rng, 16, 6, 1)
    d["single_k"] = kc
    d["single_v"] = vc
    d["single_slots"] = sslots
    d["single_token_major"] = ref_single_layer(kc, vc, sslots, True)
    d["single_kv_major"] = ref_single_layer(kc, vc, sslots, False)
    return d


def c1_inputs():
    """c1 workload inputs generated on the CPU: 4 layers of [2, 64, 16, 8, 128]
    bf16 ~N(0,1) from PCG64(0), slots from the workload generator (seed 0)."""
    sys.path.insert(0, os.path.join(ROOT, "lmcache-ascend_b200"))
    from lmcache_b200 import workloads as wl

    spec = wl.SPECS["c1"]
    rng = np.random.default_rng(0)
    layers = [bf16_bits(rng, spec.layer_shape) for _ in range(spec.num_layers)]
    slots = wl.make_slot_mapping(spec, seed=0).numpy()
    return spec, layers, slots


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    rng = np.random.default_rng(20261201)
    small = make_small(rng)
    np.savez_compressed(os.path.join(HERE, "kv_small.npz"), **small)
    spec, layers, slots = c1_inputs()
    store = ref_store_kv(layers, slots, spec.num_heads, spec.head_size)
    retrieve = ref_retrieve_kv(store, slots, tuple(spec.layer_shape), spec.num_heads,
                               spec.head_size)
    digest = {
        "workload": "c1",
        "inputs_sha256": sha(np.stack(layers)),
        "slots_sha256": sha(slots),
        "store_sha256": sha(store),
        "retrieve_sha256": sha(np.stack(retrieve)),
        "skipped_slots": int((slots < 0).sum()),
    }
    with open(os.path.join(HERE, "c1_digest.json"), "w") as f:
        json.dump(digest, f, indent=1)
        f.write("\n")
    print("wrote kv_small.npz and c1_digest.json")


if __name__ == "__main__":
    main()
