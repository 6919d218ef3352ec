"""CPU oracle of LMCache-Ascend's paged KV-cache transfer ops (test infrastructure).

This module is test infrastructure, not the product: only the tests, the smoke check
and the CPU-baseline leg of the benchmark may import it. Nothing on the
product path calls into it.

Every function restates, in numpy, the semantics of one reference op on the
same layouts, operating in place like the reference. Arrays may have any
element type: the ops are pure row copies, so callers pass bit views
(for example ``torch_bf16_tensor.view(torch.int16).numpy()``) and results are
compared bit for bit.

Semantics sources (paths within LMCache-Ascend):
  * multi_layer_kv_transfer: csrc/mem_kernels.cpp:29-47 (address formula,
    direction flag), :59-65 (kv_size, MLA); the test oracles
    tests/v1/test_mem_kernels.py:84-101 (``key_cache[slot_mapping]``) and
    :317-327 (MLA per-token loop); page_buffer_size from
    lmcache_ascend/v1/npu_connector.py:34-41.
  * single_layer_kv_transfer: csrc/mem_kernels.cpp:108-117 (layouts
    [T, 2, H] token-major or [2, T, H]).
  * load_and_reshape_flash / reshape_and_cache_back_flash:
    csrc/mem_kernels.cpp:154-159, :200-206, :190-193, :237-240.
  * Slot ids < 0 are skipped (the destination row keeps its value); slot ids
    at or beyond the paged row count are skipped as well (the reference does
    not bound-check; the B200 library skips and flags them).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np


def _valid(slots: np.ndarray, num_rows: int | None) -> tuple[np.ndarray, np.ndarray]:
    """Token positions whose slot is used, and those slots."""
    slots = np.asarray(slots).astype(np.int64)
    ok = slots >= 0
    if num_rows is not None and num_rows > 0:
        ok &= slots < num_rows
    t = np.nonzero(ok)[0]
    return t, slots[t]


def multi_layer_kv_transfer(
    key_value: np.ndarray,
    paged_layers: Sequence[np.ndarray],
    slot_mapping: np.ndarray,
    page_buffer_size: int,
    direction: bool,
    use_mla: bool,
) -> None:
    """multi_layer_kv_transfer (csrc/mem_kernels.cpp:48-92).

    key_value     [kv, L, T, H]; kv = 2, or 1 with use_mla
    paged_layers  L arrays; each is viewed as [kv, page_buffer_size, H]
                  (K/V: [2, nb, bs, heads, hd]; MLA: [nb, bs, H], where
                  page_buffer_size may be 0 as the reference's MLA tests pass)
    direction     True: paged -> key_value (store); False: the reverse.
    """
    kv = 1 if use_mla else 2
    num_layers = key_value.shape[1]
    hidden = key_value.shape[-1]
    for layer in range(num_layers):
        # Row (k, slot) of a layer lives at flat row k * page_buffer_size + slot
        # (csrc/mem_kernels.cpp:40-42); with MLA only k = 0 exists.
        flat = paged_layers[layer].reshape(-1, hidden)
        bound = flat.shape[0] if use_mla else page_buffer_size
        t, s = _valid(slot_mapping, bound)
        for k in range(kv):
            rows = k * page_buffer_size + s
            if direction:
                key_value[k, layer, t, :] = flat[rows, :]
            else:
                flat[rows, :] = key_value[k, layer, t, :]


def multi_layer_kv_transfer_unilateral(
    key_value: np.ndarray,
    key_layers: Sequence[np.ndarray],
    value_layers: Sequence[np.ndarray],
    slot_mapping: np.ndarray,
    direction: bool,
) -> None:
    """multi_layer_kv_transfer_unilateral with separate K and V caches per
    layer, each viewed as [rows, H] (the SGLang-style layout of
    tests/v1/utils.py:94-125; the reference op itself is a stub,
    csrc/mem_kernels.cpp:95-105)."""
    num_layers = key_value.shape[1]
    hidden = key_value.shape[-1]
    for layer in range(num_layers):
        for k, caches in enumerate((key_layers, value_layers)):
            view = caches[layer].reshape(-1, hidden)
            t, s = _valid(slot_mapping, view.shape[0])
            if direction:
                key_value[k, layer, t, :] = view[s, :]
            else:
                view[s, :] = key_value[k, layer, t, :]


def single_layer_kv_transfer(
    lmc_kv: np.ndarray,
    key_cache: np.ndarray,
    value_cache: np.ndarray,
    slot_mapping: np.ndarray,
    direction: bool,
    token_major: bool,
) -> None:
    """single_layer_kv_transfer (csrc/mem_kernels.cpp:108-152).

    lmc_kv  [T, 2, H] if token_major else [2, T, H]
    caches  [nb, bs, heads, hd] (viewed as [nb * bs, H])
    """
    hidden = lmc_kv.shape[-1]
    for k, cache in enumerate((key_cache, value_cache)):
        view = cache.reshape(-1, hidden)
        t, s = _valid(slot_mapping, view.shape[0])
        if token_major:
            if direction:
                lmc_kv[t, k, :] = view[s, :]
            else:
                view[s, :] = lmc_kv[t, k, :]
        else:
            if direction:
                lmc_kv[k, t, :] = view[s, :]
            else:
                view[s, :] = lmc_kv[k, t, :]


def load_and_reshape_flash(
    key_value: np.ndarray,
    key_cache: np.ndarray,
    value_cache: np.ndarray,
    slot_mapping: np.ndarray,
    layer_idx: int,
) -> None:
    """load_and_reshape_flash: paged -> layer ``layer_idx`` of a [2, L, T, H]
    object (csrc/mem_kernels.cpp:154-198, page2L = true)."""
    _flash(key_value, key_cache, value_cache, slot_mapping, layer_idx, True)


def reshape_and_cache_back_flash(
    key_value: np.ndarray,
    key_cache: np.ndarray,
    value_cache: np.ndarray,
    slot_mapping: np.ndarray,
    layer_idx: int,
) -> None:
    """reshape_and_cache_back_flash: layer ``layer_idx`` of a [2, L, T, H]
    object -> paged (csrc/mem_kernels.cpp:200-245, page2L = false)."""
    _flash(key_value, key_cache, value_cache, slot_mapping, layer_idx, False)


def _flash(key_value, key_cache, value_cache, slot_mapping, layer_idx, page2L) -> None:
    hidden = key_value.shape[-1]
    for k, cache in enumerate((key_cache, value_cache)):
        view = cache.reshape(-1, hidden)
        t, s = _valid(slot_mapping, view.shape[0])
        if page2L:
            key_value[k, layer_idx, t, :] = view[s, :]
        else:
            view[s, :] = key_value[k, layer_idx, t, :]
