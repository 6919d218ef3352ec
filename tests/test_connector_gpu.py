"""GPU tests of the connectors (lmcache_ascend/v1/npu_connector.py
counterparts): chunked from_gpu / to_gpu through VLLMPagedMemGPUConnectorV2
and the layerwise generators, checked against the oracle."""

import numpy as np
import pytest
import torch

from lmcache_b200 import workloads as wl
from lmcache_b200.v1.gpu_connector import (
    VLLMPagedMemGPUConnectorV2,
    VLLMPagedMemLayerwiseGPUConnector,
)
from lmcache_b200.v1.memory_management import PinMemoryAllocator
from oracle import kv_transfer as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


@pytest.fixture(scope="module")
def arena():
    a = PinMemoryAllocator(256 << 20)
    yield a
    a.close()


@pytest.mark.parametrize("name", ["c1", "c4"])
def test_v2_connector_chunks(name, arena):
    spec = wl.SPECS[name]
    kv = wl.make_kv_caches(spec, DEV, seed=8)
    slots = wl.make_slot_mapping(spec, seed=8)
    n = min(len(slots), 600)
    slots_dev = slots[:n].to(DEV)
    conn = VLLMPagedMemGPUConnectorV2(spec.hidden, spec.num_layers, use_mla=spec.use_mla)
    starts = list(range(0, n, 256))
    objs = []
    for s in starts:
        e = min(s + 256, n)
        mo = arena.allocate(conn.get_shape(e - s), torch.bfloat16)
        conn.from_gpu(mo, s, e, kvcaches=kv, slot_mapping=slots_dev)
        objs.append((s, e, mo))
    assert conn.page_buffer_size == spec.page_buffer_size
    kv_np = [bits(t) for t in kv]
    pbs = 0 if spec.use_mla else spec.page_buffer_size
    for s, e, mo in objs:
        want = np.zeros(mo.tensor.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, slots[s:e].numpy(), pbs, True, spec.use_mla)
        assert np.array_equal(bits(mo.tensor), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    for s, e, mo in objs:
        conn.to_gpu(mo, s, e, kvcaches=kv_new, slot_mapping=slots_dev)
    torch.cuda.synchronize()
    new_np = [np.zeros_like(a) for a in kv_np]
    for s, e, mo in objs:
        oracle.multi_layer_kv_transfer(bits(mo.tensor), new_np, slots[s:e].numpy(), pbs, False,
                                       spec.use_mla)
        arena.free(mo)
    for a, b in zip(kv_new, new_np):
        assert np.array_equal(bits(a), b)


@pytest.mark.parametrize("use_gpu", [False, True])
def test_layerwise_round_trip(use_gpu, arena):
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=9)
    slots = wl.make_slot_mapping(spec, seed=9)
    slots = slots[slots >= 0][:200]  # the staging path copies whole chunks
    slots_dev = slots.to(DEV)
    starts, ends = [0, 128], [128, 200]
    conn = VLLMPagedMemLayerwiseGPUConnector(spec.hidden, spec.num_layers, use_gpu=use_gpu)
    objs = [[arena.allocate(conn.get_shape(e - s), torch.bfloat16) for s, e in zip(starts, ends)]
            for _ in range(spec.num_layers)]
    gen = conn.batched_from_gpu(objs, starts, ends, kvcaches=kv, slot_mapping=slots_dev, sync=True)
    for _ in range(spec.num_layers + 1):
        next(gen)
    torch.cuda.synchronize()
    for layer in range(spec.num_layers):
        k_np, v_np = bits(kv[layer][0]), bits(kv[layer][1])
        for (s, e), mo in zip(zip(starts, ends), objs[layer]):
            want = np.zeros(mo.tensor.shape, dtype=np.int16)
            oracle.single_layer_kv_transfer(want, k_np, v_np, slots[s:e].numpy(), True, True)
            assert np.array_equal(bits(mo.tensor), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    gen = conn.batched_to_gpu(starts, ends, kvcaches=kv_new, slot_mapping=slots_dev, sync=True)
    next(gen)
    for layer in range(spec.num_layers):
        gen.send(objs[layer])
    next(gen)
    torch.cuda.synchronize()
    for a, b in zip(kv, kv_new):
        for k in range(2):
            fa, fb = a[k].reshape(-1, spec.hidden), b[k].reshape(-1, spec.hidden)
            assert torch.equal(fa[slots_dev], fb[slots_dev])
    for row in objs:
        for mo in row:
            arena.free(mo)
