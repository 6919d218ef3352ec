"""GPU tests of the connectors (lmcache_ascend/v1/npu_connector.py
counterparts): chunked from_gpu / to_gpu through VLLMPagedMemGPUConnectorV2
and the layerwise generators, checked against the oracle."""

import numpy as np
import pytest
import torch

from lmcache_b200 import workloads as wl
from lmcache_b200.v1.gpu_connector import (
    VLLMBufferLayerwiseGPUConnector,
    VLLMPagedMemGPUConnectorV2,
    VLLMPagedMemLayerwiseGPUConnector,
)
from lmcache_b200.v1.memory_management import MemoryFormat, PinMemoryAllocator
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
        fmt = MemoryFormat.KV_MLA_FMT if spec.use_mla else MemoryFormat.KV_2LTD
        mo = arena.allocate(conn.get_shape(e - s), torch.bfloat16, fmt)
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
    objs = [[arena.allocate(conn.get_shape(e - s), torch.bfloat16, MemoryFormat.KV_T2D)
             for s, e in zip(starts, ends)]
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


def test_v2_connector_checks_format_and_caches_pointers(arena):
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=10)
    slots = wl.make_slot_mapping(spec, seed=10).to(DEV)
    conn = VLLMPagedMemGPUConnectorV2(spec.hidden, spec.num_layers)
    wrong = arena.allocate(conn.get_shape(256), torch.bfloat16, MemoryFormat.KV_T2D)
    with pytest.raises(ValueError, match="format"):
        conn.from_gpu(wrong, 0, 256, kvcaches=kv, slot_mapping=slots)
    arena.free(wrong)
    mo = arena.allocate(conn.get_shape(256), torch.bfloat16, MemoryFormat.KV_2LTD)
    conn.from_gpu(mo, 0, 256, kvcaches=kv, slot_mapping=slots)
    dev_ptrs = conn.kv_cache_pointers_on_gpu[torch.cuda.current_device()]
    assert dev_ptrs.tolist() == [t.data_ptr() for t in kv]
    assert conn.pointer_uploads == 1
    # the same caches again: no new upload; other caches: one more
    conn.from_gpu(mo, 0, 256, kvcaches=kv, slot_mapping=slots)
    assert conn.pointer_uploads == 1
    kv2 = [torch.zeros_like(t) for t in kv]
    conn.to_gpu(mo, 0, 256, kvcaches=kv2, slot_mapping=slots)
    torch.cuda.synchronize()
    assert conn.pointer_uploads == 2
    assert dev_ptrs.tolist() == [t.data_ptr() for t in kv2]
    valid = slots[slots >= 0]
    for a, b in zip(kv, kv2):
        assert torch.equal(a.view(2, -1, spec.hidden)[:, valid], b.view(2, -1, spec.hidden)[:, valid])
    arena.free(mo)


def test_v2_connector_event_instead_of_sync(arena):
    """sync_host_objects=False: calls on host objects return at once and
    last_event marks when the data has arrived."""
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=11)
    slots = wl.make_slot_mapping(spec, seed=11)
    conn = VLLMPagedMemGPUConnectorV2(spec.hidden, spec.num_layers, sync_host_objects=False)
    objs = [arena.allocate(conn.get_shape(128), torch.bfloat16) for _ in range(2)]
    for mo in objs:
        mo.tensor.zero_()  # rows of skipped slots keep these zeros
    conn.batched_from_gpu(objs, [0, 128], [128, 256], kvcaches=kv, slot_mapping=slots.to(DEV))
    conn.last_event.synchronize()
    kv_np = [bits(t) for t in kv]
    for mo, (s, e) in zip(objs, [(0, 128), (128, 256)]):
        want = np.zeros(mo.tensor.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, slots[s:e].numpy(), spec.page_buffer_size,
                                       True, False)
        assert np.array_equal(bits(mo.tensor), want)
        arena.free(mo)


def test_buffer_layerwise_connector_is_the_staged_layerwise_path():
    spec = wl.SPECS["c1"]
    conn = VLLMBufferLayerwiseGPUConnector(spec.hidden, spec.num_layers)
    assert isinstance(conn, VLLMPagedMemLayerwiseGPUConnector) and conn.use_gpu
