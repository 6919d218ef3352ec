"""GPU tests of the batched (many chunks, one launch) transfer:
c_ops.multi_layer_kv_transfer_batched and the connector's batched_from_gpu /
batched_to_gpu, against the oracle applied object by object."""

import numpy as np
import pytest
import torch

from lmcache_b200 import c_ops
from lmcache_b200 import workloads as wl
from lmcache_b200.v1.gpu_connector import VLLMPagedMemGPUConnectorV2
from lmcache_b200.v1.memory_management import PinMemoryAllocator, TensorMemoryObj
from oracle import kv_transfer as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


@pytest.fixture(params=["auto", "vector", "bulk-small-ring"])
def transfer_path(request, monkeypatch):
    if request.param == "vector":
        monkeypatch.setenv("LMCB_TRANSFER_PATH", "vector")
    elif request.param == "bulk-small-ring":
        monkeypatch.setenv("LMCB_TRANSFER_PATH", "bulk")
        monkeypatch.setenv("LMCB_BULK_STAGES", "2")
        monkeypatch.setenv("LMCB_BULK_STAGE_KB", "4")
        monkeypatch.setenv("LMCB_BULK_CTAS_PER_SM", "1")
    return request.param


@pytest.fixture(scope="module")
def arena():
    a = PinMemoryAllocator(512 << 20)
    yield a
    a.close()


# Object slot ranges: ragged sizes, an empty object, a gap and an out-of-order
# range, so the token-to-object search sees every case.
RANGES = [(0, 256), (256, 300), (300, 300), (512, 768), (310, 500), (800, 1000)]


def make_objects(spec, where, arena):
    objs, handles = [], []
    for s, e in RANGES:
        shape = spec.memobj_shape(e - s)
        if where == "hbm":
            objs.append(torch.zeros(shape, dtype=torch.bfloat16, device=DEV))
        else:
            mo = arena.allocate(shape, torch.bfloat16)
            mo.tensor.zero_()
            handles.append(mo)
            objs.append(mo.tensor)
    return objs, handles


@pytest.mark.parametrize("name", ["c1", "c4", "c5"])
@pytest.mark.parametrize("where", ["hbm", "pinned-zerocopy", "pinned-dma"])
def test_batched_matches_oracle(name, where, transfer_path, arena, monkeypatch):
    if where == "pinned-dma":
        monkeypatch.setenv("LMCB_HOST_RETRIEVE", "dma")
    elif where == "pinned-zerocopy":
        monkeypatch.setenv("LMCB_HOST_RETRIEVE", "zerocopy")
    spec = wl.SPECS[name]
    if name != "c1":
        import dataclasses

        spec = dataclasses.replace(spec, num_blocks=256)
    kv = wl.make_kv_caches(spec, DEV, seed=41)
    g = torch.Generator().manual_seed(42)
    slots = torch.randperm(spec.page_buffer_size, generator=g)[:1000].to(torch.int64)
    slots[torch.randperm(1000, generator=g)[:30]] = -1
    sd = slots.to(DEV)
    ptrs = wl.pointer_tensor(kv, DEV)
    pbs = spec.page_buffer_size
    objs, handles = make_objects(spec, "hbm" if where == "hbm" else "pinned", arena)
    c_ops.multi_layer_kv_transfer_batched(objs, ptrs, sd, [s for s, _ in RANGES],
                                          [e for _, e in RANGES], kv[0].device, pbs, True,
                                          spec.use_mla)
    torch.cuda.synchronize()
    kv_np = [bits(t) for t in kv]
    for obj, (s, e) in zip(objs, RANGES):
        want = np.zeros(obj.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, slots[s:e].numpy(), pbs, True, spec.use_mla)
        assert np.array_equal(bits(obj), want)
    # retrieve into zeroed caches
    kv_new = [torch.zeros_like(t) for t in kv]
    c_ops.multi_layer_kv_transfer_batched(objs, wl.pointer_tensor(kv_new, DEV), sd,
                                          [s for s, _ in RANGES], [e for _, e in RANGES],
                                          kv[0].device, pbs, False, spec.use_mla)
    torch.cuda.synchronize()
    new_np = [np.zeros_like(a) for a in kv_np]
    for obj, (s, e) in zip(objs, RANGES):
        oracle.multi_layer_kv_transfer(bits(obj), new_np, slots[s:e].numpy(), pbs, False,
                                       spec.use_mla)
    for a, b in zip(kv_new, new_np):
        assert np.array_equal(bits(a), b)
    for mo in handles:
        arena.free(mo)
    assert c_ops.device_status(torch.cuda.current_device()) == 0


def test_connector_batched_round_trip(arena):
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=43)
    slots = wl.make_slot_mapping(spec, seed=43)
    sd = slots.to(DEV)
    conn = VLLMPagedMemGPUConnectorV2(spec.hidden, spec.num_layers)
    starts, ends = [0, 100, 200], [100, 200, 256]
    objs = [arena.allocate(conn.get_shape(e - s), torch.bfloat16) for s, e in zip(starts, ends)]
    for mo in objs:
        mo.tensor.zero_()  # rows of skipped slots keep these zeros
    arena.free(objs[1])
    objs[1] = TensorMemoryObj.wrap(  # one HBM object among host objects
        torch.zeros(conn.get_shape(100), dtype=torch.bfloat16, device=DEV))
    conn.batched_from_gpu(objs, starts, ends, kvcaches=kv, slot_mapping=sd)
    kv_np = [bits(t) for t in kv]
    for mo, s, e in zip(objs, starts, ends):
        want = np.zeros(mo.tensor.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, slots[s:e].numpy(), spec.page_buffer_size,
                                       True, False)
        assert np.array_equal(bits(mo.tensor), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    conn.batched_to_gpu(objs, starts, ends, kvcaches=kv_new, slot_mapping=sd)
    torch.cuda.synchronize()
    valid = sd[sd >= 0]
    for a, b in zip(kv, kv_new):
        fa, fb = a.view(2, -1, spec.hidden), b.view(2, -1, spec.hidden)
        assert torch.equal(fa[:, valid], fb[:, valid])
    arena.free(objs[0])
    arena.free(objs[2])


@pytest.mark.parametrize("token_major", [True, False])
@pytest.mark.parametrize("where", ["hbm", "pinned"])
def test_single_layer_batched_matches_oracle(token_major, where, transfer_path, arena):
    num_blocks, block_size, heads, hd = 64, 16, 8, 128
    H = heads * hd
    g = torch.Generator(device=DEV).manual_seed(44)
    kc = torch.randn(num_blocks, block_size, heads, hd, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(num_blocks, block_size, heads, hd, generator=g, device=DEV).to(torch.bfloat16)
    gc = torch.Generator().manual_seed(45)
    slots = torch.randperm(num_blocks * block_size, generator=gc)[:1000].to(torch.int64)
    slots[torch.randperm(1000, generator=gc)[:20]] = -1
    sd = slots.to(DEV)
    objs, handles = [], []
    for s, e in RANGES:
        shape = (e - s, 2, H) if token_major else (2, e - s, H)
        if where == "hbm":
            objs.append(torch.zeros(shape, dtype=torch.bfloat16, device=DEV))
        else:
            mo = arena.allocate(shape, torch.bfloat16)
            mo.tensor.zero_()
            handles.append(mo)
            objs.append(mo.tensor)
    c_ops.single_layer_kv_transfer_batched(objs, kc, vc, sd, [s for s, _ in RANGES],
                                           [e for _, e in RANGES], True, token_major)
    torch.cuda.synchronize()
    k_np, v_np = bits(kc), bits(vc)
    for obj, (s, e) in zip(objs, RANGES):
        want = np.zeros(obj.shape, dtype=np.int16)
        oracle.single_layer_kv_transfer(want, k_np, v_np, slots[s:e].numpy(), True, token_major)
        assert np.array_equal(bits(obj), want)
    kn, vn = torch.zeros_like(kc), torch.zeros_like(vc)
    c_ops.single_layer_kv_transfer_batched(objs, kn, vn, sd, [s for s, _ in RANGES],
                                           [e for _, e in RANGES], False, token_major)
    torch.cuda.synchronize()
    kw, vw = np.zeros_like(k_np), np.zeros_like(v_np)
    for obj, (s, e) in zip(objs, RANGES):
        oracle.single_layer_kv_transfer(bits(obj), kw, vw, slots[s:e].numpy(), False, token_major)
    assert np.array_equal(bits(kn), kw)
    assert np.array_equal(bits(vn), vw)
    for mo in handles:
        arena.free(mo)
    assert c_ops.device_status(torch.cuda.current_device()) == 0


def test_many_objects_split_into_several_launches(transfer_path):
    """More objects than one launch's parameter table holds (255): the library
    splits the batch into launches of at most 255 objects each."""
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=46)
    g = torch.Generator().manual_seed(47)
    slots = torch.randperm(spec.page_buffer_size, generator=g)[:900].to(torch.int64)
    sd = slots.to(DEV)
    ptrs = wl.pointer_tensor(kv, DEV)
    pbs = spec.page_buffer_size
    ranges = [(3 * i, 3 * i + 3) for i in range(300)]  # 300 objects of 3 tokens
    ranges[7] = (21, 21)  # an empty one among them
    objs = [torch.zeros(spec.memobj_shape(e - s), dtype=torch.bfloat16, device=DEV)
            for s, e in ranges]
    c_ops.multi_layer_kv_transfer_batched(objs, ptrs, sd, [s for s, _ in ranges],
                                          [e for _, e in ranges], kv[0].device, pbs, True, False)
    torch.cuda.synchronize()
    kv_np = [bits(t) for t in kv]
    for obj, (s, e) in zip(objs, ranges):
        want = np.zeros(obj.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, slots[s:e].numpy(), pbs, True, False)
        assert np.array_equal(bits(obj), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    c_ops.multi_layer_kv_transfer_batched(objs, wl.pointer_tensor(kv_new, DEV), sd,
                                          [s for s, _ in ranges], [e for _, e in ranges],
                                          kv[0].device, pbs, False, False)
    torch.cuda.synchronize()
    new_np = [np.zeros_like(a) for a in kv_np]
    for obj, (s, e) in zip(objs, ranges):
        oracle.multi_layer_kv_transfer(bits(obj), new_np, slots[s:e].numpy(), pbs, False, False)
    for a, b in zip(kv_new, new_np):
        assert np.array_equal(bits(a), b)


def test_batched_calls_replay_from_a_cuda_graph():
    """The object table travels in the kernel parameters, so the batched calls
    can be captured: a graph captured once and replayed with new cache
    contents moves the new values, identical to eager calls."""
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=48)
    slots = wl.make_slot_mapping(spec, seed=48)
    sd = slots.to(DEV)
    ranges = [(0, 100), (100, 100), (100, 256)]
    starts, ends = [s for s, _ in ranges], [e for _, e in ranges]
    objs = [torch.zeros(spec.memobj_shape(e - s), dtype=torch.bfloat16, device=DEV)
            for s, e in ranges]
    ptrs = wl.pointer_tensor(kv, DEV)
    pbs = spec.page_buffer_size
    k, v = kv[0][0], kv[0][1]
    lmc = [torch.zeros((e - s, 2, spec.hidden), dtype=torch.bfloat16, device=DEV)
           for s, e in ranges]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up outside capture
        c_ops.multi_layer_kv_transfer_batched(objs, ptrs, sd, starts, ends, kv[0].device, pbs,
                                              True, False)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        c_ops.multi_layer_kv_transfer_batched(objs, ptrs, sd, starts, ends, kv[0].device, pbs,
                                              True, False)
        c_ops.single_layer_kv_transfer_batched(lmc, k, v, sd, starts, ends, True, True)
    for seed in (49, 50):
        g = torch.Generator(device=DEV).manual_seed(seed)
        for t in kv:
            t.normal_(generator=g)
        graph.replay()
        torch.cuda.synchronize()
        kv_np = [bits(t) for t in kv]
        k_np, v_np = bits(k), bits(v)
        for obj, one, (s, e) in zip(objs, lmc, ranges):
            want = np.zeros(obj.shape, dtype=np.int16)
            oracle.multi_layer_kv_transfer(want, kv_np, slots[s:e].numpy(), pbs, True, False)
            assert np.array_equal(bits(obj), want)
            want1 = np.zeros(one.shape, dtype=np.int16)
            oracle.single_layer_kv_transfer(want1, k_np, v_np, slots[s:e].numpy(), True, True)
            assert np.array_equal(bits(one), want1)
    graph.reset()
    assert c_ops.device_status(torch.cuda.current_device()) == 0
