"""GPU parity tests of the transfer ops against the CPU oracle.

Ported from LMCache-Ascend's tests/v1/test_mem_kernels.py (same shapes,
num_tokens in {256, 500, 1024, 8000}, chunk 256, bf16), made deterministic
(seeded slots) and extended with skipped (-1) slots, fp16/fp32, int32 slot ids,
HBM and pinned-host LMCache objects, and the benchmark workloads c1-c5.
Every comparison is bit-exact.
"""

import numpy as np
import pytest
import torch

from lmcache_b200 import c_ops
from lmcache_b200 import workloads as wl
from lmcache_b200.v1.memory_management import PinMemoryAllocator
from oracle import kv_transfer as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def bits(t: torch.Tensor) -> np.ndarray:
    """Bit view of a tensor as a numpy integer array (same shape)."""
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.detach().cpu().contiguous().view(view).numpy()


def seeded_slots(n_total: int, n: int, seed: int, n_neg: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    s = torch.randperm(n_total, generator=g)[:n].to(torch.int64)
    if n_neg:
        s[torch.randperm(n, generator=g)[:n_neg]] = -1
    return s


def kv_list(num_layers, num_blocks, block_size, heads, hd, dtype, seed, mla=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    shape = [num_blocks, block_size, hd] if mla else [2, num_blocks, block_size, heads, hd]
    out = []
    for _ in range(num_layers):
        t = torch.empty(shape, dtype=dtype, device=DEV)
        if dtype.is_floating_point:
            t.normal_(generator=g)
        else:
            t.random_(generator=g)
        out.append(t)
    return out


def ptrs_of(caches):
    return torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64).to(DEV)


@pytest.fixture(params=["auto", "vector", "bulk-small-ring"])
def transfer_path(request, monkeypatch):
    """Runs a test under the default path choice, the vectorised LD/ST kernel,
    and the bulk-copy kernel with a minimal ring (2 stages of 4 KB) so stage
    reuse and partial groups are exercised."""
    if request.param == "vector":
        monkeypatch.setenv("LMCB_TRANSFER_PATH", "vector")
    elif request.param == "bulk-small-ring":
        monkeypatch.setenv("LMCB_TRANSFER_PATH", "bulk")
        monkeypatch.setenv("LMCB_BULK_STAGES", "2")
        monkeypatch.setenv("LMCB_BULK_STAGE_KB", "4")
        monkeypatch.setenv("LMCB_BULK_CTAS_PER_SM", "1")
    return request.param


@pytest.fixture(scope="module")
def pin_alloc():
    a = PinMemoryAllocator(3 << 30)
    yield a
    a.close()


# ---------------------------------------------------------------------------
# multi_layer_kv_transfer (tests/v1/test_mem_kernels.py:159-284)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("num_tokens", [256, 500, 1024, 8000])
@pytest.mark.parametrize("memobj_on", ["hbm", "pinned"])
def test_multi_layer_kernel(num_tokens, memobj_on, pin_alloc, transfer_path):
    num_layers, num_blocks, block_size, heads, hd, chunk = 32, 1000, 16, 8, 128, 256
    dtype = torch.bfloat16
    pbs = num_blocks * block_size
    kv = kv_list(num_layers, num_blocks, block_size, heads, hd, dtype, seed=num_tokens)
    slots = seeded_slots(pbs, num_tokens, seed=num_tokens, n_neg=num_tokens // 16)
    slots_dev = slots.to(DEV)
    ptrs = ptrs_of(kv)
    kv_np = [bits(t) for t in kv]

    objs, handles = [], []
    for sc in torch.split(slots_dev, chunk):
        shape = [2, num_layers, len(sc), heads * hd]
        if memobj_on == "pinned":
            mo = pin_alloc.allocate(shape, dtype)
            assert mo is not None
            mo.tensor.zero_()
            handles.append(mo)
            t = mo.tensor
        else:
            t = torch.zeros(shape, dtype=dtype, device=DEV)
        c_ops.multi_layer_kv_transfer(t, ptrs, sc, kv[0].device, pbs, True, False)
        objs.append(t)
    torch.cuda.synchronize()

    for t, sc in zip(objs, torch.split(slots, chunk)):
        want = np.zeros(t.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, sc.numpy(), pbs, True, False)
        assert np.array_equal(bits(t), want)

    # Round trip into fresh caches (test_mem_kernels.py:247-282).
    kv_new = [torch.zeros_like(t) for t in kv]
    ptrs_new = ptrs_of(kv_new)
    for t, sc in zip(objs, torch.split(slots_dev, chunk)):
        c_ops.multi_layer_kv_transfer(t, ptrs_new, sc, kv_new[0].device, pbs, False, False)
    torch.cuda.synchronize()
    new_np = [np.zeros_like(a) for a in kv_np]
    for t, sc in zip(objs, torch.split(slots, chunk)):
        oracle.multi_layer_kv_transfer(bits(t), new_np, sc.numpy(), pbs, False, False)
    for got, want in zip(kv_new, new_np):
        assert np.array_equal(bits(got), want)
    for mo in handles:
        pin_alloc.free(mo)
    assert c_ops.device_status(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("num_tokens", [256, 500, 1024, 8000])
def test_multi_layer_kernel_use_mla(num_tokens, pin_alloc, transfer_path):
    num_layers, num_blocks, block_size, hd, chunk = 32, 1000, 64, 576, 256
    dtype = torch.bfloat16
    kv = kv_list(num_layers, num_blocks, block_size, 1, hd, dtype, seed=7 + num_tokens, mla=True)
    # Skipped (-1) slots: with page_buffer_size = 0 the MLA path has no paged
    # bound, so the skip rests on the slot's sign alone.
    slots = seeded_slots(num_blocks * block_size, num_tokens, seed=num_tokens,
                         n_neg=num_tokens // 16)
    slots_dev = slots.to(DEV)
    ptrs = ptrs_of(kv)
    kv_np = [bits(t) for t in kv]
    objs = []
    for i, sc in enumerate(torch.split(slots_dev, chunk)):
        if i % 2:
            obj = pin_alloc.allocate([1, num_layers, len(sc), hd], dtype)
        else:  # alternate pinned-host and HBM objects
            obj = type("Obj", (), {})()
            obj.tensor = torch.empty([1, num_layers, len(sc), hd], dtype=dtype, device=DEV)
        obj.tensor.zero_()
        # page_buffer_size = 0 as the reference's MLA callers pass it (:359).
        c_ops.multi_layer_kv_transfer(obj.tensor, ptrs, sc, kv[0].device, 0, True, True)
        objs.append(obj)
    torch.cuda.synchronize()
    for obj, sc in zip(objs, torch.split(slots, chunk)):
        want = np.zeros(obj.tensor.shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, kv_np, sc.numpy(), 0, True, True)
        assert np.array_equal(bits(obj.tensor), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    ptrs_new = ptrs_of(kv_new)
    for obj, sc in zip(objs, torch.split(slots_dev, chunk)):
        c_ops.multi_layer_kv_transfer(obj.tensor, ptrs_new, sc, kv_new[0].device, 0, False, True)
    torch.cuda.synchronize()
    valid = slots_dev[slots_dev >= 0]
    for a, b in zip(kv, kv_new):
        fa, fb = a.reshape(-1, hd), b.reshape(-1, hd)
        assert torch.equal(fa[valid], fb[valid])
    # the whole caches, untouched rows included, equal the oracle's
    new_np = [np.zeros_like(a) for a in kv_np]
    for obj, sc in zip(objs, torch.split(slots, chunk)):
        oracle.multi_layer_kv_transfer(bits(obj.tensor), new_np, sc.numpy(), 0, False, True)
    for got, want in zip(kv_new, new_np):
        assert np.array_equal(bits(got), want)
    assert c_ops.device_status(torch.cuda.current_device()) == 0
    for i, obj in enumerate(objs):
        if i % 2:
            pin_alloc.free(obj)


# ---------------------------------------------------------------------------
# single_layer_kv_transfer (tests/v1/test_mem_kernels.py:424-476)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("num_tokens", [256, 500, 1024, 8000])
@pytest.mark.parametrize("token_major", [True, False])
def test_single_layer_kernel(num_tokens, token_major, transfer_path):
    num_layers, num_blocks, block_size, heads, hd = 32, 1000, 16, 8, 128
    dtype = torch.bfloat16
    H = heads * hd
    kv = kv_list(num_layers, num_blocks, block_size, heads, hd, dtype, seed=3)
    kv_new = [torch.zeros_like(t) for t in kv]
    slots = seeded_slots(num_blocks * block_size, num_tokens, seed=num_tokens + 1, n_neg=5)
    slots_dev = slots.to(DEV)
    shape = (num_tokens, 2, H) if token_major else (2, num_tokens, H)
    buf = torch.zeros(shape, dtype=dtype, device=DEV)
    for layer in range(num_layers):
        check = layer % 8 == 0
        if check:
            want = bits(buf).copy()  # skipped rows keep their previous values
        c_ops.single_layer_kv_transfer(buf, kv[layer][0], kv[layer][1], slots_dev, True, token_major)
        if check:
            k_np, v_np = bits(kv[layer][0]), bits(kv[layer][1])
            oracle.single_layer_kv_transfer(want, k_np, v_np, slots.numpy(), True, token_major)
            assert np.array_equal(bits(buf), want)
        c_ops.single_layer_kv_transfer(
            buf, kv_new[layer][0], kv_new[layer][1], slots_dev, False, token_major)
    torch.cuda.synchronize()
    valid = slots_dev[slots_dev >= 0]
    for a, b in zip(kv, kv_new):
        for k in range(2):
            fa, fb = a[k].reshape(-1, heads, hd), b[k].reshape(-1, heads, hd)
            assert torch.equal(fa[valid], fb[valid])
            untouched = torch.ones(fb.shape[0], dtype=torch.bool, device=DEV)
            untouched[valid] = False
            assert not fb[untouched].any()


# ---------------------------------------------------------------------------
# load_and_reshape_flash / reshape_and_cache_back_flash (:59-156)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("num_tokens", [256, 500, 1024, 8000])
def test_extract_and_load_back(num_tokens, pin_alloc, transfer_path):
    num_layers, num_blocks, block_size, heads, hd, chunk = 32, 1000, 16, 8, 128, 256
    dtype = torch.bfloat16
    H = heads * hd
    g = torch.Generator(device=DEV).manual_seed(11)
    kv = [(torch.randn(num_blocks, block_size, heads, hd, generator=g, device=DEV).to(dtype),
           torch.randn(num_blocks, block_size, heads, hd, generator=g, device=DEV).to(dtype))
          for _ in range(num_layers)]
    slots = seeded_slots(num_blocks * block_size, num_tokens, seed=num_tokens + 2, n_neg=3)
    slots_dev = slots.to(DEV)
    objs = []
    for i, sc in enumerate(torch.split(slots_dev, chunk)):
        if i % 2:
            obj = pin_alloc.allocate([2, num_layers, len(sc), H], dtype)
        else:  # alternate pinned-host and HBM objects
            obj = type("Obj", (), {})()
            obj.tensor = torch.empty([2, num_layers, len(sc), H], dtype=dtype, device=DEV)
        obj.tensor.zero_()
        for layer in range(num_layers):
            c_ops.load_and_reshape_flash(obj.tensor, kv[layer][0], kv[layer][1], sc, layer)
        objs.append(obj)
    torch.cuda.synchronize()
    k_np = [bits(k) for k, _ in kv]
    v_np = [bits(v) for _, v in kv]
    for obj, sc in zip(objs, torch.split(slots, chunk)):
        want = np.zeros(obj.tensor.shape, dtype=np.int16)
        for layer in range(num_layers):
            oracle.load_and_reshape_flash(want, k_np[layer], v_np[layer], sc.numpy(), layer)
        assert np.array_equal(bits(obj.tensor), want)
    kv_new = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in kv]
    for obj, sc in zip(objs, torch.split(slots_dev, chunk)):
        for layer in range(num_layers):
            c_ops.reshape_and_cache_back_flash(obj.tensor, kv_new[layer][0], kv_new[layer][1], sc, layer)
    torch.cuda.synchronize()
    for layer in range(num_layers):
        kw, vw = np.zeros_like(k_np[layer]), np.zeros_like(v_np[layer])
        for obj, sc in zip(objs, torch.split(slots, chunk)):
            oracle.reshape_and_cache_back_flash(bits(obj.tensor), kw, vw, sc.numpy(), layer)
        assert np.array_equal(bits(kv_new[layer][0]), kw)
        assert np.array_equal(bits(kv_new[layer][1]), vw)
    for i, obj in enumerate(objs):
        if i % 2:
            pin_alloc.free(obj)


# ---------------------------------------------------------------------------
# dtypes, slot dtypes, unilateral, edge cases
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("heads,hd", [(8, 128), (1, 128), (2, 48), (1, 3)])
def test_dtypes_and_row_widths(dtype, slot_dtype, heads, hd, transfer_path):
    num_layers, num_blocks, block_size = 3, 40, 16
    pbs = num_blocks * block_size
    kv = kv_list(num_layers, num_blocks, block_size, heads, hd, dtype, seed=5)
    slots = seeded_slots(pbs, 300, seed=9, n_neg=20)
    obj = torch.zeros([2, num_layers, 300, heads * hd], dtype=dtype, device=DEV)
    c_ops.multi_layer_kv_transfer(obj, ptrs_of(kv), slots.to(slot_dtype).to(DEV),
                                  kv[0].device, pbs, True, False)
    want = np.zeros(obj.shape, dtype=bits(obj).dtype)
    oracle.multi_layer_kv_transfer(want, [bits(t) for t in kv], slots.numpy(), pbs, True, False)
    assert np.array_equal(bits(obj), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    c_ops.multi_layer_kv_transfer(obj, ptrs_of(kv_new), slots.to(slot_dtype).to(DEV),
                                  kv[0].device, pbs, False, False)
    new_np = [np.zeros_like(bits(t)) for t in kv]
    oracle.multi_layer_kv_transfer(bits(obj), new_np, slots.numpy(), pbs, False, False)
    for a, b in zip(kv_new, new_np):
        assert np.array_equal(bits(a), b)


def test_unilateral(transfer_path):
    num_layers, rows, heads, hd = 4, 512, 8, 128
    dtype = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(2)
    kc = [torch.randn(rows, heads, hd, generator=g, device=DEV).to(dtype) for _ in range(num_layers)]
    vc = [torch.randn(rows, heads, hd, generator=g, device=DEV).to(dtype) for _ in range(num_layers)]
    slots = seeded_slots(rows, 200, seed=4, n_neg=7)
    obj = torch.zeros([2, num_layers, 200, heads * hd], dtype=dtype, device=DEV)
    c_ops.multi_layer_kv_transfer_unilateral(obj, ptrs_of(kc), ptrs_of(vc), slots.to(DEV),
                                             kc[0].device, rows, True)
    want = np.zeros(obj.shape, dtype=np.int16)
    oracle.multi_layer_kv_transfer_unilateral(want, [bits(t) for t in kc], [bits(t) for t in vc],
                                              slots.numpy(), True)
    assert np.array_equal(bits(obj), want)
    kn = [torch.zeros_like(t) for t in kc]
    vn = [torch.zeros_like(t) for t in vc]
    c_ops.multi_layer_kv_transfer_unilateral(obj, ptrs_of(kn), ptrs_of(vn), slots.to(DEV),
                                             kc[0].device, rows, False)
    kw = [np.zeros_like(bits(t)) for t in kc]
    vw = [np.zeros_like(bits(t)) for t in vc]
    oracle.multi_layer_kv_transfer_unilateral(bits(obj), kw, vw, slots.numpy(), False)
    for a, b in zip(kn + vn, kw + vw):
        assert np.array_equal(bits(a), b)


def test_inputs_written_by_the_preceding_kernel(transfer_path):
    """The slot mapping and the layer-pointer array are rewritten by a torch
    kernel right before every transfer on the same stream (as when an engine
    builds the slot mapping on the GPU). The transfer kernels start early under
    programmatic dependent launch, so this pins that they read neither input
    before the previous kernel's writes are visible."""
    L, nb, bs, heads, hd, T, n = 8, 256, 16, 8, 128, 256, 12
    pbs = nb * bs
    kv_a = kv_list(L, nb, bs, heads, hd, torch.bfloat16, seed=51)
    kv_b = kv_list(L, nb, bs, heads, hd, torch.bfloat16, seed=52)
    ptr_src = [ptrs_of(kv_a), ptrs_of(kv_b)]
    perm = torch.randperm(pbs, generator=torch.Generator().manual_seed(53))
    slot_sets = [perm[i * T:(i + 1) * T].to(torch.int32) for i in range(n)]
    slot_src = [s.to(DEV) for s in slot_sets]
    sd = torch.full((T,), -1, dtype=torch.int64, device=DEV)
    ptrs = torch.zeros(L, dtype=torch.int64, device=DEV)
    objs = [torch.zeros([2, L, T, heads * hd], dtype=torch.bfloat16, device=DEV) for _ in range(n)]
    torch.cuda.synchronize()
    for i in range(n):
        sd.copy_(slot_src[i])  # int32 -> int64: an elementwise kernel
        torch.add(ptr_src[i % 2], 0, out=ptrs)
        c_ops.multi_layer_kv_transfer(objs[i], ptrs, sd, kv_a[0].device, pbs, True, False)
    torch.cuda.synchronize()
    np_a, np_b = [bits(t) for t in kv_a], [bits(t) for t in kv_b]
    for i in range(n):
        want = np.zeros(objs[i].shape, dtype=np.int16)
        oracle.multi_layer_kv_transfer(want, np_a if i % 2 == 0 else np_b,
                                       slot_sets[i].numpy().astype(np.int64), pbs, True, False)
        assert np.array_equal(bits(objs[i]), want), i
    # retrieve each object back into fresh caches, the same way
    new_a = [torch.zeros_like(t) for t in kv_a]
    new_b = [torch.zeros_like(t) for t in kv_b]
    new_src = [ptrs_of(new_a), ptrs_of(new_b)]
    torch.cuda.synchronize()
    for i in range(n):
        sd.copy_(slot_src[i])
        torch.add(new_src[i % 2], 0, out=ptrs)
        c_ops.multi_layer_kv_transfer(objs[i], ptrs, sd, kv_a[0].device, pbs, False, False)
    torch.cuda.synchronize()
    want_a = [np.zeros_like(a) for a in np_a]
    want_b = [np.zeros_like(b) for b in np_b]
    for i in range(n):
        oracle.multi_layer_kv_transfer(bits(objs[i]), want_a if i % 2 == 0 else want_b,
                                       slot_sets[i].numpy().astype(np.int64), pbs, False, False)
    for got, want in zip(new_a + new_b, want_a + want_b):
        assert np.array_equal(bits(got), want)
    assert c_ops.device_status(torch.cuda.current_device()) == 0


def test_empty_and_all_skipped():
    kv = kv_list(2, 8, 16, 8, 128, torch.bfloat16, seed=1)
    ptrs = ptrs_of(kv)
    obj = torch.zeros([2, 2, 0, 1024], dtype=torch.bfloat16, device=DEV)
    c_ops.multi_layer_kv_transfer(obj, ptrs, torch.empty(0, dtype=torch.int64, device=DEV),
                                  kv[0].device, 128, True, False)
    obj = torch.full([2, 2, 64, 1024], 3.0, dtype=torch.bfloat16, device=DEV)
    c_ops.multi_layer_kv_transfer(obj, ptrs, torch.full((64,), -1, dtype=torch.int64, device=DEV),
                                  kv[0].device, 128, True, False)
    torch.cuda.synchronize()
    assert bool((obj == 3.0).all())
    assert c_ops.device_status(torch.cuda.current_device()) == 0


def test_out_of_range_slot_is_skipped_and_flagged(transfer_path):
    kv = kv_list(2, 8, 16, 8, 128, torch.bfloat16, seed=1)
    pbs = 8 * 16
    slots = torch.tensor([0, 5, pbs, pbs + 100, 127], dtype=torch.int64)
    obj = torch.full([2, 2, 5, 1024], 7.0, dtype=torch.bfloat16, device=DEV)
    c_ops.device_status(torch.cuda.current_device())  # clear
    c_ops.multi_layer_kv_transfer(obj, ptrs_of(kv), slots.to(DEV), kv[0].device, pbs, True, False)
    torch.cuda.synchronize()
    assert c_ops.device_status(torch.cuda.current_device()) & 0x1
    want = bits(torch.full([2, 2, 5, 1024], 7.0, dtype=torch.bfloat16))
    oracle.multi_layer_kv_transfer(want, [bits(t) for t in kv], slots.numpy(), pbs, True, False)
    assert np.array_equal(bits(obj), want)


def test_misaligned_layer_pointer_falls_back(transfer_path):
    """A layer base that is 2-byte but not 16-byte aligned is copied byte-wise."""
    heads, hd, nb, bs = 2, 64, 16, 16
    backing = torch.randn(2 * nb * bs * heads * hd + 1, device=DEV).to(torch.bfloat16)
    layer = backing[1:].view(2, nb, bs, heads, hd)  # base address offset by 2 bytes
    pbs = nb * bs
    slots = seeded_slots(pbs, 50, seed=3)
    obj = torch.zeros([2, 1, 50, heads * hd], dtype=torch.bfloat16, device=DEV)
    ptrs = torch.tensor([layer.data_ptr()], dtype=torch.int64).to(DEV)
    c_ops.multi_layer_kv_transfer(obj, ptrs, slots.to(DEV), layer.device, pbs, True, False)
    want = np.zeros(obj.shape, dtype=np.int16)
    oracle.multi_layer_kv_transfer(want, [bits(layer)], slots.numpy(), pbs, True, False)
    assert np.array_equal(bits(obj), want)


def test_unregistered_host_object_is_rejected():
    kv = kv_list(1, 8, 16, 8, 128, torch.bfloat16, seed=1)
    obj = torch.zeros([2, 1, 4, 1024], dtype=torch.bfloat16).pin_memory()
    with pytest.raises(RuntimeError, match="host registered pointer"):
        c_ops.multi_layer_kv_transfer(obj, ptrs_of(kv), torch.zeros(4, dtype=torch.int64, device=DEV),
                                      kv[0].device, 128, True, False)


# ---------------------------------------------------------------------------
# Benchmark workloads
# ---------------------------------------------------------------------------


def test_workload_c1_round_trip():
    """c1 at full size against the oracle, both directions."""
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=0)
    slots = wl.make_slot_mapping(spec, seed=0)
    assert int((slots < 0).sum()) == 16
    ptrs = wl.pointer_tensor(kv, DEV)
    obj = torch.zeros(spec.memobj_shape(256), dtype=torch.bfloat16, device=DEV)
    c_ops.multi_layer_kv_transfer(obj, ptrs, slots.to(DEV), kv[0].device,
                                  spec.page_buffer_size, True, False)
    want = np.zeros(obj.shape, dtype=np.int16)
    kv_np = [bits(t) for t in kv]
    oracle.multi_layer_kv_transfer(want, kv_np, slots.numpy(), spec.page_buffer_size, True, False)
    assert np.array_equal(bits(obj), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    c_ops.multi_layer_kv_transfer(obj, wl.pointer_tensor(kv_new, DEV), slots.to(DEV),
                                  kv[0].device, spec.page_buffer_size, False, False)
    new_np = [np.zeros_like(a) for a in kv_np]
    oracle.multi_layer_kv_transfer(want, new_np, slots.numpy(), spec.page_buffer_size, False, False)
    for a, b in zip(kv_new, new_np):
        assert np.array_equal(bits(a), b)


@pytest.mark.parametrize("name", ["c2", "c3", "c4", "c5"])
@pytest.mark.parametrize("memobj_on", ["hbm", "pinned"])
def test_workload_full_size(name, memobj_on, pin_alloc):
    """Full-size paged buffers; the first, a middle and the last chunk are
    stored, checked against the oracle on three sampled layers, then
    round-tripped: the chunk's paged rows are zeroed, retrieved from the
    object, and stored again into a second object that must equal the first."""
    spec = wl.SPECS[name]
    kv = wl.make_kv_caches(spec, DEV, seed=1)
    slots = wl.make_slot_mapping(spec, seed=1)
    ptrs = wl.pointer_tensor(kv, DEV)
    pbs = 0 if spec.use_mla else spec.page_buffer_size
    chunk_list = wl.chunks(slots, spec.chunk_size)
    picks = [0, len(chunk_list) // 2, len(chunk_list) - 1]
    layers = [0, spec.num_layers // 2, spec.num_layers - 1]
    layer_bits = {layer: bits(kv[layer]) for layer in layers}

    def new_obj(shape):
        if memobj_on == "pinned":
            mo = pin_alloc.allocate(shape, torch.bfloat16)
            assert mo is not None
            return mo, mo.tensor
        return None, torch.empty(shape, dtype=torch.bfloat16, device=DEV)

    for ci in picks:
        sc = chunk_list[ci]
        sd = sc.to(DEV)
        shape = spec.memobj_shape(len(sc))
        mo, obj = new_obj(shape)
        c_ops.multi_layer_kv_transfer(obj, ptrs, sd, kv[0].device, pbs, True, spec.use_mla)
        torch.cuda.synchronize()
        got = bits(obj)
        for layer in layers:
            want = np.zeros((spec.kv, 1, len(sc), spec.hidden), dtype=np.int16)
            oracle.multi_layer_kv_transfer(want, [layer_bits[layer]], sc.numpy(), pbs, True,
                                           spec.use_mla)
            assert np.array_equal(got[:, layer : layer + 1], want)
        for t in kv:
            t.view(spec.kv, -1, spec.hidden)[:, sd, :] = 0
        c_ops.multi_layer_kv_transfer(obj, ptrs, sd, kv[0].device, pbs, False, spec.use_mla)
        mo2, obj2 = new_obj(shape)
        obj2.zero_()
        c_ops.multi_layer_kv_transfer(obj2, ptrs, sd, kv[0].device, pbs, True, spec.use_mla)
        torch.cuda.synchronize()
        assert np.array_equal(bits(obj2), got)
        for m in (mo, mo2):
            if m is not None:
                pin_alloc.free(m)
    assert c_ops.device_status(torch.cuda.current_device()) == 0
    del kv
    torch.cuda.empty_cache()


@pytest.mark.parametrize("ctas_per_sm", ["1", "3", "default-path"])
def test_large_single_launch(ctas_per_sm, monkeypatch):
    """One launch of 262144 rows: each bulk-copy CTA resolves many 256-row
    batches and its ring wraps many times."""
    if ctas_per_sm != "default-path":
        monkeypatch.setenv("LMCB_BULK_CTAS_PER_SM", ctas_per_sm)
        # large launches default to the vectorised kernel; force the bulk ring
        monkeypatch.setenv("LMCB_TRANSFER_PATH", "bulk")
    num_layers, num_blocks, block_size, heads, hd, T = 32, 512, 16, 8, 128, 4096
    pbs = num_blocks * block_size
    kv = kv_list(num_layers, num_blocks, block_size, heads, hd, torch.bfloat16, seed=21)
    slots = seeded_slots(pbs, T, seed=22, n_neg=100)
    obj = torch.zeros([2, num_layers, T, heads * hd], dtype=torch.bfloat16, device=DEV)
    c_ops.multi_layer_kv_transfer(obj, ptrs_of(kv), slots.to(DEV), kv[0].device, pbs, True, False)
    kv_np = [bits(t) for t in kv]
    want = np.zeros(obj.shape, dtype=np.int16)
    oracle.multi_layer_kv_transfer(want, kv_np, slots.numpy(), pbs, True, False)
    assert np.array_equal(bits(obj), want)
    kv_new = [torch.zeros_like(t) for t in kv]
    c_ops.multi_layer_kv_transfer(obj, ptrs_of(kv_new), slots.to(DEV), kv[0].device, pbs, False,
                                  False)
    new_np = [np.zeros_like(a) for a in kv_np]
    oracle.multi_layer_kv_transfer(want, new_np, slots.numpy(), pbs, False, False)
    for a, b in zip(kv_new, new_np):
        assert np.array_equal(bits(a), b)
    assert c_ops.device_status(torch.cuda.current_device()) == 0
