"""GPU connectors: the callers of the transfer ops on the LMCache side.

CUDA counterparts of LMCache-Ascend's connectors
(lmcache_ascend/v1/npu_connector.py), written against this package's c_ops
instead of the Ascend module:

* VLLMPagedMemGPUConnectorV2 -- non-layerwise. ``_initialize_pointers``
  provides the per-device int64 array of per-layer KV base addresses and the
  page buffer size (npu_connector.py:24-43); ``from_gpu`` / ``to_gpu`` move
  one chunk between the paged KV cache and a MemoryObj with one
  ``multi_layer_kv_transfer`` launch (store: direction True), and
  ``batched_from_gpu`` / ``batched_to_gpu`` move many chunks in one launch.
* VLLMPagedMemLayerwiseGPUConnector -- layerwise generators
  ``batched_to_gpu`` / ``batched_from_gpu`` (npu_connector.py:46-262): every
  chunk of a layer in one ``single_layer_kv_transfer_batched`` launch on a
  dedicated load / store CUDA stream, or through a device staging buffer
  (``use_gpu``).
* VLLMBufferLayerwiseGPUConnector -- the name the reference's buffer
  layerwise connector has (npu_connector.py:20-21, a pass-through subclass);
  here it is the layerwise connector with its staging buffer on.

Upstream LMCache is not a dependency: the classes implement the part of the
upstream base-class behaviour these methods rely on (constructor fields,
``get_shape``, ``initialize_kvcaches_ptr``).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch

from .. import c_ops
from .memory_management import MemoryFormat, MemoryObj

KV_2LTD = MemoryFormat.KV_2LTD  # [2, num_layers, num_tokens, hidden]
KV_T2D = MemoryFormat.KV_T2D  # [num_tokens, 2, hidden]
KV_MLA_FMT = MemoryFormat.KV_MLA_FMT  # [1, num_layers, num_tokens, hidden]


def _check_format(memory_obj: MemoryObj, want: MemoryFormat) -> None:
    """Objects carrying metadata must be in the layout the transfer writes
    (npu_connector.py:117 asserts KV_T2D for the layerwise path)."""
    meta = getattr(memory_obj, "metadata", None)
    if meta is not None and meta.fmt != want:
        raise ValueError(f"memory object format is {meta.fmt!r}, the transfer needs {want!r}")


class VLLMPagedMemGPUConnectorV2:
    """Paged vLLM KV cache <-> LMCache object, all layers per launch.

    :param hidden_dim_size: elements per token row (heads * head_size, or the
        MLA latent width).
    :param num_layers: number of attention layers.
    :param use_mla: one latent row per token instead of K and V rows.
    :param sync_host_objects: when a call moves data to or from an object in
        host memory, return only once the data is there (default True). This
        is LMCache's contract for the connector: the engine hands a stored
        object to its storage backends right after ``from_gpu`` returns, with
        no CUDA event to wait on, and may reuse a retrieved object after
        ``to_gpu``. With False the calls return at once and ``last_event``
        (a CUDA event recorded after the call's work) tells the caller when
        the data has arrived.
    """

    def __init__(self, hidden_dim_size: int, num_layers: int, use_gpu: bool = False, **kwargs):
        self.hidden_dim_size = hidden_dim_size
        self.num_layers = num_layers
        self.use_gpu = use_gpu
        self.use_mla = bool(kwargs.get("use_mla", False))
        self.sync_host_objects = bool(kwargs.get("sync_host_objects", True))
        self.kv_cache_pointers = torch.empty(num_layers, dtype=torch.int64, device="cpu",
                                             pin_memory=torch.cuda.is_available())
        self.kv_cache_pointers_on_gpu: Dict[int, torch.Tensor] = {}
        # per device: the layer addresses its device array currently holds
        self._pointers_held: Dict[int, Tuple[int, ...]] = {}
        self.pointer_uploads = 0  # host-to-device copies of the address array
        self.page_buffer_size = 0
        self.last_event: Optional[torch.cuda.Event] = None

    def get_shape(self, num_tokens: int) -> torch.Size:
        kv = 1 if self.use_mla else 2
        return torch.Size([kv, self.num_layers, num_tokens, self.hidden_dim_size])

    def _initialize_pointers(self, kv_caches: List[torch.Tensor]) -> torch.Tensor:
        """The device array of per-layer base addresses and page_buffer_size
        (npu_connector.py:24-43 on CUDA devices).

        The reference copies the addresses to the device on every call, a
        copy that waits for the stream. Here the array is copied only when
        the set of cache addresses differs from what the device array holds
        (in practice once: vLLM allocates its KV cache once)."""
        ptrs = tuple(t.data_ptr() for t in kv_caches)
        device = kv_caches[0].device
        assert device.type == "cuda", "The device should be a CUDA GPU."
        idx = device.index if device.index is not None else torch.cuda.current_device()
        if idx not in self.kv_cache_pointers_on_gpu:
            self.kv_cache_pointers_on_gpu[idx] = torch.empty(
                self.num_layers, dtype=torch.int64, device=device)
        if self._pointers_held.get(idx) != ptrs:
            self.kv_cache_pointers.numpy()[:] = ptrs
            self.kv_cache_pointers_on_gpu[idx].copy_(self.kv_cache_pointers)
            self._pointers_held[idx] = ptrs
            self.pointer_uploads += 1
        if self.use_mla:
            # [num_pages, page_size, head_size] or [1, num_pages, page_size, head_size]
            self.page_buffer_size = kv_caches[0].shape[-3] * kv_caches[0].shape[-2]
        else:
            # [2, num_pages, page_size, num_heads, head_size]
            assert kv_caches[0].dim() == 5
            self.page_buffer_size = kv_caches[0].shape[1] * kv_caches[0].shape[2]
        return self.kv_cache_pointers_on_gpu[idx]

    def _transfer(self, memory_obj: MemoryObj, start: int, end: int, direction: bool,
                  **kwargs) -> None:
        assert memory_obj.tensor is not None
        if "kvcaches" not in kwargs:
            raise ValueError("'kvcaches' should be provided in kwargs.")
        if "slot_mapping" not in kwargs:
            raise ValueError("'slot_mapping' should be provided in kwargs.")
        kvcaches: List[torch.Tensor] = kwargs["kvcaches"]
        slot_mapping: torch.Tensor = kwargs["slot_mapping"]
        _check_format(memory_obj, KV_MLA_FMT if self.use_mla else KV_2LTD)
        ptrs = self._initialize_pointers(kvcaches)
        c_ops.multi_layer_kv_transfer(memory_obj.tensor, ptrs, slot_mapping[start:end],
                                      kvcaches[0].device, self.page_buffer_size, direction,
                                      self.use_mla)
        self._finish(not memory_obj.tensor.is_cuda)

    def _finish(self, host_objects: bool) -> None:
        """Records ``last_event``; waits for it when host objects were moved
        and sync_host_objects is set."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream())
        self.last_event = ev
        if host_objects and self.sync_host_objects:
            ev.synchronize()

    def _batched(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                 ends: Sequence[int], direction: bool, **kwargs) -> None:
        if "kvcaches" not in kwargs:
            raise ValueError("'kvcaches' should be provided in kwargs.")
        if "slot_mapping" not in kwargs:
            raise ValueError("'slot_mapping' should be provided in kwargs.")
        kvcaches: List[torch.Tensor] = kwargs["kvcaches"]
        slot_mapping: torch.Tensor = kwargs["slot_mapping"]
        ptrs = self._initialize_pointers(kvcaches)
        # One launch per residency group (device objects / pinned host objects).
        want = KV_MLA_FMT if self.use_mla else KV_2LTD
        groups: Dict[bool, list] = {}
        for obj, s, e in zip(memory_objs, starts, ends):
            assert obj.tensor is not None
            _check_format(obj, want)
            groups.setdefault(obj.tensor.is_cuda, []).append((obj.tensor, int(s), int(e)))
        for items in groups.values():
            c_ops.multi_layer_kv_transfer_batched(
                [t for t, _, _ in items], ptrs, slot_mapping, [s for _, s, _ in items],
                [e for _, _, e in items], kvcaches[0].device, self.page_buffer_size, direction,
                self.use_mla)
        self._finish(False in groups)

    def batched_from_gpu(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                         ends: Sequence[int], **kwargs) -> None:
        """Store several chunks with one kernel launch (upstream LMCache calls
        ``from_gpu`` once per chunk here)."""
        self._batched(memory_objs, starts, ends, True, **kwargs)

    def batched_to_gpu(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                       ends: Sequence[int], **kwargs) -> None:
        """Load several chunks back with one kernel launch."""
        self._batched(memory_objs, starts, ends, False, **kwargs)

    def from_gpu(self, memory_obj: MemoryObj, start: int, end: int, **kwargs) -> None:
        """Store tokens [start, end) of the paged cache into ``memory_obj``."""
        self._transfer(memory_obj, start, end, True, **kwargs)

    def to_gpu(self, memory_obj: MemoryObj, start: int, end: int, **kwargs) -> None:
        """Load ``memory_obj`` back into the paged cache at tokens [start, end)."""
        self._transfer(memory_obj, start, end, False, **kwargs)


class VLLMPagedMemLayerwiseGPUConnector:
    """Layer-by-layer transfers for pipelined prefill / decode
    (npu_connector.py:46-262). ``kvcaches[layer]`` is a [2, nb, bs, heads,
    head_size] tensor; objects are KV_T2D [num_tokens, 2, hidden]."""

    def __init__(self, hidden_dim_size: int, num_layers: int, use_gpu: bool = False, **kwargs):
        self.hidden_dim_size = hidden_dim_size
        self.num_layers = num_layers
        self.use_gpu = use_gpu
        self.dtype = kwargs.get("dtype", torch.bfloat16)
        self.device = kwargs.get("device", "cuda")
        self.kvcaches: Optional[List[torch.Tensor]] = None
        self.load_stream = torch.cuda.Stream()
        self.store_stream = torch.cuda.Stream()

    def get_shape(self, num_tokens: int) -> torch.Size:
        return torch.Size([num_tokens, 2, self.hidden_dim_size])

    def initialize_kvcaches_ptr(self, **kwargs) -> None:
        if "kvcaches" in kwargs:
            self.kvcaches = kwargs["kvcaches"]

    def _staging(self, num_tokens: int) -> torch.Tensor:
        return torch.empty(self.get_shape(num_tokens), dtype=self.dtype,
                           device=self.kvcaches[0].device)

    def _layer_batched(self, memory_objs_layer: Sequence[MemoryObj], layer_id: int,
                       slot_mapping: torch.Tensor, starts: Sequence[int], ends: Sequence[int],
                       direction: bool) -> None:
        """One single_layer_kv_transfer_batched launch per residency group."""
        groups: Dict[bool, list] = {}
        for obj, s, e in zip(memory_objs_layer, starts, ends):
            assert obj.tensor is not None
            _check_format(obj, KV_T2D)
            groups.setdefault(obj.tensor.is_cuda, []).append((obj.tensor, int(s), int(e)))
        for items in groups.values():
            c_ops.single_layer_kv_transfer_batched(
                [t for t, _, _ in items], self.kvcaches[layer_id][0], self.kvcaches[layer_id][1],
                slot_mapping, [s for _, s, _ in items], [e for _, _, e in items], direction,
                True)

    def batched_to_gpu(self, starts: List[int], ends: List[int], **kwargs):
        """Generator: MemoryObjs -> paged cache, one layer per ``send``.

        First ``next()`` prepares; each following ``send(memory_objs_layer)``
        waits for the previous layer's load (if ``sync``) and issues this
        layer's; two final iterations wait for the last layer. Yields
        num_layers + 2 times in total."""
        self.initialize_kvcaches_ptr(**kwargs)
        assert self.kvcaches is not None, (
            "kvcaches should be provided in kwargs or initialized beforehand.")
        if "slot_mapping" not in kwargs:
            raise ValueError("'slot_mapping' should be provided in kwargs.")
        if "sync" not in kwargs:
            raise ValueError("'sync' should be provided in kwargs.")
        slot_mapping: torch.Tensor = kwargs["slot_mapping"]
        sync: bool = kwargs["sync"]
        slot_mapping_full = torch.cat([slot_mapping[s:e] for s, e in zip(starts, ends)], dim=0)
        tmp = self._staging(len(slot_mapping_full)) if self.use_gpu else None
        if tmp is not None:
            tmp.record_stream(self.load_stream)
        offset = starts[0]
        current_stream = torch.cuda.current_stream()
        for layer_id in range(self.num_layers):
            memory_objs_layer = yield
            if sync:
                current_stream.wait_stream(self.load_stream)
            with torch.cuda.stream(self.load_stream):
                if self.use_gpu:
                    for start, end, memory_obj in zip(starts, ends, memory_objs_layer):
                        _check_format(memory_obj, KV_T2D)
                        tmp[start - offset : end - offset].copy_(memory_obj.tensor,
                                                                 non_blocking=True)
                else:
                    # every chunk of this layer in one launch (the reference
                    # issues one single_layer_kv_transfer per chunk)
                    self._layer_batched(memory_objs_layer, layer_id, slot_mapping, starts, ends,
                                        False)
                if self.use_gpu:
                    c_ops.single_layer_kv_transfer(
                        tmp, self.kvcaches[layer_id][0], self.kvcaches[layer_id][1],
                        slot_mapping_full, False, True)
        yield
        if sync:
            current_stream.wait_stream(self.load_stream)
        yield

    def batched_from_gpu(self, memory_objs: Union[List[List[MemoryObj]], List[MemoryObj]],
                         starts: List[int], ends: List[int], **kwargs):
        """Generator: paged cache -> MemoryObjs, one layer per iteration
        (memory_objs[layer][chunk]); yields num_layers + 1 times."""
        self.initialize_kvcaches_ptr(**kwargs)
        assert self.kvcaches is not None, (
            "kvcaches should be provided in kwargs or initialized beforehand.")
        if "slot_mapping" not in kwargs:
            raise ValueError("'slot_mapping' should be provided in kwargs.")
        if "sync" not in kwargs:
            raise ValueError("'sync' should be provided in kwargs.")
        slot_mapping: torch.Tensor = kwargs["slot_mapping"]
        sync: bool = kwargs["sync"]
        slot_mapping_full = torch.cat([slot_mapping[s:e] for s, e in zip(starts, ends)], dim=0)
        tmp = self._staging(len(slot_mapping_full)) if self.use_gpu else None
        if tmp is not None:
            tmp.record_stream(self.store_stream)
        offset = starts[0]
        current_stream = torch.cuda.current_stream()
        for layer_id in range(self.num_layers):
            memory_objs_layer: Sequence[MemoryObj] = memory_objs[layer_id]
            with torch.cuda.stream(self.store_stream):
                self.store_stream.wait_stream(current_stream)
                if self.use_gpu:
                    c_ops.single_layer_kv_transfer(
                        tmp, self.kvcaches[layer_id][0], self.kvcaches[layer_id][1],
                        slot_mapping_full, True, True)
                if self.use_gpu:
                    for start, end, memory_obj in zip(starts, ends, memory_objs_layer):
                        assert memory_obj.tensor is not None
                        _check_format(memory_obj, KV_T2D)
                        memory_obj.tensor.copy_(tmp[start - offset : end - offset],
                                                non_blocking=True)
                else:
                    self._layer_batched(memory_objs_layer, layer_id, slot_mapping, starts, ends,
                                        True)
            yield
            if sync:
                self.store_stream.synchronize()
        yield


class VLLMBufferLayerwiseGPUConnector(VLLMPagedMemLayerwiseGPUConnector):
    """The buffer layerwise connector (npu_connector.py:20-21 subclasses the
    upstream class without changes): the layerwise generators with every
    layer staged through one device buffer (``use_gpu`` on by default)."""

    def __init__(self, hidden_dim_size: int, num_layers: int, use_gpu: bool = True, **kwargs):
        super().__init__(hidden_dim_size, num_layers, use_gpu=use_gpu, **kwargs)
