// c_ops.cpp -- PyTorch/pybind11 surface of lmcache_b200.
//
// Exports the same eleven names, positional argument order and tensor layouts
// as the reference's c_ops module (csrc/pybind.cpp:13-26), so that
// `sys.modules["lmcache.c_ops"] = lmcache_b200.c_ops` is a drop-in. Every
// function validates its tensors, resolves device addresses (device tensors
// directly, pinned CPU tensors through the host registry, as
// get_kernel_ptr does at csrc/mem_kernels.cpp:11-26) and calls the C ABI of
// liblmcache_b200.so on the current CUDA stream. Nothing here computes on the
// CPU: a missing CUDA library makes the import fail.

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "lmcache_b200.h"

namespace py = pybind11;

namespace {

// torch dtype -> lmcb_dtype; same accepted set as csrc/utils.h:22-38.
int to_lmcb_dtype(at::ScalarType t) {
  switch (t) {
    case at::ScalarType::Float: return LMCB_DTYPE_FP32;
    case at::ScalarType::BFloat16: return LMCB_DTYPE_BF16;
    case at::ScalarType::Half: return LMCB_DTYPE_FP16;
    case at::ScalarType::Long: return LMCB_DTYPE_INT64;
    case at::ScalarType::Int: return LMCB_DTYPE_INT32;
    default: TORCH_CHECK(false, "ScalarType not supported.");
  }
  return -1;
}

int to_slot_dtype(at::ScalarType t) {
  TORCH_CHECK(t == at::ScalarType::Long || t == at::ScalarType::Int,
              "ScalarType not supported.");
  return to_lmcb_dtype(t);
}

// Device-usable address of a tensor's data (csrc/mem_kernels.cpp:11-26).
void* get_kernel_ptr(const torch::Tensor& tensor) {
  const torch::Device device = tensor.device();
  if (device.is_cuda()) {
    return tensor.data_ptr();
  } else if (device.is_cpu()) {
    void* dev = lmcb_host_get_device_ptr(tensor.data_ptr());
    TORCH_CHECK(dev != nullptr,
                "Unable to retrieve device ptr, is this a host registered pointer ?");
    return dev;
  }
  TORCH_CHECK(false, "Invalid device. Device must be cuda or pinned cpu.");
  return nullptr;
}

// CUDA tensors of one call must live on the device the kernel runs on: a
// pointer to another GPU's memory would be dereferenced as a peer access.
void check_device(const torch::Tensor& t, const torch::Device& dev, const char* name) {
  TORCH_CHECK(!t.is_cuda() || t.device() == dev, name, " is on ", t.device(),
              " but the paged KV cache is on ", dev);
}

torch::Device cuda_device_of(const torch::Device& d) {
  TORCH_CHECK(d.is_cuda(), "paged_memory_device must be a CUDA device, got ", d);
  return d.has_index() ? d : torch::Device(torch::kCUDA, c10::cuda::current_device());
}

void check_status(int status) {
  if (status == LMCB_OK) return;
  if (status == LMCB_ERR_NOT_IMPLEMENTED) {
    PyErr_SetString(PyExc_NotImplementedError, lmcb_last_error());
    throw py::error_already_set();
  }
  TORCH_CHECK(false, std::string(lmcb_status_string(status)) + ": " + lmcb_last_error());
}

cudaStream_t current_stream() {
  return at::cuda::getCurrentCUDAStream().stream();
}

// Byte stride between consecutive slots of a paged K or V cache laid out
// [num_blocks, block_size, ...row dims]; checks the row is dense and that
// slot * stride addresses every (block, offset) pair.
int64_t paged_row_stride(const torch::Tensor& cache, int64_t hidden, const char* name) {
  TORCH_CHECK(cache.dim() >= 3, name, " must be [num_blocks, block_size, ...]");
  int64_t row_elems = 1;
  for (int64_t d = 2; d < cache.dim(); ++d) row_elems *= cache.size(d);
  TORCH_CHECK(row_elems == hidden, name, " row has ", row_elems,
              " elements but the LMCache side has ", hidden);
  int64_t expect = 1;
  for (int64_t d = cache.dim() - 1; d >= 2; --d) {
    TORCH_CHECK(cache.size(d) == 1 || cache.stride(d) == expect, name,
                " rows must be contiguous");
    expect *= cache.size(d);
  }
  TORCH_CHECK(cache.size(0) == 1 || cache.stride(0) == cache.size(1) * cache.stride(1), name,
              " blocks must be evenly strided by block_size rows");
  return cache.stride(1) * cache.element_size();
}

enum class HostRetrievePath { kAuto, kZeroCopy, kDma };

HostRetrievePath host_path_from_env(const char* name) {
  const char* env = std::getenv(name);
  if (env == nullptr) return HostRetrievePath::kAuto;
  if (std::strcmp(env, "zerocopy") == 0) return HostRetrievePath::kZeroCopy;
  if (std::strcmp(env, "dma") == 0) return HostRetrievePath::kDma;
  return HostRetrievePath::kAuto;
}

HostRetrievePath host_retrieve_path() { return host_path_from_env("LMCB_HOST_RETRIEVE"); }
HostRetrievePath host_store_path() { return host_path_from_env("LMCB_HOST_STORE"); }

// Objects at least this large are retrieved from pinned host memory with one
// DMA into a device staging buffer plus an HBM scatter instead of zero-copy
// kernel reads. Measured on B200 (PCIe Gen5 x16), per retrieve of one object:
//   2 MiB: zero-copy 46.6 GB/s, DMA 39.5;   8 MiB: 50.1 vs 50.7;
//   32 MiB: 51.1 vs 53.6;                    64 MiB: 51.3 vs 54.0.
constexpr int64_t kDmaRetrieveMinBytes = int64_t(8) << 20;

// Same choice for stores into pinned host memory: gather into a device
// staging buffer (skipped rows read back from the object) and one DMA to the
// host, instead of zero-copy kernel writes.
constexpr int64_t kDmaStoreMinBytes = int64_t(8) << 20;

}  // namespace

// ---------------------------------------------------------------------------
// Host registration (csrc/managed_mem.cpp:296-315)
// ---------------------------------------------------------------------------

void* register_memory(torch::Tensor& tensor) {
  if (!tensor.device().is_cpu() || !tensor.is_pinned()) {
    TORCH_CHECK(false, "Invalid device. Device must be CPU and tensor must be pinned.");
  }
  void* dev = nullptr;
  check_status(lmcb_host_register(tensor.data_ptr(), tensor.nbytes(), &dev));
  return dev;
}

void unregister_memory(torch::Tensor& tensor) {
  check_status(lmcb_host_unregister(tensor.data_ptr()));
}

int64_t get_device_ptr(int64_t host_ptr) {
  return reinterpret_cast<int64_t>(lmcb_host_get_device_ptr(reinterpret_cast<void*>(host_ptr)));
}

// ---------------------------------------------------------------------------
// Transfers (csrc/mem_kernels.cpp)
// ---------------------------------------------------------------------------

void multi_layer_kv_transfer(torch::Tensor& key_value,             // [kv, L, T, H]
                             const torch::Tensor& key_value_ptrs,  // [L] int64
                             const torch::Tensor& slot_mapping,    // [T]
                             const torch::Device& paged_memory_device,
                             const int page_buffer_size, const bool direction,
                             const bool use_mla) {
  TORCH_CHECK(key_value.dim() >= 3, "key_value must be [kv, num_layers, num_tokens, hidden]");
  TORCH_CHECK(key_value.is_contiguous(), "key_value must be contiguous");
  TORCH_CHECK(key_value_ptrs.scalar_type() == at::ScalarType::Long,
              "key_value_ptrs must be int64");
  const int kv_size = use_mla ? 1 : 2;
  const int64_t num_layers = key_value.size(1);
  const int64_t num_tokens = slot_mapping.size(0);
  const int64_t hidden = key_value.size(-1);
  TORCH_CHECK(key_value_ptrs.numel() >= num_layers, "key_value_ptrs has fewer than ",
              num_layers, " entries");
  TORCH_CHECK(key_value.numel() >= kv_size * num_layers * num_tokens * hidden,
              "key_value is smaller than [", kv_size, ", ", num_layers, ", ", num_tokens,
              ", ", hidden, "]");
  const int dtype = to_lmcb_dtype(key_value.scalar_type());
  const int slot_dtype = to_slot_dtype(slot_mapping.scalar_type());

  const torch::Device dev = cuda_device_of(paged_memory_device);
  check_device(key_value, dev, "key_value");
  check_device(key_value_ptrs, dev, "key_value_ptrs");
  check_device(slot_mapping, dev, "slot_mapping");
  const c10::OptionalDeviceGuard device_guard(dev);
  cudaStream_t stream = current_stream();

  const uint64_t* ptrs = static_cast<const uint64_t*>(get_kernel_ptr(key_value_ptrs));
  const void* slots = get_kernel_ptr(slot_mapping);

  if (key_value.device().is_cpu() && !direction) {
    const int64_t bytes = kv_size * num_layers * num_tokens * hidden * key_value.element_size();
    const HostRetrievePath path = host_retrieve_path();
    const bool use_dma = path == HostRetrievePath::kDma ||
                         (path == HostRetrievePath::kAuto && bytes >= kDmaRetrieveMinBytes);
    if (use_dma && bytes > 0) {
      // Registered but not necessarily CUDA-pinned memory is still a valid
      // DMA source: the registry pinned it.
      void* host = key_value.data_ptr();
      TORCH_CHECK(lmcb_host_get_device_ptr(host) != nullptr,
                  "Unable to retrieve device ptr, is this a host registered pointer ?");
      auto staging = torch::empty(
          {bytes}, torch::TensorOptions().dtype(torch::kUInt8).device(
                       torch::kCUDA, c10::cuda::current_device()));
      check_status(lmcb_multi_layer_kv_retrieve_staged(
          dtype, slot_dtype, stream, ptrs, host, staging.data_ptr(),
          static_cast<size_t>(bytes), slots, hidden, kv_size,
          static_cast<int32_t>(num_layers), page_buffer_size,
          static_cast<int32_t>(num_tokens)));
      return;
    }
  }
  if (key_value.device().is_cpu() && direction) {
    const int64_t bytes = kv_size * num_layers * num_tokens * hidden * key_value.element_size();
    const HostRetrievePath path = host_store_path();
    const bool use_dma = path == HostRetrievePath::kDma ||
                         (path == HostRetrievePath::kAuto && bytes >= kDmaStoreMinBytes);
    if (use_dma && bytes > 0) {
      void* host_dev = get_kernel_ptr(key_value);  // registered: device alias
      auto staging = torch::empty(
          {bytes}, torch::TensorOptions().dtype(torch::kUInt8).device(
                       torch::kCUDA, c10::cuda::current_device()));
      check_status(lmcb_multi_layer_kv_store_staged(
          dtype, slot_dtype, stream, ptrs, key_value.data_ptr(), host_dev, staging.data_ptr(),
          static_cast<size_t>(bytes), slots, hidden, kv_size, static_cast<int32_t>(num_layers),
          page_buffer_size, static_cast<int32_t>(num_tokens)));
      return;
    }
  }
  void* lmc = get_kernel_ptr(key_value);
  check_status(lmcb_multi_layer_kv_transfer_kernel(
      dtype, slot_dtype, stream, ptrs, lmc, slots, hidden, kv_size,
      static_cast<int32_t>(num_layers), page_buffer_size, static_cast<int32_t>(num_tokens),
      direction ? 1 : 0));
}

// All chunks of a request in one launch (an addition to the reference
// surface; the connector's batched_from_gpu / batched_to_gpu call it).
// key_values[i] is a [kv, L, T_i, H] object holding slot_mapping[starts[i]:
// ends[i]]. The objects are all CUDA tensors on one device, or all pinned
// host tensors registered with host_register. Retrieval from host objects
// of at least kDmaRetrieveMinBytes in total copies each object into one
// device staging buffer (one cudaMemcpyAsync per object) and scatters from
// there.
void multi_layer_kv_transfer_batched(const std::vector<torch::Tensor>& key_values,
                                     const torch::Tensor& key_value_ptrs,
                                     const torch::Tensor& slot_mapping,
                                     const std::vector<int64_t>& starts,
                                     const std::vector<int64_t>& ends,
                                     const torch::Device& paged_memory_device,
                                     const int64_t page_buffer_size, const bool direction,
                                     const bool use_mla) {
  const int64_t n = static_cast<int64_t>(key_values.size());
  TORCH_CHECK(static_cast<int64_t>(starts.size()) == n && static_cast<int64_t>(ends.size()) == n,
              "starts and ends must have one entry per object");
  if (n == 0) return;
  TORCH_CHECK(key_value_ptrs.scalar_type() == at::ScalarType::Long,
              "key_value_ptrs must be int64");
  const int kv_size = use_mla ? 1 : 2;
  const auto& first = key_values[0];
  TORCH_CHECK(first.dim() >= 3, "key_values must be [kv, num_layers, num_tokens, hidden]");
  const int64_t num_layers = first.size(1);
  const int64_t hidden = first.size(-1);
  const bool on_device = first.is_cuda();
  TORCH_CHECK(key_value_ptrs.numel() >= num_layers, "key_value_ptrs has fewer than ",
              num_layers, " entries");
  const int dtype = to_lmcb_dtype(first.scalar_type());
  const int slot_dtype = to_slot_dtype(slot_mapping.scalar_type());
  int64_t total = 0;
  for (int64_t i = 0; i < n; ++i) {
    const auto& t = key_values[i];
    TORCH_CHECK(t.scalar_type() == first.scalar_type() && t.size(1) == num_layers &&
                    t.size(-1) == hidden && t.is_cuda() == on_device,
                "key_values must share dtype, layer count, hidden size and residency");
    TORCH_CHECK(t.is_contiguous(), "key_values must be contiguous");
    TORCH_CHECK(0 <= starts[i] && starts[i] <= ends[i] && ends[i] <= slot_mapping.size(0),
                "object ", i, ": slot range out of bounds");
    TORCH_CHECK(t.numel() >= kv_size * num_layers * (ends[i] - starts[i]) * hidden, "object ",
                i, " is smaller than its slot range");
    total += ends[i] - starts[i];
  }
  if (total == 0) return;
  TORCH_CHECK(total < (int64_t(1) << 31), "too many tokens in one batch");

  const torch::Device dev = cuda_device_of(paged_memory_device);
  check_device(key_value_ptrs, dev, "key_value_ptrs");
  check_device(slot_mapping, dev, "slot_mapping");
  for (const auto& t : key_values) check_device(t, dev, "key_values");
  const c10::OptionalDeviceGuard device_guard(dev);
  cudaStream_t stream = current_stream();
  const uint64_t* ptrs = static_cast<const uint64_t*>(get_kernel_ptr(key_value_ptrs));
  const void* slots = get_kernel_ptr(slot_mapping);
  const int64_t esz = first.element_size();

  bool staged = false;
  torch::Tensor staging;
  if (!on_device && !direction) {
    const int64_t bytes = kv_size * num_layers * total * hidden * esz;
    const HostRetrievePath path = host_retrieve_path();
    staged = path == HostRetrievePath::kDma ||
             (path == HostRetrievePath::kAuto && bytes >= kDmaRetrieveMinBytes);
    if (staged) {
      // Each object starts on a 256-byte boundary of the staging buffer.
      int64_t staging_bytes = 0;
      for (int64_t i = 0; i < n; ++i) {
        const int64_t obj_bytes = kv_size * num_layers * (ends[i] - starts[i]) * hidden * esz;
        staging_bytes += (obj_bytes + 255) / 256 * 256;
      }
      staging = torch::empty({staging_bytes},
                             torch::TensorOptions().dtype(torch::kUInt8).device(dev));
    }
  }

  // Object table (host arrays; the library passes it in the kernel parameters).
  std::vector<uint64_t> obj_ptrs(n);
  std::vector<int64_t> offsets(n + 1), slot_starts(n);
  int64_t off = 0, staged_off = 0;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t count = ends[i] - starts[i];
    const int64_t obj_bytes = kv_size * num_layers * count * hidden * esz;
    void* obj = nullptr;  // empty objects hold no token; their address is never used
    if (count == 0) {
    } else if (staged) {
      obj = static_cast<uint8_t*>(staging.data_ptr()) + staged_off;
      if (obj_bytes > 0) {
        auto dst = staging.narrow(0, staged_off, obj_bytes);
        dst.copy_(key_values[i].view(torch::kUInt8).reshape({-1}).narrow(0, 0, obj_bytes),
                  /*non_blocking=*/true);
      }
      staged_off += (obj_bytes + 255) / 256 * 256;
    } else {
      obj = get_kernel_ptr(key_values[i]);
    }
    obj_ptrs[i] = reinterpret_cast<uint64_t>(obj);
    offsets[i] = off;
    slot_starts[i] = starts[i];
    off += count;
  }
  offsets[n] = off;
  check_status(lmcb_multi_layer_kv_transfer_batched_kernel(
      dtype, slot_dtype, stream, ptrs, obj_ptrs.data(), offsets.data(), slot_starts.data(),
      static_cast<int32_t>(n), (on_device || staged) ? 1 : 0, slots, hidden,
      kv_size, static_cast<int32_t>(num_layers), page_buffer_size, static_cast<int32_t>(total),
      direction ? 1 : 0));
}

// single_layer_kv_transfer for every chunk of a layer in one launch (an
// addition to the reference surface, used by the layerwise connector).
// lmc_kvs[i] is [T_i, 2, H] (token_major) or [2, T_i, H] and holds
// slot_mapping[starts[i]:ends[i]]; all CUDA tensors on the caches' device, or
// all registered pinned host tensors (zero-copy).
void single_layer_kv_transfer_batched(const std::vector<torch::Tensor>& lmc_kvs,
                                      torch::Tensor& vllm_key_cache,
                                      torch::Tensor& vllm_value_cache,
                                      torch::Tensor& slot_mapping,
                                      const std::vector<int64_t>& starts,
                                      const std::vector<int64_t>& ends, const bool direction,
                                      const bool token_major) {
  const int64_t n = static_cast<int64_t>(lmc_kvs.size());
  TORCH_CHECK(static_cast<int64_t>(starts.size()) == n && static_cast<int64_t>(ends.size()) == n,
              "starts and ends must have one entry per object");
  if (n == 0) return;
  TORCH_CHECK(vllm_key_cache.is_cuda(), "vllm_key_cache must be a CUDA tensor");
  const torch::Device dev = vllm_key_cache.device();
  check_device(vllm_value_cache, dev, "vllm_value_cache");
  check_device(slot_mapping, dev, "slot_mapping");
  const int64_t hidden = lmc_kvs[0].size(-1);
  const bool on_device = lmc_kvs[0].is_cuda();
  TORCH_CHECK(vllm_key_cache.scalar_type() == lmc_kvs[0].scalar_type() &&
                  vllm_value_cache.scalar_type() == lmc_kvs[0].scalar_type(),
              "K/V caches and the objects must have the same dtype");
  const int64_t k_stride = paged_row_stride(vllm_key_cache, hidden, "vllm_key_cache");
  const int64_t v_stride = paged_row_stride(vllm_value_cache, hidden, "vllm_value_cache");
  TORCH_CHECK(k_stride == v_stride, "K and V caches must have the same row stride");
  const int64_t rows = std::min(vllm_key_cache.size(0) * vllm_key_cache.size(1),
                                vllm_value_cache.size(0) * vllm_value_cache.size(1));
  int64_t total = 0;
  for (int64_t i = 0; i < n; ++i) {
    const auto& t = lmc_kvs[i];
    check_device(t, dev, "lmc_kvs");
    TORCH_CHECK(t.scalar_type() == lmc_kvs[0].scalar_type() && t.size(-1) == hidden &&
                    t.is_cuda() == on_device && t.is_contiguous(),
                "objects must share dtype, hidden size and residency, and be contiguous");
    TORCH_CHECK(0 <= starts[i] && starts[i] <= ends[i] && ends[i] <= slot_mapping.size(0),
                "object ", i, ": slot range out of bounds");
    TORCH_CHECK(t.numel() >= 2 * (ends[i] - starts[i]) * hidden, "object ", i,
                " is smaller than its slot range");
    total += ends[i] - starts[i];
  }
  if (total == 0) return;
  TORCH_CHECK(total < (int64_t(1) << 31), "too many tokens in one batch");
  const int dtype = to_lmcb_dtype(vllm_key_cache.scalar_type());
  const int slot_dtype = to_slot_dtype(slot_mapping.scalar_type());
  const c10::OptionalDeviceGuard device_guard(dev);
  cudaStream_t stream = current_stream();
  std::vector<uint64_t> obj_ptrs(n);
  std::vector<int64_t> offsets(n + 1), slot_starts(n);
  int64_t off = 0;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t count = ends[i] - starts[i];
    obj_ptrs[i] = count == 0 ? 0 : reinterpret_cast<uint64_t>(get_kernel_ptr(lmc_kvs[i]));
    offsets[i] = off;
    slot_starts[i] = starts[i];
    off += count;
  }
  offsets[n] = off;
  check_status(lmcb_single_layer_kv_transfer_batched_kernel(
      dtype, slot_dtype, stream, obj_ptrs.data(), offsets.data(), slot_starts.data(),
      static_cast<int32_t>(n), on_device ? 1 : 0, get_kernel_ptr(vllm_key_cache),
      get_kernel_ptr(vllm_value_cache), get_kernel_ptr(slot_mapping), hidden,
      static_cast<int32_t>(total), direction ? 1 : 0, token_major ? 1 : 0, k_stride, rows));
}

void multi_layer_kv_transfer_unilateral(torch::Tensor& key_value,
                                        const torch::Tensor& key_ptrs,
                                        const torch::Tensor& value_ptrs,
                                        const torch::Tensor& slot_mapping,
                                        const torch::Device& paged_memory_device,
                                        const int page_buffer_size,
                                        const bool direction) {
  TORCH_CHECK(key_value.dim() >= 3, "key_value must be [2, num_layers, num_tokens, hidden]");
  TORCH_CHECK(key_value.is_contiguous(), "key_value must be contiguous");
  TORCH_CHECK(key_ptrs.scalar_type() == at::ScalarType::Long &&
                  value_ptrs.scalar_type() == at::ScalarType::Long,
              "key_ptrs and value_ptrs must be int64");
  const int64_t num_layers = key_value.size(1);
  const int64_t num_tokens = slot_mapping.size(0);
  const int64_t hidden = key_value.size(-1);
  TORCH_CHECK(key_ptrs.numel() >= num_layers && value_ptrs.numel() >= num_layers,
              "pointer arrays have fewer than ", num_layers, " entries");
  TORCH_CHECK(key_value.numel() >= 2 * num_layers * num_tokens * hidden,
              "key_value is smaller than [2, ", num_layers, ", ", num_tokens, ", ", hidden, "]");
  const int dtype = to_lmcb_dtype(key_value.scalar_type());
  const int slot_dtype = to_slot_dtype(slot_mapping.scalar_type());
  const torch::Device dev = cuda_device_of(paged_memory_device);
  check_device(key_value, dev, "key_value");
  check_device(key_ptrs, dev, "key_ptrs");
  check_device(value_ptrs, dev, "value_ptrs");
  check_device(slot_mapping, dev, "slot_mapping");
  const c10::OptionalDeviceGuard device_guard(dev);
  cudaStream_t stream = current_stream();
  check_status(lmcb_multi_layer_kv_transfer_unilateral_kernel(
      dtype, slot_dtype, stream, static_cast<const uint64_t*>(get_kernel_ptr(key_ptrs)),
      static_cast<const uint64_t*>(get_kernel_ptr(value_ptrs)), get_kernel_ptr(key_value),
      get_kernel_ptr(slot_mapping), hidden, static_cast<int32_t>(num_layers),
      page_buffer_size, static_cast<int32_t>(num_tokens), direction ? 1 : 0));
}

void single_layer_kv_transfer(torch::Tensor& lmc_key_value_cache,  // [T,2,H] or [2,T,H]
                              torch::Tensor& vllm_key_cache,       // [nb, bs, heads, hd]
                              torch::Tensor& vllm_value_cache,
                              torch::Tensor& slot_mapping,  // [T]
                              const bool direction, const bool token_major) {
  TORCH_CHECK(lmc_key_value_cache.is_contiguous(), "lmc_key_value_cache must be contiguous");
  const int64_t num_tokens = slot_mapping.size(0);
  const int64_t hidden = lmc_key_value_cache.size(-1);
  TORCH_CHECK(lmc_key_value_cache.numel() >= 2 * num_tokens * hidden,
              "lmc_key_value_cache is smaller than 2 x ", num_tokens, " x ", hidden);
  TORCH_CHECK(vllm_key_cache.scalar_type() == lmc_key_value_cache.scalar_type() &&
                  vllm_value_cache.scalar_type() == lmc_key_value_cache.scalar_type(),
              "K/V caches and lmc_key_value_cache must have the same dtype");
  const int64_t k_stride = paged_row_stride(vllm_key_cache, hidden, "vllm_key_cache");
  const int64_t v_stride = paged_row_stride(vllm_value_cache, hidden, "vllm_value_cache");
  TORCH_CHECK(k_stride == v_stride, "K and V caches must have the same row stride");
  const int64_t rows = std::min(vllm_key_cache.size(0) * vllm_key_cache.size(1),
                                vllm_value_cache.size(0) * vllm_value_cache.size(1));
  const int dtype = to_lmcb_dtype(vllm_key_cache.scalar_type());
  const int slot_dtype = to_slot_dtype(slot_mapping.scalar_type());

  TORCH_CHECK(vllm_key_cache.is_cuda(), "vllm_key_cache must be a CUDA tensor");
  const torch::Device dev = vllm_key_cache.device();
  check_device(vllm_value_cache, dev, "vllm_value_cache");
  check_device(lmc_key_value_cache, dev, "lmc_key_value_cache");
  check_device(slot_mapping, dev, "slot_mapping");
  const c10::OptionalDeviceGuard device_guard(dev);
  cudaStream_t stream = current_stream();
  check_status(lmcb_single_layer_kv_transfer_kernel(
      dtype, slot_dtype, stream, get_kernel_ptr(lmc_key_value_cache),
      get_kernel_ptr(vllm_key_cache), get_kernel_ptr(vllm_value_cache),
      get_kernel_ptr(slot_mapping), hidden, static_cast<int32_t>(num_tokens),
      direction ? 1 : 0, token_major ? 1 : 0, /*isMLA=*/0, k_stride, rows));
}

namespace {

void flash_transfer(torch::Tensor& key_value, torch::Tensor& key_cache,
                    torch::Tensor& value_cache, torch::Tensor& slot_mapping,
                    const int layer_idx, bool page2L) {
  TORCH_CHECK(key_value.dim() >= 3, "key_value must be [2, num_layers, num_tokens, hidden]");
  TORCH_CHECK(key_value.is_contiguous(), "key_value must be contiguous");
  const int64_t num_tokens = slot_mapping.size(0);
  const int64_t num_layers = key_value.size(1);
  const int64_t hidden = key_value.size(-1);
  TORCH_CHECK(key_value.numel() >= 2 * num_layers * num_tokens * hidden,
              "key_value is smaller than [2, ", num_layers, ", ", num_tokens, ", ", hidden, "]");
  TORCH_CHECK(key_cache.scalar_type() == key_value.scalar_type() &&
                  value_cache.scalar_type() == key_value.scalar_type(),
              "K/V caches and key_value must have the same dtype");
  const int64_t k_stride = paged_row_stride(key_cache, hidden, "key_cache");
  const int64_t v_stride = paged_row_stride(value_cache, hidden, "value_cache");
  TORCH_CHECK(k_stride == v_stride, "K and V caches must have the same row stride");
  TORCH_CHECK(key_cache.size(0) == value_cache.size(0) &&
                  key_cache.size(1) == value_cache.size(1),
              "K and V caches must have the same number of blocks and block size");
  const int dtype = to_lmcb_dtype(key_value.scalar_type());
  const int slot_dtype = to_slot_dtype(slot_mapping.scalar_type());
  TORCH_CHECK(key_cache.is_cuda(), "key_cache must be a CUDA tensor");
  const torch::Device dev = key_cache.device();
  check_device(value_cache, dev, "value_cache");
  check_device(key_value, dev, "key_value");
  check_device(slot_mapping, dev, "slot_mapping");
  const c10::OptionalDeviceGuard device_guard(dev);
  cudaStream_t stream = current_stream();
  check_status(lmcb_load_and_reshape_flash_kernel(
      dtype, slot_dtype, stream, get_kernel_ptr(key_value), get_kernel_ptr(key_cache),
      get_kernel_ptr(value_cache), get_kernel_ptr(slot_mapping), hidden, key_cache.size(0),
      static_cast<int32_t>(key_cache.size(1)), static_cast<int32_t>(num_tokens),
      static_cast<int32_t>(num_layers), layer_idx, page2L ? 1 : 0, k_stride));
}

}  // namespace

void load_and_reshape_flash(torch::Tensor& key_value, torch::Tensor& key_cache,
                            torch::Tensor& value_cache, torch::Tensor& slot_mapping,
                            const int layer_idx) {
  flash_transfer(key_value, key_cache, value_cache, slot_mapping, layer_idx, true);
}

void reshape_and_cache_back_flash(torch::Tensor& key_value, torch::Tensor& key_cache,
                                  torch::Tensor& value_cache, torch::Tensor& slot_mapping,
                                  const int layer_idx) {
  flash_transfer(key_value, key_cache, value_cache, slot_mapping, layer_idx, false);
}

// ---------------------------------------------------------------------------
// CacheGen (csrc/cachegen_kernels.h:7-16)
// ---------------------------------------------------------------------------

namespace {

void check_symbols(const at::Tensor& sym, const char* name) {
  TORCH_CHECK(sym.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(sym.dim() == 3, name, " must be [num_layers, num_tokens, num_channels]");
  TORCH_CHECK(sym.scalar_type() == at::kChar || sym.scalar_type() == at::kByte, name,
              " must be int8 or uint8");
  TORCH_CHECK(sym.is_contiguous(), name, " must be contiguous");
}

void check_cdf(const at::Tensor& cdf, int64_t layers, int64_t channels) {
  TORCH_CHECK(cdf.is_cuda(), "cdf must be a CUDA tensor");
  TORCH_CHECK(cdf.scalar_type() == at::kShort, "cdf must be int16");
  TORCH_CHECK(cdf.dim() == 3 && cdf.size(0) == layers && cdf.size(1) == channels,
              "cdf must be [num_layers, num_channels, max_bins + 1]");
  TORCH_CHECK(cdf.is_contiguous(), "cdf must be contiguous");
}

}  // namespace

at::Tensor calculate_cdf(const at::Tensor& input, const int max_bins) {
  check_symbols(input, "input");
  const c10::cuda::CUDAGuard guard(input.device());
  auto cdf = torch::empty({input.size(0), input.size(2), max_bins + 1},
                          input.options().dtype(torch::kShort));
  check_status(lmcb_calculate_cdf(
      static_cast<const int8_t*>(input.data_ptr()), static_cast<int16_t*>(cdf.data_ptr()),
      static_cast<int32_t>(input.size(0)), static_cast<int32_t>(input.size(1)),
      static_cast<int32_t>(input.size(2)), max_bins, current_stream()));
  return cdf;
}

void encode_cuda_new(const at::Tensor& cdf, const at::Tensor& input_sym,
                     at::Tensor& output_buffer, at::Tensor& output_lengths) {
  check_symbols(input_sym, "input_sym");
  const int64_t L = input_sym.size(0), T = input_sym.size(1), C = input_sym.size(2);
  check_cdf(cdf, L, C);
  TORCH_CHECK(output_buffer.is_cuda() && output_buffer.is_contiguous() &&
                  output_buffer.dim() == 3 && output_buffer.size(0) == L &&
                  output_buffer.size(1) == C && output_buffer.element_size() == 1,
              "output_buffer must be a contiguous uint8 [num_layers, num_channels, capacity]");
  TORCH_CHECK(output_lengths.is_cuda() && output_lengths.is_contiguous() &&
                  output_lengths.scalar_type() == at::kInt && output_lengths.numel() == L * C,
              "output_lengths must be a contiguous int32 [num_layers, num_channels]");
  const c10::cuda::CUDAGuard guard(input_sym.device());
  check_status(lmcb_encode(static_cast<const int16_t*>(cdf.data_ptr()),
                           static_cast<const int8_t*>(input_sym.data_ptr()),
                           static_cast<uint8_t*>(output_buffer.data_ptr()),
                           static_cast<int32_t*>(output_lengths.data_ptr()),
                           static_cast<int32_t>(L), static_cast<int32_t>(T),
                           static_cast<int32_t>(C), static_cast<int32_t>(cdf.size(2) - 1),
                           output_buffer.size(2), current_stream()));
}

void decode_cuda_new(const at::Tensor& cdf, const at::Tensor& bytestreams,
                     const at::Tensor& lengths, at::Tensor& output) {
  check_symbols(output, "output");
  const int64_t L = output.size(0), T = output.size(1), C = output.size(2);
  check_cdf(cdf, L, C);
  TORCH_CHECK(bytestreams.is_cuda() && bytestreams.is_contiguous() &&
                  bytestreams.element_size() == 1 && bytestreams.dim() == 3 &&
                  bytestreams.size(0) == L && bytestreams.size(1) == C,
              "bytestreams must be a contiguous uint8 [num_layers, num_channels, capacity]");
  TORCH_CHECK(lengths.is_cuda() && lengths.is_contiguous() &&
                  lengths.scalar_type() == at::kInt && lengths.numel() == L * C,
              "lengths must be a contiguous int32 [num_layers, num_channels]");
  const c10::cuda::CUDAGuard guard(output.device());
  check_status(lmcb_decode(static_cast<const int16_t*>(cdf.data_ptr()),
                           static_cast<const uint8_t*>(bytestreams.data_ptr()),
                           static_cast<const int32_t*>(lengths.data_ptr()),
                           static_cast<int8_t*>(output.data_ptr()), static_cast<int32_t>(L),
                           static_cast<int32_t>(T), static_cast<int32_t>(C),
                           static_cast<int32_t>(cdf.size(2) - 1), bytestreams.size(2),
                           current_stream()));
}

void decode_cuda_prefsum(const at::Tensor& cdf, const at::Tensor& bytestreams,
                         const at::Tensor& lengths, at::Tensor& output) {
  check_symbols(output, "output");
  const int64_t L = output.size(0), T = output.size(1), C = output.size(2);
  check_cdf(cdf, L, C);
  TORCH_CHECK(bytestreams.is_cuda() && bytestreams.is_contiguous() &&
                  bytestreams.element_size() == 1,
              "bytestreams must be a contiguous uint8 CUDA tensor");
  TORCH_CHECK(lengths.is_cuda() && lengths.is_contiguous() &&
                  lengths.scalar_type() == at::kLong && lengths.numel() == L * C,
              "lengths must be contiguous int64 prefix sums [num_layers * num_channels]");
  const c10::cuda::CUDAGuard guard(output.device());
  check_status(lmcb_decode_prefsum(static_cast<const int16_t*>(cdf.data_ptr()),
                                   static_cast<const uint8_t*>(bytestreams.data_ptr()),
                                   bytestreams.numel(),
                                   static_cast<const int64_t*>(lengths.data_ptr()),
                                   static_cast<int8_t*>(output.data_ptr()),
                                   static_cast<int32_t>(L), static_cast<int32_t>(T),
                                   static_cast<int32_t>(C),
                                   static_cast<int32_t>(cdf.size(2) - 1), current_stream()));
}

// ---------------------------------------------------------------------------
// Fused rotary (csrc/pos_kernels.h:7-10; unimplemented in the reference)
// ---------------------------------------------------------------------------

void rotary_embedding_k_fused(const torch::Tensor& old_positions,
                              const torch::Tensor& new_positions, torch::Tensor& key,
                              int64_t head_size, const torch::Tensor& cos_sin_cache,
                              bool is_neox) {
  TORCH_CHECK(key.is_cuda() && old_positions.is_cuda() && new_positions.is_cuda() &&
                  cos_sin_cache.is_cuda(),
              "rotary_embedding_k_fused: all tensors must be CUDA tensors");
  TORCH_CHECK(key.dim() >= 2, "key must be [num_tokens, num_heads * head_size] or "
                              "[num_tokens, num_heads, head_size]");
  const int64_t num_tokens = key.size(0);
  TORCH_CHECK(old_positions.numel() == num_tokens && new_positions.numel() == num_tokens,
              "positions must have one entry per token");
  TORCH_CHECK(old_positions.scalar_type() == new_positions.scalar_type(),
              "old and new positions must have the same dtype");
  TORCH_CHECK(old_positions.is_contiguous() && new_positions.is_contiguous(),
              "positions must be contiguous");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous(),
              "cos_sin_cache must be a contiguous [max_position, rot_dim] tensor");
  // Everything after the token dimension must be dense.
  int64_t row = 1;
  for (int64_t d = key.dim() - 1; d >= 1; --d) {
    TORCH_CHECK(key.size(d) == 1 || key.stride(d) == row, "key rows must be contiguous");
    row *= key.size(d);
  }
  TORCH_CHECK(head_size > 0 && row % head_size == 0,
              "head_size does not divide the key row");
  const int pos_type = to_slot_dtype(old_positions.scalar_type());
  const c10::cuda::CUDAGuard guard(key.device());
  check_status(lmcb_rotary_embedding_k_fused(
      old_positions.data_ptr(), new_positions.data_ptr(), pos_type, key.data_ptr(),
      to_lmcb_dtype(key.scalar_type()), num_tokens, row / head_size, head_size,
      num_tokens > 1 ? key.stride(0) : row, cos_sin_cache.data_ptr(),
      to_lmcb_dtype(cos_sin_cache.scalar_type()), cos_sin_cache.size(1),
      cos_sin_cache.size(0), is_neox ? 1 : 0, current_stream()));
}

uint32_t device_status(int device) {
  uint32_t flags = 0;
  check_status(lmcb_device_status(device, &flags));
  return flags;
}

PYBIND11_MODULE(c_ops, m) {
  m.def("host_register", &register_memory);
  m.def("multi_layer_kv_transfer", &multi_layer_kv_transfer);
  m.def("single_layer_kv_transfer", &single_layer_kv_transfer);
  m.def("multi_layer_kv_transfer_unilateral", &multi_layer_kv_transfer_unilateral);
  m.def("load_and_reshape_flash", &load_and_reshape_flash);
  m.def("reshape_and_cache_back_flash", &reshape_and_cache_back_flash);
  m.def("encode_fast_new", &encode_cuda_new);
  m.def("decode_fast_new", &decode_cuda_new);
  m.def("decode_fast_prefsum", &decode_cuda_prefsum);
  m.def("calculate_cdf", &calculate_cdf);
  m.def("rotary_embedding_k_fused", &rotary_embedding_k_fused);
  // Additions beyond the reference surface.
  m.def("multi_layer_kv_transfer_batched", &multi_layer_kv_transfer_batched);
  m.def("single_layer_kv_transfer_batched", &single_layer_kv_transfer_batched);
  m.def("host_unregister", &unregister_memory);
  m.def("get_device_ptr", &get_device_ptr);
  m.def("device_status", &device_status);
}
