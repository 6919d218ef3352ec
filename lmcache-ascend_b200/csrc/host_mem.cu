// host_mem.cu -- registry of host memory ranges that kernels may address.
//
// B200 counterpart of the reference's HostRegisteredMemoryManager
// (csrc/managed_mem.h:19-56, csrc/managed_mem.cpp:37-174). A registered range
// maps host addresses to device-usable aliases so a kernel can read or write a
// pinned-host LMCache object directly over PCIe (zero-copy).
//
// On CUDA, memory that is already pinned by the CUDA runtime (for example a
// torch tensor created with pin_memory=True) is device-mapped under unified
// addressing; registering it only records the range and its device alias
// (cudaHostGetDevicePointer). Pageable memory is page-locked and mapped with
// cudaHostRegister and unpinned again on unregister. There is no
// driver-version split as on Ascend (managed_mem.cpp:298-315): one path
// serves all supported drivers.
//
// The map is ordered by start address, so lookups are O(log n) instead of the
// reference's linear scan (managed_mem.cpp:142-152); it is guarded by a
// shared mutex (exclusive for register / unregister, shared for lookups), as
// in the reference.

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <shared_mutex>
#include <string>

#include "common.cuh"
#include "lmcache_b200.h"

namespace lmcb {
namespace {

struct Record {
  uintptr_t host;
  uintptr_t dev;
  size_t bytes;
  bool owned;  // pinned by this library (cudaHostRegister), unpin on removal
};

class HostRegistry {
 public:
  static HostRegistry& instance() {
    // Never destroyed: CUDA calls from static destructors at process exit may
    // run after the runtime has shut down; the OS releases pinned pages.
    static HostRegistry* inst = new HostRegistry();
    return *inst;
  }

  int add(void* host, size_t bytes, void** dev_out) {
    std::unique_lock<std::shared_mutex> guard(mu_);
    const uintptr_t h = reinterpret_cast<uintptr_t>(host);
    auto it = map_.find(h);
    if (it != map_.end()) {
      *dev_out = reinterpret_cast<void*>(it->second.dev);
      return LMCB_OK;
    }
    cudaPointerAttributes attr{};
    cudaError_t err = cudaPointerGetAttributes(&attr, host);
    if (err != cudaSuccess) {
      cudaGetLastError();
      return cuda_fail(err, "cudaPointerGetAttributes");
    }
    bool owned = false;
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
      return fail(LMCB_ERR_INVALID_ARGUMENT,
                  "host_register: pointer is device memory, not host memory.");
    }
    if (attr.type != cudaMemoryTypeHost) {
      err = cudaHostRegister(host, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
      if (err != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(err, "cudaHostRegister");
      }
      owned = true;
    }
    void* dev = nullptr;
    err = cudaHostGetDevicePointer(&dev, host, 0);
    if (err != cudaSuccess) {
      cudaGetLastError();
      if (owned) cudaHostUnregister(host);
      return cuda_fail(err, "cudaHostGetDevicePointer");
    }
    map_.emplace(h, Record{h, reinterpret_cast<uintptr_t>(dev), bytes, owned});
    *dev_out = dev;
    return LMCB_OK;
  }

  int remove(void* host) {
    std::unique_lock<std::shared_mutex> guard(mu_);
    auto it = map_.find(reinterpret_cast<uintptr_t>(host));
    if (it == map_.end()) return LMCB_OK;
    if (it->second.owned) cudaHostUnregister(host);
    map_.erase(it);
    return LMCB_OK;
  }

  int remove_all() {
    std::unique_lock<std::shared_mutex> guard(mu_);
    for (auto& kv : map_) {
      if (kv.second.owned) cudaHostUnregister(reinterpret_cast<void*>(kv.second.host));
    }
    map_.clear();
    return LMCB_OK;
  }

  // Record containing `host`, or nullptr.
  const Record* find(uintptr_t h) const {
    auto it = map_.upper_bound(h);
    if (it == map_.begin()) return nullptr;
    --it;
    const Record& r = it->second;
    if (h >= r.host && h < r.host + r.bytes) return &r;
    return nullptr;
  }

  void* device_ptr(void* host) const {
    if (host == nullptr) return nullptr;
    std::shared_lock<std::shared_mutex> guard(mu_);
    const uintptr_t h = reinterpret_cast<uintptr_t>(host);
    const Record* r = find(h);
    return r ? reinterpret_cast<void*>(r->dev + (h - r->host)) : nullptr;
  }

  size_t record_size(void* host) const {
    if (host == nullptr) return 0;
    std::shared_lock<std::shared_mutex> guard(mu_);
    const Record* r = find(reinterpret_cast<uintptr_t>(host));
    return r ? r->bytes : 0;
  }

 private:
  HostRegistry() = default;
  mutable std::shared_mutex mu_;
  std::map<uintptr_t, Record> map_;
};

}  // namespace
}  // namespace lmcb

extern "C" {

int lmcb_host_register(void* hostPtr, size_t bytes, void** devPtrOut) {
  lmcb::clear_error();
  if (hostPtr == nullptr || bytes == 0 || devPtrOut == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      "Error: hostPtr cannot be null and bufferSize must be greater than 0.");
  }
  return lmcb::HostRegistry::instance().add(hostPtr, bytes, devPtrOut);
}

int lmcb_host_unregister(void* hostPtr) {
  lmcb::clear_error();
  if (hostPtr == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "Error: hostPtr cannot be null.");
  }
  return lmcb::HostRegistry::instance().remove(hostPtr);
}

void* lmcb_host_get_device_ptr(void* hostPtr) {
  return lmcb::HostRegistry::instance().device_ptr(hostPtr);
}

size_t lmcb_host_record_size(void* hostPtr) {
  return lmcb::HostRegistry::instance().record_size(hostPtr);
}

int lmcb_host_unregister_all(void) {
  lmcb::clear_error();
  return lmcb::HostRegistry::instance().remove_all();
}

}  // extern "C"
