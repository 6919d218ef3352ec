// noalloc.cu -- staged retrieve through a staging area built into the library.
//
// lmcb_multi_layer_kv_retrieve_staged needs a device staging buffer as large
// as the LMCache object, which its caller must allocate. Some callers cannot
// allocate device memory at the moment they retrieve: a serving engine that
// has reserved nearly all HBM for its paged KV cache up front (any later
// cudaMalloc may fail), or a native host without a caching allocator, where a
// cudaMalloc / cudaFree pair around every chunk would synchronise the device
// and stall its other streams. This entry point gives them the same staged
// retrieve with the staging area held by the library itself.
//
// The staging area is a file-scope device array of LMCB_NOALLOC_STAGING_BYTES
// (64 MiB). Every GPU on which this library's module is loaded holds it until
// the process exits. Host code cannot use the array's name as a device
// address (in host code it names a host-side stand-in), so the device address
// is looked up once per device with cudaGetSymbolAddress, with that device
// current, and passed to the kernels. The address is kept per device ordinal
// for the life of the process; a cudaDeviceReset while the library is in use
// is not supported (the primary context it was looked up in is gone).
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "lmcache_b200.h"

namespace lmcb {
namespace {

static __device__ __align__(256) uint8_t g_noalloc_staging[LMCB_NOALLOC_STAGING_BYTES];

std::mutex g_noalloc_mutex;
std::vector<void*> g_noalloc_ptr;  // device address of the array, per device ordinal

// Device address of the staging array on the current device; the lookup
// runs on the first call per device. Returns nullptr (and records the error)
// on failure.
void* noalloc_staging_ptr() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    cuda_fail(err, "cudaGetDevice");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (dev >= static_cast<int>(g_noalloc_ptr.size())) g_noalloc_ptr.resize(dev + 1, nullptr);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_staging);
    if (err != cudaSuccess) {
      cuda_fail(err, "cudaGetSymbolAddress(staging area)");
      return nullptr;
    }
    g_noalloc_ptr[dev] = p;
  }
  return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace lmcb

extern "C" {

int lmcb_multi_layer_kv_retrieve_staged_noalloc(int type, int slotType, void* stream,
                                                const uint64_t* pagedKVCaches,
                                                const void* hostCacheTensor,
                                                const void* slotmappings, int64_t hiddenDims,
                                                int32_t kvs, int32_t numLayers,
                                                int64_t pageBuffSize, int32_t numTokensChunk) {
  lmcb::clear_error();
  const int64_t esz = lmcb::dtype_size(type);
  if (esz == 0) {
    return lmcb::fail(LMCB_ERR_UNSUPPORTED_DTYPE,
                      "multi_layer_kv_retrieve_staged_noalloc: ScalarType not supported.");
  }
  if (kvs != 1 && kvs != 2) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      "multi_layer_kv_retrieve_staged_noalloc: kvs must be 1 or 2.");
  }
  if (hiddenDims < 0 || numLayers < 0 || numTokensChunk < 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      "multi_layer_kv_retrieve_staged_noalloc: negative size.");
  }
  // A product that does not fit 64 bits is certainly larger than the area;
  // checking for overflow keeps a wrapped size from passing the bound.
  uint64_t bytes = 0;
  if (!lmcb::object_bytes(kvs, numLayers, numTokensChunk, hiddenDims, esz, &bytes)) {
    bytes = UINT64_MAX;
  }
  if (bytes > LMCB_NOALLOC_STAGING_BYTES) {
    return lmcb::fail(LMCB_ERR_CAPACITY,
                      "multi_layer_kv_retrieve_staged_noalloc: the object is " +
                          std::to_string(bytes) + " bytes; the built-in staging area holds " +
                          std::to_string(static_cast<uint64_t>(LMCB_NOALLOC_STAGING_BYTES)) +
                          " (use lmcb_multi_layer_kv_retrieve_staged with a caller buffer)");
  }
  if (bytes == 0) return LMCB_OK;
  void* staging = lmcb::noalloc_staging_ptr();
  if (staging == nullptr) return LMCB_ERR_CUDA;
  // Every byte the scatter reads is first written by this call's copy, so
  // what an earlier call left in the area never reaches the output.
  return lmcb_multi_layer_kv_retrieve_staged(type, slotType, stream, pagedKVCaches,
                                             hostCacheTensor, staging,
                                             LMCB_NOALLOC_STAGING_BYTES, slotmappings,
                                             hiddenDims, kvs, numLayers, pageBuffSize,
                                             numTokensChunk);
}

}  // extern "C"
