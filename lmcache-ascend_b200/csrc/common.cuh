// common.cuh -- shared host/device helpers of the lmcache_b200 library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "lmcache_b200.h"

namespace lmcb {

// Thread-local message of the last failing C-ABI call.
void set_error(const std::string& msg);
void clear_error();

// Records `msg` and returns `status` (for `return fail(...)`).
int fail(int status, const std::string& msg);

// Turns a CUDA error into LMCB_ERR_CUDA with a message naming `what`.
int cuda_fail(cudaError_t err, const char* what);

#define LMCB_CUDA_TRY(expr)                                  \
  do {                                                       \
    cudaError_t lmcb_err_ = (expr);                          \
    if (lmcb_err_ != cudaSuccess) {                          \
      return ::lmcb::cuda_fail(lmcb_err_, #expr);            \
    }                                                        \
  } while (0)

// Number of SMs of the current device (cached per device).
int current_sm_count();

// Element size of an lmcb_dtype (0 if unknown).
int dtype_size(int dtype);

// Bytes of a dense [kvs, layers, tokens, hidden] object of `esz`-byte
// elements. Returns false, leaving *out unset, when a factor is negative or
// the product does not fit 64 bits.
inline bool object_bytes(int64_t kvs, int64_t layers, int64_t tokens, int64_t hidden,
                         int64_t esz, uint64_t* out) {
  if (kvs < 0 || layers < 0 || tokens < 0 || hidden < 0 || esz < 0) return false;
  uint64_t b = static_cast<uint64_t>(kvs);
  for (int64_t f : {layers, tokens, hidden, esz}) {
    if (__builtin_mul_overflow(b, static_cast<uint64_t>(f), &b)) return false;
  }
  *out = b;
  return true;
}

// Device address of the current device's status word (LMCB_DEVICE_FLAG_*
// bits). Kernels receive it as an argument and set bits with atomicOr; the
// address is looked up once per device ordinal and kept for the life of the
// process, so a cudaDeviceReset while the library is in use is not supported.
// Returns NULL on failure (and records the error).
unsigned int* device_status_ptr();

__device__ __forceinline__ void raise_flag(unsigned int* status, unsigned int flag) {
  atomicOr(status, flag);
}

// Raises kernel `Fn`'s dynamic shared-memory limit to max(bytes, cap) once
// per device (the attribute call costs microseconds; later launches only
// compare against the cached limit). One cache per kernel: Fn is a template
// argument, not a parameter, so kernels with equal signatures stay distinct.
template <auto Fn>
cudaError_t ensure_smem_limit(size_t bytes, size_t cap) {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> limit[kMaxDevices];
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const int want = static_cast<int>(bytes > cap ? bytes : cap);
  if (dev < 0 || dev >= kMaxDevices) {
    return cudaFuncSetAttribute(reinterpret_cast<const void*>(Fn),
                                cudaFuncAttributeMaxDynamicSharedMemorySize, want);
  }
  if (limit[dev].load(std::memory_order_relaxed) >= static_cast<int>(bytes)) return cudaSuccess;
  err = cudaFuncSetAttribute(reinterpret_cast<const void*>(Fn),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, want);
  if (err == cudaSuccess) limit[dev].store(want, std::memory_order_relaxed);
  return err;
}

// Unsigned division by a loop-invariant divisor with a multiply-high and a
// shift (the round-up method of Granlund and Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994). Valid for
// numerators below 2^31 and divisors in [1, 2^31).
struct FastDiv {
  uint32_t d;
  uint32_t m;
  uint32_t s;

  __host__ __device__ FastDiv() : d(1), m(0), s(0) {}

  __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
    uint32_t l = 0;
    while ((uint64_t(1) << l) < divisor) ++l;
    s = l;
    // m = floor(2^32 * (2^l - d) / d) + 1
    m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - divisor)) / divisor + 1);
  }

  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    uint32_t t = __umulhi(n, m);
    return (t + n) >> s;
  }
};

}  // namespace lmcb
