// common.cu -- error state, device properties and small C-ABI helpers.
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace lmcb {

namespace {
__device__ unsigned int g_device_status = 0;

thread_local std::string t_last_error;

std::mutex g_sm_mutex;
std::vector<int> g_sm_count;  // indexed by device ordinal, 0 = not queried
std::vector<unsigned int*> g_status_ptr;  // indexed by device ordinal
}  // namespace

unsigned int* device_status_ptr() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    cuda_fail(err, "cudaGetDevice");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (dev >= static_cast<int>(g_status_ptr.size())) g_status_ptr.resize(dev + 1, nullptr);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_device_status);
    if (err != cudaSuccess) {
      cuda_fail(err, "cudaGetSymbolAddress(status word)");
      return nullptr;
    }
    g_status_ptr[dev] = static_cast<unsigned int*>(p);
  }
  return g_status_ptr[dev];
}

void set_error(const std::string& msg) { t_last_error = msg; }
void clear_error() { t_last_error.clear(); }

int fail(int status, const std::string& msg) {
  set_error(msg);
  return status;
}

int cuda_fail(cudaError_t err, const char* what) {
  set_error(std::string(what) + ": " + cudaGetErrorName(err) + " (" +
            cudaGetErrorString(err) + ")");
  return LMCB_ERR_CUDA;
}

int current_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (dev >= static_cast<int>(g_sm_count.size())) g_sm_count.resize(dev + 1, 0);
  if (g_sm_count[dev] == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0) {
      sms = 148;
    }
    g_sm_count[dev] = sms;
  }
  return g_sm_count[dev];
}

int dtype_size(int dtype) {
  switch (dtype) {
    case LMCB_DTYPE_FP32: return 4;
    case LMCB_DTYPE_BF16: return 2;
    case LMCB_DTYPE_FP16: return 2;
    case LMCB_DTYPE_INT64: return 8;
    case LMCB_DTYPE_INT32: return 4;
    default: return 0;
  }
}

}  // namespace lmcb

extern "C" {

const char* lmcb_version(void) { return "0.1.0"; }

const char* lmcb_last_error(void) { return lmcb::t_last_error.c_str(); }

const char* lmcb_status_string(int status) {
  switch (status) {
    case LMCB_OK: return "LMCB_OK";
    case LMCB_ERR_INVALID_ARGUMENT: return "LMCB_ERR_INVALID_ARGUMENT";
    case LMCB_ERR_UNSUPPORTED_DTYPE: return "LMCB_ERR_UNSUPPORTED_DTYPE";
    case LMCB_ERR_CUDA: return "LMCB_ERR_CUDA";
    case LMCB_ERR_NOT_REGISTERED: return "LMCB_ERR_NOT_REGISTERED";
    case LMCB_ERR_NOT_IMPLEMENTED: return "LMCB_ERR_NOT_IMPLEMENTED";
    case LMCB_ERR_CAPACITY: return "LMCB_ERR_CAPACITY";
    default: return "LMCB_ERR_UNKNOWN";
  }
}

int lmcb_dtype_size(int dtype) { return lmcb::dtype_size(dtype); }

int lmcb_device_status(int device, uint32_t* flags_out) {
  lmcb::clear_error();
  if (flags_out == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "lmcb_device_status: flags_out is NULL");
  }
  int prev = 0;
  LMCB_CUDA_TRY(cudaGetDevice(&prev));
  LMCB_CUDA_TRY(cudaSetDevice(device));
  unsigned int value = 0;
  const unsigned int zero = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&value, lmcb::g_device_status, sizeof(value));
  if (err == cudaSuccess) {
    err = cudaMemcpyToSymbol(lmcb::g_device_status, &zero, sizeof(zero));
  }
  cudaSetDevice(prev);
  if (err != cudaSuccess) return lmcb::cuda_fail(err, "lmcb_device_status");
  *flags_out = value;
  return LMCB_OK;
}

}  // extern "C"
