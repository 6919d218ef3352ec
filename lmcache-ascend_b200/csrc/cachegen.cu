// cachegen.cu -- CacheGen per-channel CDF and range-coder kernels for sm_100a.
//
// The reference exports calculate_cdf / encode_fast_new / decode_fast_new /
// decode_fast_prefsum (csrc/pybind.cpp:21-24) but leaves them unimplemented
// (csrc/cachegen_kernels.cpp:7-32). This file implements them with the format
// declared in include/lmcache_b200.h:
//   * CDF per (layer, channel) stream: add-one-smoothed scaled empirical
//     cumulative counts, cdf[0] = 0, cdf[max_bins] = 2^15, uint16 values.
//   * Carry-less byte-oriented range coder (D. Subbotin, 1999): 32-bit low and
//     range, renormalisation when the top byte is settled (TOP = 2^24) or the
//     range drops below BOT = 2^16, total frequency 2^15 (so the per-symbol
//     range division is a shift on the encoder side).
//
// Kernels:
//   cdf_kernel     one CTA per (layer, 32 channels): the 8 warps stream the
//                  [T, 32] symbol tile with coalesced 32-byte row reads and
//                  count into per-channel shared-memory histograms; then one
//                  warp per channel scans its histogram (warp shuffle prefix
//                  sum) and writes the channel's CDF row.
//   encode/decode  one thread per (layer, channel) stream, 32 consecutive
//                  channels per warp so symbol reads and writes of one token
//                  row are coalesced; the CTA's CDF rows are staged in shared
//                  memory; symbols pass through a shared-memory tile of
//                  kTokTile tokens. The coder itself is sequential per stream.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "common.cuh"
#include "lmcache_b200.h"

namespace lmcb {
namespace {

constexpr uint32_t kProbBits = 15;
constexpr uint32_t kTotal = 1u << kProbBits;
constexpr uint32_t kTop = 1u << 24;
constexpr uint32_t kBot = 1u << 16;
constexpr int kMaxBins = 256;
constexpr int kMaxRenorm = 16;

// ---------------------------------------------------------------------------
// calculate_cdf
// ---------------------------------------------------------------------------

constexpr int kCdfThreads = 256;
constexpr int kCdfChannels = 32;

__global__ void __launch_bounds__(kCdfThreads)
cdf_kernel(const uint8_t* __restrict__ sym, uint16_t* __restrict__ cdf, int T, int C,
           int max_bins, unsigned int* status) {
  __shared__ uint32_t hist[kCdfChannels][kMaxBins + 1];
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCdfChannels;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  constexpr int kWarps = kCdfThreads / 32;

  for (int i = threadIdx.x; i < kCdfChannels * (kMaxBins + 1); i += kCdfThreads) {
    (&hist[0][0])[i] = 0;
  }
  __syncthreads();

  const int c = c0 + lane;
  const uint8_t* base = sym + static_cast<int64_t>(l) * T * C;
  bool oor = false;
  if (c < C) {
    for (int t = warp; t < T; t += kWarps) {
      const uint32_t s = base[static_cast<int64_t>(t) * C + c];
      if (s < static_cast<uint32_t>(max_bins)) {
        atomicAdd(&hist[lane][s], 1u);
      } else {
        oor = true;
      }
    }
  }
  if (__any_sync(0xffffffffu, oor) && lane == 0) raise_flag(status, LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE);
  __syncthreads();

  // One warp per channel: lane j owns bins [8j, 8j + 8).
  for (int ch = warp; ch < kCdfChannels; ch += kWarps) {
    const int cc = c0 + ch;
    if (cc >= C) break;  // warp-uniform
    uint32_t local[8];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = lane * 8 + j;
      local[j] = k < max_bins ? hist[ch][k] : 0u;
      sum += local[j];
    }
    // Inclusive warp scan of per-lane sums.
    uint32_t incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    const uint32_t n = __shfl_sync(0xffffffffu, incl, 31);
    uint32_t cum = incl - sum;  // exclusive prefix = symbols below bin 8*lane
    uint16_t* out = cdf + (static_cast<int64_t>(l) * C + cc) * (max_bins + 1);
    const uint64_t scale = kTotal - static_cast<uint32_t>(max_bins);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = lane * 8 + j;
      if (k < max_bins) {
        uint32_t v;
        if (n > 0) {
          v = static_cast<uint32_t>(static_cast<uint64_t>(cum) * scale / n) + k;
        } else {
          v = static_cast<uint32_t>((static_cast<uint64_t>(k) * kTotal) / max_bins);
        }
        out[k] = static_cast<uint16_t>(v);
      }
      cum += local[j];
    }
    if (lane == 0) out[max_bins] = static_cast<uint16_t>(kTotal);
  }
}

// ---------------------------------------------------------------------------
// encode / decode
// ---------------------------------------------------------------------------

constexpr int kCoderThreads = 128;  // channels per CTA
constexpr int kTokTile = 32;        // tokens staged per shared-memory tile

// Shared memory: CDF rows [kCoderThreads][max_bins + 1] (uint16), then the
// symbol tile [kTokTile][kCoderThreads] (uint8).
inline size_t coder_smem_bytes(int max_bins) {
  size_t cdf = static_cast<size_t>(kCoderThreads) * (max_bins + 1) * sizeof(uint16_t);
  cdf = (cdf + 15) & ~size_t(15);
  return cdf + static_cast<size_t>(kTokTile) * kCoderThreads;
}

__device__ __forceinline__ void load_cdf_rows(uint16_t* s_cdf, const uint16_t* cdf, int l, int c0,
                                              int C, int max_bins) {
  const int n_ch = min(kCoderThreads, C - c0);
  const int64_t n = static_cast<int64_t>(n_ch) * (max_bins + 1);
  const uint16_t* src = cdf + (static_cast<int64_t>(l) * C + c0) * (max_bins + 1);
  for (int64_t i = threadIdx.x; i < n; i += kCoderThreads) s_cdf[i] = src[i];
}

struct ByteSink {
  uint8_t* out;
  int64_t cap;
  int64_t pos;
  uint32_t word;
  bool words;  // 4-byte aligned stream start and cap % 4 == 0
  bool overflow;

  __device__ __forceinline__ void put(uint32_t b) {
    b &= 0xffu;
    if (pos < cap) {
      if (words) {
        word |= b << (8 * (pos & 3));
        if ((pos & 3) == 3) {
          reinterpret_cast<uint32_t*>(out)[pos >> 2] = word;
          word = 0;
        }
      } else {
        out[pos] = static_cast<uint8_t>(b);
      }
    } else {
      overflow = true;
    }
    ++pos;
  }

  __device__ __forceinline__ void flush() {
    if (words && (pos & 3) != 0 && pos <= cap) {
      const int64_t base = pos & ~int64_t(3);
      for (int64_t i = base; i < pos; ++i) out[i] = static_cast<uint8_t>(word >> (8 * (i - base)));
    }
  }
};

__global__ void __launch_bounds__(kCoderThreads)
encode_kernel(const uint16_t* __restrict__ cdf, const uint8_t* __restrict__ sym,
              uint8_t* __restrict__ out, int32_t* __restrict__ lengths, int T, int C,
              int max_bins, int64_t stride, unsigned int* status) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* s_cdf = reinterpret_cast<uint16_t*>(smem);
  uint8_t* s_sym = smem + ((static_cast<size_t>(kCoderThreads) * (max_bins + 1) * 2 + 15) & ~size_t(15));
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCoderThreads;
  const int tid = threadIdx.x;
  const int c = c0 + tid;
  const bool active = c < C;
  load_cdf_rows(s_cdf, cdf, l, c0, C, max_bins);

  const uint16_t* my_cdf = s_cdf + tid * (max_bins + 1);
  const int64_t stream = static_cast<int64_t>(l) * C + c;
  ByteSink sink;
  sink.out = out + stream * stride;
  sink.cap = stride;
  sink.pos = 0;
  sink.word = 0;
  sink.words = ((reinterpret_cast<uintptr_t>(out) | static_cast<uint64_t>(stride)) & 3) == 0;
  sink.overflow = false;
  uint32_t low = 0, range = 0xFFFFFFFFu;
  bool oor = false;
  const uint8_t* base = sym + static_cast<int64_t>(l) * T * C;
  const int n_ch = min(kCoderThreads, C - c0);

  for (int t0 = 0; t0 < T; t0 += kTokTile) {
    const int nt = min(kTokTile, T - t0);
    __syncthreads();  // previous tile consumed (and the CDF rows loaded)
    for (int i = tid; i < nt * kCoderThreads; i += kCoderThreads) {
      const int tt = i / kCoderThreads;
      const int cc = i - tt * kCoderThreads;
      if (cc < n_ch) s_sym[tt * kCoderThreads + cc] = base[static_cast<int64_t>(t0 + tt) * C + c0 + cc];
    }
    __syncthreads();
    if (active) {
      for (int tt = 0; tt < nt; ++tt) {
        uint32_t s = s_sym[tt * kCoderThreads + tid];
        if (s >= static_cast<uint32_t>(max_bins)) {
          oor = true;
          s = max_bins - 1;
        }
        const uint32_t lo = my_cdf[s];
        const uint32_t hi = my_cdf[s + 1];
        const uint32_t r = range >> kProbBits;
        low += lo * r;
        range = r * (hi - lo);
        // At most four byte shifts are ever needed; the bound only guards
        // against a state the coder cannot reach.
        for (int it = 0; it < kMaxRenorm; ++it) {
          if ((low ^ (low + range)) >= kTop) {
            if (range >= kBot) break;
            range = (0u - low) & (kBot - 1u);
          }
          sink.put(low >> 24);
          low <<= 8;
          range <<= 8;
        }
      }
    }
  }
  if (active) {
    for (int i = 0; i < 4; ++i) {
      sink.put(low >> 24);
      low <<= 8;
    }
    sink.flush();
    lengths[stream] = sink.overflow ? -1 : static_cast<int32_t>(sink.pos);
    if (sink.overflow) raise_flag(status, LMCB_DEVICE_FLAG_STREAM_OVERFLOW);
    if (oor) raise_flag(status, LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE);
  }
}

// Decodes with streams either at fixed stride (ends == nullptr) or
// concatenated with inclusive end offsets.
__global__ void __launch_bounds__(kCoderThreads)
decode_kernel(const uint16_t* __restrict__ cdf, const uint8_t* __restrict__ in,
              const int32_t* __restrict__ lengths, const int64_t* __restrict__ ends,
              uint8_t* __restrict__ sym, int T, int C, int max_bins, int64_t stride,
              int64_t total_bytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* s_cdf = reinterpret_cast<uint16_t*>(smem);
  uint8_t* s_sym = smem + ((static_cast<size_t>(kCoderThreads) * (max_bins + 1) * 2 + 15) & ~size_t(15));
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCoderThreads;
  const int tid = threadIdx.x;
  const int c = c0 + tid;
  const bool active = c < C;
  load_cdf_rows(s_cdf, cdf, l, c0, C, max_bins);

  const uint16_t* my_cdf = s_cdf + tid * (max_bins + 1);
  const int64_t stream = static_cast<int64_t>(l) * C + c;
  const uint8_t* src = nullptr;
  int64_t len = 0;
  if (active) {
    if (ends == nullptr) {
      src = in + stream * stride;
      len = lengths[stream];
      if (len < 0) len = 0;
      if (len > stride) len = stride;
    } else {
      // Offsets are clamped to the buffer, so a bad prefix sum cannot read
      // outside it.
      int64_t start = stream == 0 ? 0 : ends[stream - 1];
      int64_t end = ends[stream];
      start = start < 0 ? 0 : (start > total_bytes ? total_bytes : start);
      end = end < start ? start : (end > total_bytes ? total_bytes : end);
      src = in + start;
      len = end - start;
    }
  }
  int64_t pos = 0;
  auto next = [&]() -> uint32_t {
    const uint32_t b = pos < len ? static_cast<uint32_t>(__ldg(src + pos)) : 0u;
    ++pos;
    return b;
  };
  uint32_t low = 0, range = 0xFFFFFFFFu, code = 0;
  if (active) {
    for (int i = 0; i < 4; ++i) code = (code << 8) | next();
  }
  uint8_t* base = sym + static_cast<int64_t>(l) * T * C;
  const int n_ch = min(kCoderThreads, C - c0);

  for (int t0 = 0; t0 < T; t0 += kTokTile) {
    const int nt = min(kTokTile, T - t0);
    if (active) {
      for (int tt = 0; tt < nt; ++tt) {
        const uint32_t r = range >> kProbBits;
        uint32_t v = (code - low) / r;
        if (v >= kTotal) v = kTotal - 1;
        int a = 0, b = max_bins;  // cdf[a] <= v < cdf[b]
        while (b - a > 1) {
          const int m = (a + b) >> 1;
          if (my_cdf[m] <= v) a = m; else b = m;
        }
        const uint32_t lo = my_cdf[a];
        const uint32_t hi = my_cdf[a + 1];
        low += lo * r;
        range = r * (hi - lo);
        for (int it = 0; it < kMaxRenorm; ++it) {
          if ((low ^ (low + range)) >= kTop) {
            if (range >= kBot) break;
            range = (0u - low) & (kBot - 1u);
          }
          code = (code << 8) | next();
          low <<= 8;
          range <<= 8;
        }
        s_sym[tt * kCoderThreads + tid] = static_cast<uint8_t>(a);
      }
    }
    __syncthreads();
    for (int i = tid; i < nt * kCoderThreads; i += kCoderThreads) {
      const int tt = i / kCoderThreads;
      const int cc = i - tt * kCoderThreads;
      if (cc < n_ch) base[static_cast<int64_t>(t0 + tt) * C + c0 + cc] = s_sym[tt * kCoderThreads + cc];
    }
    __syncthreads();
  }
}

int check_codec_args(const char* who, int L, int T, int C, int max_bins) {
  if (L < 0 || T < 0 || C < 0) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": negative size.");
  }
  if (max_bins < 1 || max_bins > kMaxBins) {
    return fail(LMCB_ERR_INVALID_ARGUMENT,
                std::string(who) + ": max_bins must be in [1, 256], got " + std::to_string(max_bins));
  }
  return LMCB_OK;
}

// Largest coder shared-memory footprint (max_bins = 256).
inline size_t coder_smem_cap() { return coder_smem_bytes(kMaxBins); }

}  // namespace
}  // namespace lmcb

extern "C" {

int lmcb_calculate_cdf(const int8_t* input, int16_t* cdfOut, int32_t numLayers, int32_t numTokens,
                       int32_t numChannels, int32_t maxBins, void* stream) {
  lmcb::clear_error();
  int st = lmcb::check_codec_args("calculate_cdf", numLayers, numTokens, numChannels, maxBins);
  if (st != LMCB_OK) return st;
  if (numLayers == 0 || numChannels == 0) return LMCB_OK;
  if ((input == nullptr && numTokens > 0) || cdfOut == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "calculate_cdf: NULL pointer.");
  }
  unsigned int* status = lmcb::device_status_ptr();
  if (status == nullptr) return LMCB_ERR_CUDA;
  dim3 grid((numChannels + lmcb::kCdfChannels - 1) / lmcb::kCdfChannels, numLayers);
  lmcb::cdf_kernel<<<grid, lmcb::kCdfThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint8_t*>(input), reinterpret_cast<uint16_t*>(cdfOut), numTokens,
      numChannels, maxBins, status);
  LMCB_CUDA_TRY(cudaGetLastError());
  return LMCB_OK;
}

int lmcb_encode(const int16_t* cdf, const int8_t* inputSym, uint8_t* outputBuffer,
                int32_t* outputLengths, int32_t numLayers, int32_t numTokens, int32_t numChannels,
                int32_t maxBins, int64_t bufferStride, void* stream) {
  lmcb::clear_error();
  int st = lmcb::check_codec_args("encode", numLayers, numTokens, numChannels, maxBins);
  if (st != LMCB_OK) return st;
  if (numLayers == 0 || numChannels == 0) return LMCB_OK;
  if (bufferStride <= 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "encode: buffer capacity must be positive.");
  }
  if (cdf == nullptr || (inputSym == nullptr && numTokens > 0) || outputBuffer == nullptr ||
      outputLengths == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "encode: NULL pointer.");
  }
  unsigned int* status = lmcb::device_status_ptr();
  if (status == nullptr) return LMCB_ERR_CUDA;
  const size_t smem = lmcb::coder_smem_bytes(maxBins);
  LMCB_CUDA_TRY(lmcb::ensure_smem_limit<&lmcb::encode_kernel>(smem, lmcb::coder_smem_cap()));
  dim3 grid((numChannels + lmcb::kCoderThreads - 1) / lmcb::kCoderThreads, numLayers);
  lmcb::encode_kernel<<<grid, lmcb::kCoderThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(cdf), reinterpret_cast<const uint8_t*>(inputSym),
      outputBuffer, outputLengths, numTokens, numChannels, maxBins, bufferStride, status);
  LMCB_CUDA_TRY(cudaGetLastError());
  return LMCB_OK;
}

int lmcb_decode(const int16_t* cdf, const uint8_t* bytestreams, const int32_t* lengths,
                int8_t* output, int32_t numLayers, int32_t numTokens, int32_t numChannels,
                int32_t maxBins, int64_t bufferStride, void* stream) {
  lmcb::clear_error();
  int st = lmcb::check_codec_args("decode", numLayers, numTokens, numChannels, maxBins);
  if (st != LMCB_OK) return st;
  if (numLayers == 0 || numChannels == 0 || numTokens == 0) return LMCB_OK;
  if (bufferStride <= 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "decode: buffer capacity must be positive.");
  }
  if (cdf == nullptr || bytestreams == nullptr || lengths == nullptr || output == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "decode: NULL pointer.");
  }
  const size_t smem = lmcb::coder_smem_bytes(maxBins);
  LMCB_CUDA_TRY(lmcb::ensure_smem_limit<&lmcb::decode_kernel>(smem, lmcb::coder_smem_cap()));
  dim3 grid((numChannels + lmcb::kCoderThreads - 1) / lmcb::kCoderThreads, numLayers);
  lmcb::decode_kernel<<<grid, lmcb::kCoderThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(cdf), bytestreams, lengths, nullptr,
      reinterpret_cast<uint8_t*>(output), numTokens, numChannels, maxBins, bufferStride, 0);
  LMCB_CUDA_TRY(cudaGetLastError());
  return LMCB_OK;
}

int lmcb_decode_prefsum(const int16_t* cdf, const uint8_t* bytestreams, int64_t streamBytes,
                        const int64_t* endOffsets, int8_t* output, int32_t numLayers,
                        int32_t numTokens, int32_t numChannels, int32_t maxBins, void* stream) {
  lmcb::clear_error();
  int st = lmcb::check_codec_args("decode_prefsum", numLayers, numTokens, numChannels, maxBins);
  if (st != LMCB_OK) return st;
  if (numLayers == 0 || numChannels == 0 || numTokens == 0) return LMCB_OK;
  if (cdf == nullptr || (bytestreams == nullptr && streamBytes > 0) || endOffsets == nullptr ||
      output == nullptr || streamBytes < 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, "decode_prefsum: NULL pointer or negative size.");
  }
  const size_t smem = lmcb::coder_smem_bytes(maxBins);
  LMCB_CUDA_TRY(lmcb::ensure_smem_limit<&lmcb::decode_kernel>(smem, lmcb::coder_smem_cap()));
  dim3 grid((numChannels + lmcb::kCoderThreads - 1) / lmcb::kCoderThreads, numLayers);
  lmcb::decode_kernel<<<grid, lmcb::kCoderThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(cdf), bytestreams, nullptr, endOffsets,
      reinterpret_cast<uint8_t*>(output), numTokens, numChannels, maxBins, 0, streamBytes);
  LMCB_CUDA_TRY(cudaGetLastError());
  return LMCB_OK;
}

}  // extern "C"
