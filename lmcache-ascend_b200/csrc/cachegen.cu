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
//   cdf_kernel     one CTA per (layer, 32 channels), lane = channel: the 8
//                  warps stream the [T, 32] symbol tile with coalesced 32-byte
//                  row reads and count into transposed shared-memory
//                  histograms (conflict-free atomics); then each warp scales
//                  an eighth of the bins of every channel, and the CTA writes
//                  its CDF rows with one coalesced copy.
//   encode/decode  one thread per (layer, channel) stream, 32 consecutive
//                  channels per warp so symbol reads and writes of one token
//                  row are coalesced; the CTA's CDF rows are staged in shared
//                  memory, transposed so probes are bank-conflict free. The
//                  coder itself is sequential per stream, so both kernels are
//                  bound by the latency of one symbol step: encode prefetches
//                  symbols several tokens ahead, decode loads the next input
//                  byte ahead, keeps the search's first levels in registers
//                  and tests all probes of a round at once.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
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
constexpr int kCdfWarps = kCdfThreads / 32;

// floor(x / n) for x < 2^46 and 0 < n < 2^31, with rn = 1.0 / n (rounded):
// the double-precision product is within 2^-6 of x / n (relative error below
// 2^-51), so its truncation is floor(x / n) or one off, and one exact integer
// test each way fixes it. This replaces a 64-bit integer division (a long
// software sequence) per CDF bin.
__device__ __forceinline__ uint64_t div_floor(uint64_t x, uint32_t n, double rn) {
  uint64_t q = static_cast<uint64_t>(static_cast<double>(x) * rn);
  q = q * n > x ? q - 1 : q;
  q = (q + 1) * n <= x ? q + 1 : q;
  return q;
}

// Shared memory of one cdf_kernel CTA: the histograms transposed,
// hist[bin][lane] (each lane counts into its own bank, so atomics never
// conflict), eight per-warp partial sums per channel, and the CTA's output
// rows [32 channels][max_bins + 1] staged for one coalesced write.
inline size_t cdf_smem_bytes(int max_bins) {
  return static_cast<size_t>(max_bins) * kCdfChannels * sizeof(uint32_t) +
         static_cast<size_t>(kCdfWarps) * kCdfChannels * sizeof(uint32_t) +
         static_cast<size_t>(kCdfChannels) * (max_bins + 1) * sizeof(uint16_t);
}

// One CTA per (layer, 32 channels), lane = channel. The eight warps count
// interleaved token rows (32-byte coalesced row reads, four rows per warp in
// flight) into the transposed histograms; eight CTAs per SM (32 registers a
// thread) put a c2 chunk's 1,024 CTAs in one wave; then warp w takes the bins
// [w * ceil(max_bins / 8), ...) of every channel, so each channel's prefix
// sum is the warps' partial sums plus the warp's own running sum.
__global__ void __launch_bounds__(kCdfThreads, 8)
cdf_kernel(const uint8_t* __restrict__ sym, uint16_t* __restrict__ cdf, int T, int C,
           int max_bins, unsigned int* status) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem);  // [max_bins][32]
  uint32_t* part = hist + max_bins * kCdfChannels;      // [8][32]
  uint16_t* tile = reinterpret_cast<uint16_t*>(part + kCdfWarps * kCdfChannels);
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCdfChannels;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;

  for (int i = threadIdx.x; i < max_bins * kCdfChannels; i += kCdfThreads) hist[i] = 0;
  __syncthreads();

  const int c = c0 + lane;
  const uint8_t* base = sym + static_cast<int64_t>(l) * T * C + c;
  bool oor = false;
  auto count = [&](uint32_t s) {
    if (s < static_cast<uint32_t>(max_bins)) {
      atomicAdd(&hist[s * kCdfChannels + lane], 1u);
    } else {
      oor = true;
    }
  };
  if (c < C) {
    constexpr int kRows = 4;
    int t = warp;
    for (; t + (kRows - 1) * kCdfWarps < T; t += kRows * kCdfWarps) {
      uint32_t v[kRows];
#pragma unroll
      for (int j = 0; j < kRows; ++j) v[j] = base[static_cast<int64_t>(t + j * kCdfWarps) * C];
#pragma unroll
      for (int j = 0; j < kRows; ++j) count(v[j]);
    }
    for (; t < T; t += kCdfWarps) count(base[static_cast<int64_t>(t) * C]);
  }
  if (__any_sync(0xffffffffu, oor) && lane == 0) raise_flag(status, LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE);
  __syncthreads();

  const int per = (max_bins + kCdfWarps - 1) / kCdfWarps;
  const int b0 = min(warp * per, max_bins);
  const int b1 = min(b0 + per, max_bins);
  uint32_t sum = 0;
  for (int k = b0; k < b1; ++k) sum += hist[k * kCdfChannels + lane];
  part[warp * kCdfChannels + lane] = sum;
  __syncthreads();
  uint32_t n = 0, cum = 0;
#pragma unroll
  for (int w = 0; w < kCdfWarps; ++w) {
    const uint32_t v = part[w * kCdfChannels + lane];
    n += v;
    cum += w < warp ? v : 0u;  // symbols below bin b0
  }
  const uint64_t scale = kTotal - static_cast<uint32_t>(max_bins);
  const double rn = n > 0 ? 1.0 / static_cast<double>(n) : 0.0;
  uint16_t* row = tile + lane * (max_bins + 1);
  for (int k = b0; k < b1; ++k) {
    uint32_t v;
    if (n > 0) {
      v = static_cast<uint32_t>(div_floor(static_cast<uint64_t>(cum) * scale, n, rn)) + k;
    } else {
      v = (static_cast<uint32_t>(k) * kTotal) / static_cast<uint32_t>(max_bins);
    }
    row[k] = static_cast<uint16_t>(v);
    cum += hist[k * kCdfChannels + lane];
  }
  if (warp == 0) row[max_bins] = static_cast<uint16_t>(kTotal);
  __syncthreads();

  // The CTA's rows are contiguous in the output.
  const int nch = min(kCdfChannels, C - c0);
  const int count_out = nch * (max_bins + 1);
  uint16_t* out = cdf + (static_cast<int64_t>(l) * C + c0) * (max_bins + 1);
  for (int i = threadIdx.x; i < count_out; i += kCdfThreads) out[i] = tile[i];
}

// ---------------------------------------------------------------------------
// encode / decode
// ---------------------------------------------------------------------------

constexpr int kCoderThreads = 128;  // channels (streams) per CTA
constexpr int kSymAhead = 8;        // encode: symbols prefetched per stream

// Shared memory holds the CTA's CDF rows transposed and widened to 32 bits:
// s_cdf[k * kCoderThreads + i] = cdf[k] of the CTA's i-th channel. Each lane
// owns one bank, so a warp's probes never conflict whatever bin each lane
// looks at.
inline size_t coder_smem_bytes(int max_bins) {
  return static_cast<size_t>(kCoderThreads) * (max_bins + 1) * sizeof(uint32_t);
}

__device__ __forceinline__ void load_cdf_rows(uint32_t* s_cdf, const uint16_t* cdf, int l, int c0,
                                              int C, int max_bins) {
  const int c = c0 + static_cast<int>(threadIdx.x);
  if (c >= C) return;
  const uint16_t* row = cdf + (static_cast<int64_t>(l) * C + c) * (max_bins + 1);
  for (int k = 0; k <= max_bins; ++k) s_cdf[k * kCoderThreads + threadIdx.x] = row[k];
}

// The bytes of one encoded stream, appended in order. With kWords (4-byte
// aligned stream start and capacity) they collect in a 64-bit accumulator and
// leave as whole 32-bit words; otherwise they are stored one by one. Bytes at
// positions >= cap are dropped and set `overflow`.
template <bool kWords>
struct StreamSink {
  uint8_t* out;
  int64_t cap;
  int64_t pos;   // !kWords: bytes appended
  int64_t done;  // kWords: whole words written (or dropped)
  uint64_t acc;  // kWords: pending bytes, the oldest in the low byte
  int na;        // kWords: bytes pending in acc, 0..3 between appends
  bool overflow;

  __device__ __forceinline__ void init(uint8_t* o, int64_t c) {
    out = o;
    cap = c;
    pos = 0;
    done = 0;
    acc = 0;
    na = 0;
    overflow = false;
  }

  // Appends the k (0..4) bytes in the low bytes of v, the first in the
  // lowest byte; the bytes of v above them are zero. In words mode the body
  // is straight-line (a predicated store, selects): lanes of a warp fill
  // their words on different steps, so a branch here would be taken by some
  // lane on almost every step.
  __device__ __forceinline__ void append(uint32_t v, int k) {
    if constexpr (kWords) {
      acc |= static_cast<uint64_t>(v) << (8 * na);
      na += k;
      const bool full = na >= 4;
      const bool fits = done < (cap >> 2);
      if (full && fits) reinterpret_cast<uint32_t*>(out)[done] = static_cast<uint32_t>(acc);
      overflow |= full && !fits;
      done += full ? 1 : 0;
      acc = full ? (acc >> 32) : acc;
      na -= full ? 4 : 0;
    } else {
      for (int i = 0; i < k; ++i) {
        if (pos + i < cap) {
          out[pos + i] = static_cast<uint8_t>(v >> (8 * i));
        } else {
          overflow = true;
        }
      }
      pos += k;
    }
  }

  // Writes the pending bytes; returns the stream length.
  __device__ __forceinline__ int64_t finish() {
    if constexpr (kWords) {
      const int64_t base = done * 4;
      if (na > 0) {
        if (base < cap) {  // cap % 4 == 0, so all na bytes fit
          for (int i = 0; i < na; ++i) out[base + i] = static_cast<uint8_t>(acc >> (8 * i));
        } else {
          overflow = true;
        }
      }
      return base + na;
    } else {
      return pos;
    }
  }
};

// One stream per thread, 32 consecutive channels per warp. Symbols are read
// straight from global memory (a warp reads one 32-byte run of a token row)
// kSymAhead tokens ahead of their use, so their latency overlaps the coding
// of the tokens before them; no block-wide barrier after the CDF load.
template <bool kWords>
__global__ void __launch_bounds__(kCoderThreads)
encode_kernel(const uint16_t* __restrict__ cdf, const uint8_t* __restrict__ sym,
              uint8_t* __restrict__ out, int32_t* __restrict__ lengths, int T, int C,
              int max_bins, int64_t stride, unsigned int* status) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* s_cdf = reinterpret_cast<uint32_t*>(smem);
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCoderThreads;
  const int tid = threadIdx.x;
  const int c = c0 + tid;
  load_cdf_rows(s_cdf, cdf, l, c0, C, max_bins);
  __syncthreads();
  if (c >= C) return;

  const uint32_t* my_cdf = s_cdf + tid;  // my_cdf[k * kCoderThreads] = cdf[k]
  const int64_t stream = static_cast<int64_t>(l) * C + c;
  StreamSink<kWords> sink;
  sink.init(out + stream * stride, stride);
  uint32_t low = 0, range = 0xFFFFFFFFu;
  bool oor = false;
  const uint8_t* in = sym + static_cast<int64_t>(l) * T * C + c;

  auto clamp_symbol = [&](uint32_t s) -> uint32_t {
    if (s >= static_cast<uint32_t>(max_bins)) {
      oor = true;
      s = max_bins - 1;
    }
    return s;
  };
  auto code_range = [&](uint32_t lo, uint32_t hi) {
    const uint32_t r = range >> kProbBits;
    low += lo * r;
    range = r * (hi - lo);
    // Renormalisation emits the top byte of low while it is settled (the
    // same in low and low + range). A shift by 8 bits shifts d = low ^
    // (low + range) by 8 bits too, so the settled bytes are d's leading zero
    // bytes: k = clz(d) / 8 <= 3 of them leave at once, with no loop.
    const uint32_t d = low ^ (low + range);
    const int k = d != 0 ? static_cast<int>(__clz(d) >> 3) : 0;
    // Straight-line for every k, 0 included (mask 0, shifts by 0).
    const uint32_t rev = __byte_perm(low, 0, 0x0123);  // top byte of low lowest
    sink.append(rev & ((1u << (8 * k)) - 1u), k);
    low <<= 8 * k;
    range <<= 8 * k;
    // Now the top byte is unsettled. Done if range >= BOT. Otherwise (or for
    // d == 0, which a valid CDF never produces) continue with the step-by-step
    // rule; at most a few more shifts ever happen, and the bound only guards
    // against a state the coder cannot reach.
    if (range < kBot || d == 0) {
      for (int it = k; it < kMaxRenorm; ++it) {
        if ((low ^ (low + range)) >= kTop) {
          if (range >= kBot) break;
          range = (0u - low) & (kBot - 1u);
        }
        sink.append(low >> 24, 1);
        low <<= 8;
        range <<= 8;
      }
    }
  };
  auto code_symbol = [&](uint32_t s) {
    s = clamp_symbol(s);
    code_range(my_cdf[s * kCoderThreads], my_cdf[(s + 1) * kCoderThreads]);
  };

  uint32_t cur[kSymAhead];
#pragma unroll
  for (int j = 0; j < kSymAhead; ++j) {
    cur[j] = j < T ? static_cast<uint32_t>(__ldg(in + static_cast<int64_t>(j) * C)) : 0u;
  }
  int t0 = 0;
  // Whole blocks of kSymAhead tokens: the next block's symbols are loaded,
  // then this block's are coded with no per-token bounds test.
  for (; t0 + kSymAhead <= T; t0 += kSymAhead) {
    uint32_t nxt[kSymAhead];
#pragma unroll
    for (int j = 0; j < kSymAhead; ++j) {
      const int t = t0 + kSymAhead + j;
      nxt[j] = t < T ? static_cast<uint32_t>(__ldg(in + static_cast<int64_t>(t) * C)) : 0u;
    }
    // The block's CDF lookups depend only on its symbols, not on the coder
    // state, so all of them are issued before the first is used.
    uint32_t lo[kSymAhead], hi[kSymAhead];
#pragma unroll
    for (int j = 0; j < kSymAhead; ++j) {
      const uint32_t sj = clamp_symbol(cur[j]);
      lo[j] = my_cdf[sj * kCoderThreads];
      hi[j] = my_cdf[(sj + 1) * kCoderThreads];
    }
#pragma unroll
    for (int j = 0; j < kSymAhead; ++j) code_range(lo[j], hi[j]);
#pragma unroll
    for (int j = 0; j < kSymAhead; ++j) cur[j] = nxt[j];
  }
  // The last T % kSymAhead tokens (already in cur).
#pragma unroll
  for (int j = 0; j < kSymAhead; ++j) {
    if (t0 + j < T) code_symbol(cur[j]);
  }
  // Four bytes of low end the stream.
  sink.append(__byte_perm(low, 0, 0x0123), 4);
  const int64_t n = sink.finish();
  lengths[stream] = sink.overflow ? -1 : static_cast<int32_t>(n);
  if (sink.overflow) raise_flag(status, LMCB_DEVICE_FLAG_STREAM_OVERFLOW);
  if (oor) raise_flag(status, LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE);
}

// One level of the decoder's symbol search: the largest a with cdf[a] <= v,
// v = min((code - low) / r, kTotal - 1), by the halving search
// m = (a + b) / 2 over [a, b). For integers cdf[m] <= floor(x / r) exactly
// when cdf[m] * r <= x, and cdf[m] <= kTotal - 1 is the clamp, so a probe is
// a product and two compares (the product of a value below 2^15 and r below
// 2^17 fits 32 bits). lo / hi carry cdf[a] / cdf[b] (the last accepted and
// the last rejected probe), so the coder needs no separate loads of them.
__device__ __forceinline__ bool probe_ok(uint32_t cm, uint32_t r, uint32_t x) {
  return cm < kTotal && cm * r <= x;
}

// Any alphabet size: the halving search over [0, max_bins), two levels per
// shared-memory round trip (the probe m and both probes the next level can
// take are loaded together, then the taken one is kept). The probe sequence
// is exactly that of the one-level search.
__device__ __forceinline__ uint32_t search_any(const uint32_t* my_cdf, uint32_t r, uint32_t x,
                                               int max_bins, int depth, uint32_t& lo,
                                               uint32_t& hi) {
  uint32_t a = 0, b = static_cast<uint32_t>(max_bins);
  for (int lvl = 0; lvl < depth; lvl += 2) {
    if (b - a <= 1) break;
    const uint32_t m = (a + b) >> 1;
    const uint32_t m_lo = (a + m) >> 1;  // next probe if cdf[m] is rejected
    const uint32_t m_hi = (m + b) >> 1;  // next probe if cdf[m] is accepted
    const uint32_t cm = my_cdf[m * kCoderThreads];
    const uint32_t c_lo = my_cdf[m_lo * kCoderThreads];
    const uint32_t c_hi = my_cdf[m_hi * kCoderThreads];
    const bool ok = probe_ok(cm, r, x);
    if (ok) {
      a = m;
      lo = cm;
    } else {
      b = m;
      hi = cm;
    }
    if (b - a > 1) {
      const uint32_t m2 = ok ? m_hi : m_lo;
      const uint32_t c2 = ok ? c_hi : c_lo;
      if (probe_ok(c2, r, x)) {
        a = m2;
        lo = c2;
      } else {
        b = m2;
        hi = c2;
      }
    }
  }
  return a;
}

// The halving search's choice inside a round of M levels whose probes
// j = 1 .. 2^M - 1 (in units of the round's last step) were all tested at
// once: ok[j - 1] says whether probe j was accepted. The path taken is that of
// the one-level search: the round's first level probes 2^(M-1), and each
// further level probes the middle of the half that the one before it kept.
template <int M>
__device__ __forceinline__ uint32_t pick(const bool (&ok)[(1 << M) - 1]) {
  static_assert(M >= 1 && M <= 3, "rounds of one to three levels");
  if constexpr (M == 1) {
    return ok[0] ? 1u : 0u;
  } else if constexpr (M == 2) {
    const bool o2 = ok[1];
    const bool o1 = o2 ? ok[2] : ok[0];
    return (o2 ? 2u : 0u) + (o1 ? 1u : 0u);
  } else {
    const bool o4 = ok[3];
    const bool o2 = o4 ? ok[5] : ok[1];
    const bool o1 = o4 ? (o2 ? ok[6] : ok[4]) : (o2 ? ok[2] : ok[0]);
    return (o4 ? 4u : 0u) + (o2 ? 2u : 0u) + (o1 ? 1u : 0u);
  }
}

// Search over an alphabet of 2^D symbols (D >= 2) in at most three rounds,
// each testing all probes of its levels at once:
//   * the first R = min(D - 2, 3) levels start from a = 0, so their 2^R - 1
//     probes are the same for every symbol and sit in registers;
//   * the next M = D - 2 - R levels (D > 5 only) take one shared-memory round
//     at probes a + 4j;
//   * the last two levels load cdf[a .. a + 4] together, which also gives
//     cdf[a] and cdf[a + 1] without tracking them through the search.
// The probe sequence, and so the result for any CDF, is the one-level
// search's.
template <int D>
struct Pow2Search {
  static_assert(D >= 2 && D <= 8, "alphabets of 4 to 256 symbols");
  static constexpr int R = (D - 2) < 3 ? (D - 2) : 3;
  static constexpr int M = D - 2 - R;
  // top[j - 1] = min(cdf[j << (D - R)], 2^15), j = 1 .. 2^R - 1.
  uint32_t top[R > 0 ? (1 << R) - 1 : 1];

  __device__ __forceinline__ void init(const uint32_t* my_cdf) {
    if constexpr (R > 0) {
#pragma unroll
      for (int j = 1; j < (1 << R); ++j) {
        const uint32_t v = my_cdf[(j << (D - R)) * kCoderThreads];
        top[j - 1] = v < kTotal ? v : kTotal;
        asm("" : "+r"(top[j - 1]));  // kept in a register, not reloaded per symbol
      }
    }
  }

  __device__ __forceinline__ uint32_t find(const uint32_t* my_cdf, uint32_t range, uint32_t r,
                                           uint32_t x, uint32_t& lo, uint32_t& hi) const {
    uint32_t a = 0;
    if constexpr (R > 0) {
      // For v <= 2^15 and r >= 1 (range >= 2^16 whenever a symbol starts),
      // v <= min(x / r, 2^15 - 1) exactly when v * r <= min(x, 2^15 * r - 1):
      // a value clamped to 2^15 is never accepted, as v >= 2^15 never is.
      const uint32_t xc = min(x, (range & ~(kTotal - 1u)) - 1u);
      bool ok[(1 << R) - 1];
#pragma unroll
      for (int j = 0; j < (1 << R) - 1; ++j) ok[j] = top[j] * r <= xc;
      a = pick<R>(ok) << (D - R);
    }
    if constexpr (M > 0) {
      const uint32_t* row = my_cdf + a * kCoderThreads;
      bool ok[(1 << M) - 1];
#pragma unroll
      for (int j = 1; j < (1 << M); ++j) ok[j - 1] = probe_ok(row[(j << 2) * kCoderThreads], r, x);
      a += pick<M>(ok) << 2;
    }
    const uint32_t* row = my_cdf + a * kCoderThreads;
    const uint32_t c0 = row[0];
    const uint32_t c1 = row[kCoderThreads];
    const uint32_t c2 = row[2 * kCoderThreads];
    const uint32_t c3 = row[3 * kCoderThreads];
    const uint32_t c4 = row[4 * kCoderThreads];
    const bool o2 = probe_ok(c2, r, x);
    const bool o1 = o2 ? probe_ok(c3, r, x) : probe_ok(c1, r, x);
    lo = o2 ? (o1 ? c3 : c2) : (o1 ? c1 : c0);
    hi = o2 ? (o1 ? c4 : c3) : (o1 ? c2 : c1);
    return a + (o2 ? 2u : 0u) + (o1 ? 1u : 0u);
  }
};

// Decodes with streams either at fixed stride (ends == nullptr) or
// concatenated with inclusive end offsets. `depth` = ceil(log2(max_bins)),
// the most levels the halving search can take; kPow2Depth = depth when
// max_bins is a power of two of at least 4 (the three-round search), -1
// otherwise.
// src[i] for i < n, else 0, as a predicated load (no branch around it).
__device__ __forceinline__ uint32_t fetch(const uint8_t* src, int32_t i, int32_t n) {
  uint32_t v;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.lt.s32 p, %1, %2;\n\t"
      "mov.u32 %0, 0;\n\t"
      "@p ld.global.nc.u8 %0, [%3];\n\t}"
      : "=r"(v)
      : "r"(i), "r"(n), "l"(src + i));
  return v;
}

template <int kPow2Depth>
__global__ void __launch_bounds__(kCoderThreads)
decode_kernel(const uint16_t* __restrict__ cdf, const uint8_t* __restrict__ in,
              const int32_t* __restrict__ lengths, const int64_t* __restrict__ ends,
              uint8_t* __restrict__ sym, int T, int C, int max_bins, int depth, int64_t stride,
              int64_t total_bytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* s_cdf = reinterpret_cast<uint32_t*>(smem);
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCoderThreads;
  const int tid = threadIdx.x;
  const int c = c0 + tid;
  load_cdf_rows(s_cdf, cdf, l, c0, C, max_bins);
  __syncthreads();
  if (c >= C) return;

  const uint32_t* my_cdf = s_cdf + tid;  // my_cdf[k * kCoderThreads] = cdf[k]
  const int64_t stream = static_cast<int64_t>(l) * C + c;
  const uint8_t* src;
  int64_t len;
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
  // Bytes past the stream's end read as zero. Positions are 32-bit: the
  // length is clamped below 2^31 - 1 and a position stops at it (every byte
  // from there on reads as zero), so it cannot overflow. (A symbol costs at
  // most about 16 bits, so a stream of 2^31 bytes would hold over 2^30
  // symbols.) The next byte is always loaded one ahead of its use.
  const int32_t n = static_cast<int32_t>(len < INT32_MAX - 1 ? len : INT32_MAX - 1);
  uint32_t code = 0;
  for (int i = 0; i < 4; ++i) code = (code << 8) | fetch(src, i, n);
  int32_t pos = 4;
  uint32_t ahead = fetch(src, pos, n);
  uint32_t low = 0, range = 0xFFFFFFFFu;
  Pow2Search<(kPow2Depth >= 2 ? kPow2Depth : 2)> pow2;
  if constexpr (kPow2Depth >= 2) pow2.init(my_cdf);
  const uint32_t cdf_first = my_cdf[0];
  const uint32_t cdf_last = my_cdf[max_bins * kCoderThreads];
  uint8_t* dst = sym + static_cast<int64_t>(l) * T * C + c;

  for (int t = 0; t < T; ++t) {
    const uint32_t r = range >> kProbBits;
    const uint32_t x = code - low;
    uint32_t lo = cdf_first, hi = cdf_last;
    uint32_t a;
    if constexpr (kPow2Depth >= 2) {
      a = pow2.find(my_cdf, range, r, x, lo, hi);
    } else {
      a = search_any(my_cdf, r, x, max_bins, depth, lo, hi);
    }
    low += lo * r;
    range = r * (hi - lo);
    // The byte-at-a-time rule with one exit test per step; the range reset
    // is a select and the byte load is predicated, so a step has no branch
    // but the exit (lanes of a warp renormalise on different symbols).
    for (int it = 0; it < kMaxRenorm; ++it) {
      const bool unsettled = (low ^ (low + range)) >= kTop;
      if (unsettled && range >= kBot) break;
      range = unsettled ? ((0u - low) & (kBot - 1u)) : range;
      code = (code << 8) | ahead;
      pos = min(pos + 1, n);
      ahead = fetch(src, pos, n);
      low <<= 8;
      range <<= 8;
    }
    dst[static_cast<int64_t>(t) * C] = static_cast<uint8_t>(a);
  }
}

int search_depth(int max_bins) {
  int d = 0;
  while ((1 << d) < max_bins) ++d;
  return d;
}

struct DecodeArgs {
  const uint16_t* cdf;
  const uint8_t* in;
  const int32_t* lengths;  // fixed-stride streams, or
  const int64_t* ends;     // concatenated streams
  uint8_t* sym;
  int L, T, C, max_bins;
  int64_t stride, total_bytes;
};

inline size_t coder_smem_cap();

template <int kPow2Depth>
cudaError_t launch_decode_as(const DecodeArgs& a, cudaStream_t stream) {
  const size_t smem = coder_smem_bytes(a.max_bins);
  cudaError_t err = ensure_smem_limit<&decode_kernel<kPow2Depth>>(smem, coder_smem_cap());
  if (err != cudaSuccess) return err;
  const dim3 grid((a.C + kCoderThreads - 1) / kCoderThreads, a.L);
  decode_kernel<kPow2Depth><<<grid, kCoderThreads, smem, stream>>>(
      a.cdf, a.in, a.lengths, a.ends, a.sym, a.T, a.C, a.max_bins, search_depth(a.max_bins),
      a.stride, a.total_bytes);
  return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream) {
  const int d = search_depth(a.max_bins);
  if ((1 << d) != a.max_bins || d < 2) return launch_decode_as<-1>(a, stream);
  switch (d) {
    case 2: return launch_decode_as<2>(a, stream);
    case 3: return launch_decode_as<3>(a, stream);
    case 4: return launch_decode_as<4>(a, stream);
    case 5: return launch_decode_as<5>(a, stream);
    case 6: return launch_decode_as<6>(a, stream);
    case 7: return launch_decode_as<7>(a, stream);
    default: return launch_decode_as<8>(a, stream);
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
  const size_t smem = lmcb::cdf_smem_bytes(maxBins);
  LMCB_CUDA_TRY(
      lmcb::ensure_smem_limit<&lmcb::cdf_kernel>(smem, lmcb::cdf_smem_bytes(lmcb::kMaxBins)));
  lmcb::cdf_kernel<<<grid, lmcb::kCdfThreads, smem, static_cast<cudaStream_t>(stream)>>>(
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
  dim3 grid((numChannels + lmcb::kCoderThreads - 1) / lmcb::kCoderThreads, numLayers);
  const bool words =
      ((reinterpret_cast<uintptr_t>(outputBuffer) | static_cast<uint64_t>(bufferStride)) & 3) == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (words) {
    LMCB_CUDA_TRY(lmcb::ensure_smem_limit<&lmcb::encode_kernel<true>>(smem, lmcb::coder_smem_cap()));
    lmcb::encode_kernel<true><<<grid, lmcb::kCoderThreads, smem, s>>>(
        reinterpret_cast<const uint16_t*>(cdf), reinterpret_cast<const uint8_t*>(inputSym),
        outputBuffer, outputLengths, numTokens, numChannels, maxBins, bufferStride, status);
  } else {
    LMCB_CUDA_TRY(lmcb::ensure_smem_limit<&lmcb::encode_kernel<false>>(smem, lmcb::coder_smem_cap()));
    lmcb::encode_kernel<false><<<grid, lmcb::kCoderThreads, smem, s>>>(
        reinterpret_cast<const uint16_t*>(cdf), reinterpret_cast<const uint8_t*>(inputSym),
        outputBuffer, outputLengths, numTokens, numChannels, maxBins, bufferStride, status);
  }
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
  const lmcb::DecodeArgs args{reinterpret_cast<const uint16_t*>(cdf), bytestreams, lengths,
                              nullptr, reinterpret_cast<uint8_t*>(output), numLayers, numTokens,
                              numChannels, maxBins, bufferStride, 0};
  LMCB_CUDA_TRY(lmcb::launch_decode(args, static_cast<cudaStream_t>(stream)));
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
  const lmcb::DecodeArgs args{reinterpret_cast<const uint16_t*>(cdf), bytestreams, nullptr,
                              endOffsets, reinterpret_cast<uint8_t*>(output), numLayers,
                              numTokens, numChannels, maxBins, 0, streamBytes};
  LMCB_CUDA_TRY(lmcb::launch_decode(args, static_cast<cudaStream_t>(stream)));
  return LMCB_OK;
}

}  // extern "C"
