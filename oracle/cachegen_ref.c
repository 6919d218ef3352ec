/*
 * cachegen_ref.c -- CPU oracle of the CacheGen codec entry points (test
 * infrastructure only: the tests and the smoke check compare the kernels with it).
 *
 * Reference status: LMCache-Ascend exports calculate_cdf, encode_fast_new,
 * decode_fast_new and decode_fast_prefsum (csrc/pybind.cpp:21-24) but every
 * body raises NotImplementedError (csrc/cachegen_kernels.cpp:7-32); the
 * upstream LMCache v0.3.3 CUDA codec is not part of the reference tree. Parity
 * with upstream bitstreams is therefore unpinned; this file defines the
 * format the B200 kernels must reproduce byte for byte:
 *
 *  Symbols   uint8 values (the int8 tensor's bit patterns) in [0, max_bins),
 *            layout [L, T, C]; one stream per (layer, channel), tokens in order.
 *  CDF       uint16 per (layer, channel): cdf[k], k = 0..max_bins, with
 *            cum[k] = number of in-range symbols < k among the stream's n
 *            in-range symbols:
 *              n > 0:  cdf[k] = floor(cum[k] * (2^15 - max_bins) / n) + k
 *              n == 0: cdf[k] = floor(k * 2^15 / max_bins)
 *            so cdf[0] = 0, cdf[max_bins] = 2^15 and every frequency is >= 1
 *            (add-one smoothing of the scaled empirical distribution).
 *  Coder     the carry-less range coder of D. Subbotin (1999): 32-bit low and
 *            range, TOP = 2^24, BOT = 2^16, total frequency 2^15. Encoding a
 *            symbol s: r = range >> 15; low += cdf[s] * r;
 *            range = r * (cdf[s+1] - cdf[s]); then while
 *            (low ^ (low + range)) < TOP, or range < BOT (in which case
 *            range = -low & (BOT - 1) first), emit the top byte of low and
 *            shift low and range left by 8. Four bytes of low end the stream.
 *            Decoding mirrors it with code = the first four bytes (big-endian).
 *            All arithmetic is modulo 2^32.
 */
#include <stdint.h>
#include <string.h>

#define CG_PROB_BITS 15u
#define CG_TOTAL (1u << CG_PROB_BITS)
#define CG_TOP (1u << 24)
#define CG_BOT (1u << 16)

/* cdf for one stream of n_tokens symbols read with stride `stride`. */
static void cdf_one(const uint8_t* sym, int64_t stride, int n_tokens, int max_bins,
                    uint16_t* cdf, int* out_of_range) {
  uint32_t hist[257];
  memset(hist, 0, sizeof(hist));
  for (int t = 0; t < n_tokens; ++t) {
    uint8_t s = sym[(int64_t)t * stride];
    if (s < max_bins) {
      hist[s]++;
    } else {
      *out_of_range = 1;
    }
  }
  uint64_t n = 0;
  for (int k = 0; k < max_bins; ++k) n += hist[k];
  uint64_t cum = 0;
  for (int k = 0; k <= max_bins; ++k) {
    uint64_t v;
    if (n > 0) {
      v = cum * (uint64_t)(CG_TOTAL - (uint32_t)max_bins) / n + (uint64_t)k;
    } else {
      v = (uint64_t)k * CG_TOTAL / (uint64_t)max_bins;
    }
    cdf[k] = (uint16_t)v;
    if (k < max_bins) cum += hist[k];
  }
}

/* calculate_cdf: sym [L, T, C] -> cdf [L, C, max_bins + 1]. Returns 1 if a
 * symbol was >= max_bins (it is left out of the counts), else 0. */
int oracle_calculate_cdf(const uint8_t* sym, int L, int T, int C, int max_bins, uint16_t* cdf) {
  int oor = 0;
  for (int l = 0; l < L; ++l) {
    for (int c = 0; c < C; ++c) {
      cdf_one(sym + (int64_t)l * T * C + c, C, T, max_bins,
              cdf + ((int64_t)l * C + c) * (max_bins + 1), &oor);
    }
  }
  return oor;
}

/* Encodes one stream; returns its length in bytes, or -1 if it does not fit
 * in `cap` bytes (the first `cap` bytes are still written). */
static int64_t encode_one(const uint16_t* cdf, const uint8_t* sym, int64_t stride,
                          int n_tokens, int max_bins, uint8_t* out, int64_t cap) {
  uint32_t low = 0, range = 0xFFFFFFFFu;
  int64_t pos = 0;
  int overflow = 0;
#define CG_EMIT(b)                 \
  do {                             \
    if (pos < cap) {               \
      out[pos] = (uint8_t)(b);     \
    } else {                       \
      overflow = 1;                \
    }                              \
    ++pos;                         \
  } while (0)
  for (int t = 0; t < n_tokens; ++t) {
    uint32_t s = sym[(int64_t)t * stride];
    if (s >= (uint32_t)max_bins) s = (uint32_t)max_bins - 1u; /* caller flags it */
    uint32_t lo = cdf[s], hi = cdf[s + 1];
    uint32_t r = range >> CG_PROB_BITS;
    low += lo * r;
    range = r * (hi - lo);
    for (;;) {
      if ((low ^ (low + range)) >= CG_TOP) {
        if (range >= CG_BOT) break;
        range = (0u - low) & (CG_BOT - 1u);
      }
      CG_EMIT(low >> 24);
      low <<= 8;
      range <<= 8;
    }
  }
  for (int i = 0; i < 4; ++i) {
    CG_EMIT(low >> 24);
    low <<= 8;
  }
#undef CG_EMIT
  return overflow ? -1 : pos;
}

/* encode: cdf [L, C, max_bins + 1], sym [L, T, C] -> out [L, C, cap],
 * lengths [L, C] (-1 for a stream that did not fit). Returns the number of
 * overflowing streams. */
int oracle_encode(const uint16_t* cdf, const uint8_t* sym, int L, int T, int C, int max_bins,
                  uint8_t* out, int64_t cap, int32_t* lengths) {
  int overflows = 0;
  for (int l = 0; l < L; ++l) {
    for (int c = 0; c < C; ++c) {
      const int64_t i = (int64_t)l * C + c;
      int64_t n = encode_one(cdf + i * (max_bins + 1), sym + (int64_t)l * T * C + c, C, T,
                             max_bins, out + i * cap, cap);
      if (n < 0) overflows++;
      lengths[i] = (int32_t)n;
    }
  }
  return overflows;
}

/* Decodes one stream of n_tokens symbols from in[0, len). Bytes past len
 * read as zero. */
static void decode_one(const uint16_t* cdf, const uint8_t* in, int64_t len, int n_tokens,
                       int max_bins, uint8_t* sym, int64_t stride) {
  int64_t pos = 0;
#define CG_NEXT() (pos < len ? in[pos++] : (pos++, 0u))
  uint32_t low = 0, range = 0xFFFFFFFFu, code = 0;
  for (int i = 0; i < 4; ++i) code = (code << 8) | CG_NEXT();
  for (int t = 0; t < n_tokens; ++t) {
    uint32_t r = range >> CG_PROB_BITS;
    uint32_t v = (code - low) / r;
    if (v >= CG_TOTAL) v = CG_TOTAL - 1u;
    /* largest s with cdf[s] <= v */
    int a = 0, b = max_bins; /* invariant: cdf[a] <= v < cdf[b] */
    while (b - a > 1) {
      int m = (a + b) >> 1;
      if (cdf[m] <= v) a = m; else b = m;
    }
    uint32_t lo = cdf[a], hi = cdf[a + 1];
    low += lo * r;
    range = r * (hi - lo);
    for (;;) {
      if ((low ^ (low + range)) >= CG_TOP) {
        if (range >= CG_BOT) break;
        range = (0u - low) & (CG_BOT - 1u);
      }
      code = (code << 8) | CG_NEXT();
      low <<= 8;
      range <<= 8;
    }
    sym[(int64_t)t * stride] = (uint8_t)a;
  }
#undef CG_NEXT
}

/* decode: bytestreams [L, C, cap] with lengths [L, C] -> sym [L, T, C]. */
void oracle_decode(const uint16_t* cdf, const uint8_t* streams, const int32_t* lengths, int L,
                   int T, int C, int max_bins, int64_t cap, uint8_t* sym) {
  for (int l = 0; l < L; ++l) {
    for (int c = 0; c < C; ++c) {
      const int64_t i = (int64_t)l * C + c;
      int64_t len = lengths[i] < 0 ? 0 : lengths[i];
      if (len > cap) len = cap;
      decode_one(cdf + i * (max_bins + 1), streams + i * cap, len, T, max_bins,
                 sym + (int64_t)l * T * C + c, C);
    }
  }
}

/* decode_prefsum: streams concatenated; stream i spans
 * [i ? ends[i-1] : 0, ends[i]). */
void oracle_decode_prefsum(const uint16_t* cdf, const uint8_t* streams, const int64_t* ends,
                           int L, int T, int C, int max_bins, uint8_t* sym) {
  for (int l = 0; l < L; ++l) {
    for (int c = 0; c < C; ++c) {
      const int64_t i = (int64_t)l * C + c;
      const int64_t start = i ? ends[i - 1] : 0;
      decode_one(cdf + i * (max_bins + 1), streams + start, ends[i] - start, T, max_bins,
                 sym + (int64_t)l * T * C + c, C);
    }
  }
}
