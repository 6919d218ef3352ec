// pos_kernels.cu -- fused K re-rotation for CacheBlend (rotary_embedding_k_fused).
//
// The reference exports rotary_embedding_k_fused (csrc/pybind.cpp:25) but its
// body raises NotImplementedError (csrc/pos_kernels.cpp:7-14). Its caller
// (lmcache_ascend/v1/blend/positional_encoding.py:57-77) moves cached K rows
// from the positions they were encoded at to new positions; the unfused
// equivalent there (DummyFusedRope, :80-101) undoes the rotary embedding at
// the old positions and applies it at the new ones. This kernel does both in
// one pass: for each rotated pair (x1, x2) with angles a (old) and b (new),
//   (x1, x2) <- R(b - a) (x1, x2),
//   cos(b - a) = cos b cos a + sin b sin a,  sin(b - a) = sin b cos a - cos b sin a,
// in fp32, rounding once to the key's type. Pairs follow the rotary layouts
// of the cos/sin cache [max_position, rot_dim] = [cos | sin]: neox style pairs
// dims (i, i + rot_dim/2), GPT-J style pairs (2i, 2i + 1); dims at and beyond
// rot_dim are left unchanged.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "lmcache_b200.h"

namespace lmcb {
namespace {

constexpr int kRopeThreads = 128;

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// The rotation of one pair, with every rounding explicit: products by
// __fmul_rn and sums by __fmaf_rn leave the compiler no multiply-add to
// contract on its own, so the three kernels below compute bit-identical
// results whatever their instruction schedule.
//   c = cos(b - a) = cos b cos a + sin b sin a,  s = sin(b - a) = sin b cos a - cos b sin a
//   y1 = x1 c - x2 s,                             y2 = x2 c + x1 s
__device__ __forceinline__ void angle_diff(float cos_a, float sin_a, float cos_b, float sin_b,
                                           float& c, float& s) {
  c = __fmaf_rn(cos_b, cos_a, __fmul_rn(sin_b, sin_a));
  s = __fmaf_rn(sin_b, cos_a, -__fmul_rn(cos_b, sin_a));
}

__device__ __forceinline__ void rotate_pair(float x1, float x2, float c, float s, float& y1,
                                            float& y2) {
  y1 = __fmaf_rn(x1, c, -__fmul_rn(x2, s));
  y2 = __fmaf_rn(x2, c, __fmul_rn(x1, s));
}

struct RopeParams {
  const void* old_pos;
  const void* new_pos;
  void* key;
  const void* cache;
  int64_t num_tokens;
  int64_t num_heads;
  int64_t head_size;
  int64_t token_stride;  // elements between consecutive tokens of `key`
  int64_t rot_dim;
  int64_t max_position;
  int is_neox;
  unsigned int* status;
  FastDiv div_half;  // pair index -> head: by rot_dim / 2 (rot_dim / 4 in the vec2 kernel)
};

// A CTA walks tokens in a grid-stride loop (one launch of up to
// kRopeBlocksPerSm CTAs per SM, instead of a tiny CTA per token); within a
// token, thread q handles rotated pairs q, q + blockDim.x, ... with 32-bit
// pair arithmetic (pairs per token = num_heads * rot_dim / 2 < 2^31, checked
// by the entry point).
template <typename KeyT, typename CacheT, typename PosT>
__global__ void __launch_bounds__(kRopeThreads) rope_k_fused_kernel(const RopeParams p) {
  const int half = static_cast<int>(p.rot_dim / 2);
  const int pairs = static_cast<int>(p.num_heads) * half;
  for (int64_t token = blockIdx.x; token < p.num_tokens; token += gridDim.x) {
    const int64_t a = static_cast<int64_t>(static_cast<const PosT*>(p.old_pos)[token]);
    const int64_t b = static_cast<int64_t>(static_cast<const PosT*>(p.new_pos)[token]);
    if (a < 0 || a >= p.max_position || b < 0 || b >= p.max_position) {
      if (threadIdx.x == 0) raise_flag(p.status, LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE);
      continue;  // uniform across the CTA
    }
    const CacheT* ca = static_cast<const CacheT*>(p.cache) + a * p.rot_dim;
    const CacheT* cb = static_cast<const CacheT*>(p.cache) + b * p.rot_dim;
    KeyT* k = static_cast<KeyT*>(p.key) + token * p.token_stride;
    for (int q = threadIdx.x; q < pairs; q += blockDim.x) {
      const int h = static_cast<int>(p.div_half.div(static_cast<uint32_t>(q)));
      const int i = q - h * half;
      const float cos_a = to_f(ca[i]), sin_a = to_f(ca[half + i]);
      const float cos_b = to_f(cb[i]), sin_b = to_f(cb[half + i]);
      float c, s;
      angle_diff(cos_a, sin_a, cos_b, sin_b, c, s);
      KeyT* row = k + static_cast<int64_t>(h) * p.head_size;
      const int i1 = p.is_neox ? i : 2 * i;
      const int i2 = p.is_neox ? i + half : 2 * i + 1;
      float y1, y2;
      rotate_pair(to_f(row[i1]), to_f(row[i2]), c, s, y1, y2);
      row[i1] = from_f<KeyT>(y1);
      row[i2] = from_f<KeyT>(y2);
    }
  }
}

// Same rotation, two adjacent pairs per step with 2-element vector accesses:
// neox pairs (i, i + half) and (i + 1, i + 1 + half), GPT-J pairs (2i, 2i + 1)
// and (2i + 2, 2i + 3), i even; cos/sin of both pairs come in one 2-element
// load each. The per-pair arithmetic is that of rope_k_fused_kernel, so the
// results are identical. Launched only when the host has checked that every
// access is aligned to its vector width (rope_vec_ok).
template <typename T, int N>
struct alignas(sizeof(T) * N) RopeVec {
  T v[N];
};

template <typename KeyT, typename CacheT, typename PosT>
__global__ void __launch_bounds__(kRopeThreads) rope_k_fused_vec2_kernel(const RopeParams p) {
  const int half = static_cast<int>(p.rot_dim / 2);
  const int quads = static_cast<int>(p.num_heads) * (half / 2);  // pair pairs per token
  const FastDiv& div_q = p.div_half;  // here: division by half / 2
  for (int64_t token = blockIdx.x; token < p.num_tokens; token += gridDim.x) {
    const int64_t a = static_cast<int64_t>(static_cast<const PosT*>(p.old_pos)[token]);
    const int64_t b = static_cast<int64_t>(static_cast<const PosT*>(p.new_pos)[token]);
    if (a < 0 || a >= p.max_position || b < 0 || b >= p.max_position) {
      if (threadIdx.x == 0) raise_flag(p.status, LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE);
      continue;  // uniform across the CTA
    }
    const CacheT* ca = static_cast<const CacheT*>(p.cache) + a * p.rot_dim;
    const CacheT* cb = static_cast<const CacheT*>(p.cache) + b * p.rot_dim;
    KeyT* k = static_cast<KeyT*>(p.key) + token * p.token_stride;
    for (int q = threadIdx.x; q < quads; q += blockDim.x) {
      const int h = static_cast<int>(div_q.div(static_cast<uint32_t>(q)));
      const int i = 2 * (q - h * (half / 2));
      using C2 = RopeVec<CacheT, 2>;
      const C2 cos_a = *reinterpret_cast<const C2*>(ca + i);
      const C2 sin_a = *reinterpret_cast<const C2*>(ca + half + i);
      const C2 cos_b = *reinterpret_cast<const C2*>(cb + i);
      const C2 sin_b = *reinterpret_cast<const C2*>(cb + half + i);
      float c[2], sn[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float ca_j = to_f(cos_a.v[j]), sa_j = to_f(sin_a.v[j]);
        const float cb_j = to_f(cos_b.v[j]), sb_j = to_f(sin_b.v[j]);
        angle_diff(ca_j, sa_j, cb_j, sb_j, c[j], sn[j]);
      }
      KeyT* row = k + static_cast<int64_t>(h) * p.head_size;
      if (p.is_neox) {
        using K2 = RopeVec<KeyT, 2>;
        K2* p1 = reinterpret_cast<K2*>(row + i);
        K2* p2 = reinterpret_cast<K2*>(row + half + i);
        K2 x1 = *p1, x2 = *p2;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float y1, y2;
          rotate_pair(to_f(x1.v[j]), to_f(x2.v[j]), c[j], sn[j], y1, y2);
          x1.v[j] = from_f<KeyT>(y1);
          x2.v[j] = from_f<KeyT>(y2);
        }
        *p1 = x1;
        *p2 = x2;
      } else {
        using K4 = RopeVec<KeyT, 4>;
        K4* px = reinterpret_cast<K4*>(row + 2 * i);
        K4 x = *px;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float y1, y2;
          rotate_pair(to_f(x.v[2 * j]), to_f(x.v[2 * j + 1]), c[j], sn[j], y1, y2);
          x.v[2 * j] = from_f<KeyT>(y1);
          x.v[2 * j + 1] = from_f<KeyT>(y2);
        }
        *px = x;
      }
    }
  }
}

// Same rotation with 16-byte key vectors, the angles computed once per token
// for all heads. An item is (token, vector v): v selects E = 16 /
// sizeof(KeyT) key elements -- for neox the E dims at v * E of the first
// rotary half, paired with the E dims at half + v * E; for GPT-J E / 2
// adjacent pairs at v * E -- and the item rotates that vector of every head.
// The cos/sin runs the vector needs are loaded once per item and the angle
// differences computed once, not once per head (heads of a token share its
// positions): cache traffic per token is one pass over its two cache rows
// against two passes over its key rows. Items are numbered token-major with
// v fastest, so the threads of a warp read and write whole 128-byte segments
// of each head. A thread loads eight key vectors (kRopeHeadsInFlight heads,
// half as many for neox, whose heads take two vectors each) and, for the
// first group, the positions before it uses any, then rotates and stores
// them. The per-pair arithmetic is angle_diff / rotate_pair, as in the
// other kernels, so the results are identical. Launched only when the host
// has checked alignment and that the item count is below 2^31 (rope_v16_ok).
constexpr int kRopeV16Threads = 256;
constexpr int kRopeHeadsInFlight = 8;

template <typename T>
struct alignas(16) Vec16 {
  T v[16 / sizeof(T)];
};

// N consecutive cache values at `src` as floats: 16-byte loads when the run
// is at least 16 bytes (src 16-byte aligned), else one load of the run.
template <typename CacheT, int N>
__device__ __forceinline__ void load_cache_run(const CacheT* src, float (&out)[N]) {
  constexpr int kBytes = N * static_cast<int>(sizeof(CacheT));
  if constexpr (kBytes >= 16) {
    constexpr int kPer = 16 / sizeof(CacheT);
#pragma unroll
    for (int c = 0; c < N / kPer; ++c) {
      const Vec16<CacheT> piece = reinterpret_cast<const Vec16<CacheT>*>(src)[c];
#pragma unroll
      for (int j = 0; j < kPer; ++j) out[c * kPer + j] = to_f(piece.v[j]);
    }
  } else {
    const RopeVec<CacheT, N> piece = *reinterpret_cast<const RopeVec<CacheT, N>*>(src);
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = to_f(piece.v[j]);
  }
}

template <typename KeyT, typename CacheT, typename PosT, bool kNeox>
__global__ void __launch_bounds__(kRopeV16Threads, 2)
rope_k_fused_v16_kernel(const RopeParams p, const uint32_t num_items, const FastDiv div_vec) {
  constexpr int E = 16 / sizeof(KeyT);   // key elements per vector
  constexpr int NP = kNeox ? E : E / 2;  // pairs per vector
  constexpr int HF = kNeox ? kRopeHeadsInFlight / 2 : kRopeHeadsInFlight;  // vectors in flight: 8
  using KV = Vec16<KeyT>;
  const int half = static_cast<int>(p.rot_dim / 2);
  const int heads = static_cast<int>(p.num_heads);
  for (uint32_t item = blockIdx.x * kRopeV16Threads + threadIdx.x; item < num_items;
       item += gridDim.x * kRopeV16Threads) {
    const uint32_t t = div_vec.div(item);
    const int v = static_cast<int>(item - t * div_vec.d);
    const int e0 = v * E;                 // first key element of the vector
    const int col = kNeox ? e0 : e0 / 2;  // its first cache column (pair index)
    KeyT* row0 = static_cast<KeyT*>(p.key) + static_cast<int64_t>(t) * p.token_stride + e0;
    float c[NP], sn[NP];
    for (int h0 = 0; h0 < heads; h0 += HF) {
      KV x1[HF], x2[HF];
      // 1. this group's key vectors (and, for the first group, the positions)
#pragma unroll
      for (int hh = 0; hh < HF; ++hh) {
        if (h0 + hh < heads) {
          const KeyT* r = row0 + static_cast<int64_t>(h0 + hh) * p.head_size;
          x1[hh] = *reinterpret_cast<const KV*>(r);
          if constexpr (kNeox) x2[hh] = *reinterpret_cast<const KV*>(r + half);
        }
      }
      if (h0 == 0) {
        const int64_t a = static_cast<int64_t>(static_cast<const PosT*>(p.old_pos)[t]);
        const int64_t b = static_cast<int64_t>(static_cast<const PosT*>(p.new_pos)[t]);
        if (a < 0 || a >= p.max_position || b < 0 || b >= p.max_position) {
          if (v == 0) raise_flag(p.status, LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE);
          break;  // the token is left unchanged
        }
        const CacheT* ca = static_cast<const CacheT*>(p.cache) + a * p.rot_dim + col;
        const CacheT* cb = static_cast<const CacheT*>(p.cache) + b * p.rot_dim + col;
        float cos_a[NP], sin_a[NP], cos_b[NP], sin_b[NP];
        load_cache_run<CacheT, NP>(ca, cos_a);
        load_cache_run<CacheT, NP>(ca + half, sin_a);
        load_cache_run<CacheT, NP>(cb, cos_b);
        load_cache_run<CacheT, NP>(cb + half, sin_b);
#pragma unroll
        for (int j = 0; j < NP; ++j) angle_diff(cos_a[j], sin_a[j], cos_b[j], sin_b[j], c[j], sn[j]);
      }
      // 2. rotate and store
#pragma unroll
      for (int hh = 0; hh < HF; ++hh) {
        if (h0 + hh >= heads) continue;
        KeyT* r = row0 + static_cast<int64_t>(h0 + hh) * p.head_size;
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          float y1, y2;
          if constexpr (kNeox) {
            rotate_pair(to_f(x1[hh].v[j]), to_f(x2[hh].v[j]), c[j], sn[j], y1, y2);
            x1[hh].v[j] = from_f<KeyT>(y1);
            x2[hh].v[j] = from_f<KeyT>(y2);
          } else {
            rotate_pair(to_f(x1[hh].v[2 * j]), to_f(x1[hh].v[2 * j + 1]), c[j], sn[j], y1, y2);
            x1[hh].v[2 * j] = from_f<KeyT>(y1);
            x1[hh].v[2 * j + 1] = from_f<KeyT>(y2);
          }
        }
        *reinterpret_cast<KV*>(r) = x1[hh];
        if constexpr (kNeox) *reinterpret_cast<KV*>(r + half) = x2[hh];
      }
    }
  }
}

// True when every access of rope_k_fused_v16_kernel is aligned and its item
// count fits: E = 16 / sizeof(KeyT); neox needs rot_dim a multiple of 2E,
// GPT-J of E; the key base, token stride and head size multiples of 16 bytes;
// the cache base 16-byte aligned.
template <typename KeyT, typename CacheT>
bool rope_v16_ok(const RopeParams& p, uint32_t* vecs_per_head) {
  constexpr int64_t E = 16 / sizeof(KeyT);
  const int64_t unit = p.is_neox ? 2 * E : E;
  if (p.rot_dim % unit != 0) return false;
  if (reinterpret_cast<uintptr_t>(p.key) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(p.cache) % 16 != 0) {
    return false;
  }
  if ((p.token_stride * static_cast<int64_t>(sizeof(KeyT))) % 16 != 0 ||
      (p.head_size * static_cast<int64_t>(sizeof(KeyT))) % 16 != 0) {
    return false;
  }
  const int64_t vph = p.is_neox ? p.rot_dim / 2 / E : p.rot_dim / E;
  if (p.num_tokens * vph >= (int64_t(1) << 31)) return false;
  *vecs_per_head = static_cast<uint32_t>(vph);
  return true;
}

constexpr int kRopeBlocksPerSm = 16;

// True when every access of rope_k_fused_vec2_kernel is aligned: rot_dim a
// multiple of 4 (so i and half + i are even), the key base, token stride and
// head size multiples of the key vector (2 elements neox, 4 GPT-J) and the
// cache base a multiple of 2 cache elements.
template <typename KeyT, typename CacheT>
bool rope_vec_ok(const RopeParams& p) {
  if (p.rot_dim % 4 != 0) return false;
  const int64_t kv = p.is_neox ? 2 : 4;
  const uint64_t kbytes = static_cast<uint64_t>(kv) * sizeof(KeyT);
  if (reinterpret_cast<uintptr_t>(p.key) % kbytes != 0) return false;
  if ((p.token_stride % kv) != 0 || (p.head_size % kv) != 0) return false;
  return reinterpret_cast<uintptr_t>(p.cache) % (2 * sizeof(CacheT)) == 0;
}

template <typename KeyT, typename CacheT, typename PosT>
void launch_rope_v16(const RopeParams& p, uint32_t vph, cudaStream_t stream) {
  const uint32_t items = static_cast<uint32_t>(p.num_tokens) * vph;
  const int64_t blocks = (static_cast<int64_t>(items) + kRopeV16Threads - 1) / kRopeV16Threads;
  const int64_t max_grid = static_cast<int64_t>(current_sm_count()) * 2;
  const dim3 grid(static_cast<unsigned>(blocks < max_grid ? blocks : max_grid));
  const FastDiv div_vec(vph);
  if (p.is_neox) {
    rope_k_fused_v16_kernel<KeyT, CacheT, PosT, true>
        <<<grid, kRopeV16Threads, 0, stream>>>(p, items, div_vec);
  } else {
    rope_k_fused_v16_kernel<KeyT, CacheT, PosT, false>
        <<<grid, kRopeV16Threads, 0, stream>>>(p, items, div_vec);
  }
}

template <typename KeyT, typename CacheT>
cudaError_t launch_rope_pos(RopeParams p, int pos_type, cudaStream_t stream) {
  const int64_t max_grid = static_cast<int64_t>(current_sm_count()) * kRopeBlocksPerSm;
  const dim3 grid(static_cast<unsigned>(p.num_tokens < max_grid ? p.num_tokens : max_grid));
  uint32_t vph = 0;
  const char* force = std::getenv("LMCB_ROPE_KERNEL");  // "vec2" or "pair": tests, tuning
  const bool allow_v16 = force == nullptr || std::strcmp(force, "v16") == 0;
  const bool allow_vec2 = force == nullptr || std::strcmp(force, "pair") != 0;
  if (allow_v16 && rope_v16_ok<KeyT, CacheT>(p, &vph)) {
    if (pos_type == LMCB_DTYPE_INT64) {
      launch_rope_v16<KeyT, CacheT, int64_t>(p, vph, stream);
    } else {
      launch_rope_v16<KeyT, CacheT, int32_t>(p, vph, stream);
    }
  } else if (allow_vec2 && rope_vec_ok<KeyT, CacheT>(p)) {
    p.div_half = FastDiv(static_cast<uint32_t>(p.rot_dim / 4));
    if (pos_type == LMCB_DTYPE_INT64) {
      rope_k_fused_vec2_kernel<KeyT, CacheT, int64_t><<<grid, kRopeThreads, 0, stream>>>(p);
    } else {
      rope_k_fused_vec2_kernel<KeyT, CacheT, int32_t><<<grid, kRopeThreads, 0, stream>>>(p);
    }
  } else if (pos_type == LMCB_DTYPE_INT64) {
    rope_k_fused_kernel<KeyT, CacheT, int64_t><<<grid, kRopeThreads, 0, stream>>>(p);
  } else {
    rope_k_fused_kernel<KeyT, CacheT, int32_t><<<grid, kRopeThreads, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

template <typename KeyT>
cudaError_t launch_rope_cache(const RopeParams& p, int cache_type, int pos_type,
                              cudaStream_t stream) {
  switch (cache_type) {
    case LMCB_DTYPE_FP32: return launch_rope_pos<KeyT, float>(p, pos_type, stream);
    case LMCB_DTYPE_BF16: return launch_rope_pos<KeyT, __nv_bfloat16>(p, pos_type, stream);
    default: return launch_rope_pos<KeyT, __half>(p, pos_type, stream);
  }
}

bool float_type(int t) {
  return t == LMCB_DTYPE_FP32 || t == LMCB_DTYPE_BF16 || t == LMCB_DTYPE_FP16;
}

}  // namespace
}  // namespace lmcb

extern "C" {

int lmcb_rotary_embedding_k_fused(const void* oldPositions, const void* newPositions, int posType,
                                  void* key, int keyType, int64_t numTokens, int64_t numHeads,
                                  int64_t headSize, int64_t keyTokenStride,
                                  const void* cosSinCache, int cacheType, int64_t rotDim,
                                  int64_t maxPosition, int isNeox, void* stream) {
  lmcb::clear_error();
  const char* who = "rotary_embedding_k_fused";
  if (!lmcb::float_type(keyType) || !lmcb::float_type(cacheType)) {
    return lmcb::fail(LMCB_ERR_UNSUPPORTED_DTYPE, std::string(who) + ": ScalarType not supported.");
  }
  if (posType != LMCB_DTYPE_INT64 && posType != LMCB_DTYPE_INT32) {
    return lmcb::fail(LMCB_ERR_UNSUPPORTED_DTYPE,
                      std::string(who) + ": positions must be int64 or int32.");
  }
  if (numTokens < 0 || numHeads < 0 || headSize <= 0 || rotDim <= 0 || rotDim % 2 != 0 ||
      rotDim > headSize || maxPosition <= 0 || keyTokenStride < numHeads * headSize ||
      numTokens > 0x7fffffff || numHeads * (rotDim / 2) > 0x7fffffff) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      std::string(who) + ": invalid shape (rot_dim must be even and <= head_size).");
  }
  if (numTokens == 0 || numHeads == 0) return LMCB_OK;
  if (oldPositions == nullptr || newPositions == nullptr || key == nullptr ||
      cosSinCache == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL pointer.");
  }
  lmcb::RopeParams p;
  p.old_pos = oldPositions;
  p.new_pos = newPositions;
  p.key = key;
  p.cache = cosSinCache;
  p.num_tokens = numTokens;
  p.num_heads = numHeads;
  p.head_size = headSize;
  p.token_stride = keyTokenStride;
  p.rot_dim = rotDim;
  p.max_position = maxPosition;
  p.is_neox = isNeox ? 1 : 0;
  p.div_half = lmcb::FastDiv(static_cast<uint32_t>(rotDim / 2));
  p.status = lmcb::device_status_ptr();
  if (p.status == nullptr) return LMCB_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  switch (keyType) {
    case LMCB_DTYPE_FP32: err = lmcb::launch_rope_cache<float>(p, cacheType, posType, s); break;
    case LMCB_DTYPE_BF16:
      err = lmcb::launch_rope_cache<__nv_bfloat16>(p, cacheType, posType, s);
      break;
    default: err = lmcb::launch_rope_cache<__half>(p, cacheType, posType, s); break;
  }
  if (err != cudaSuccess) return lmcb::cuda_fail(err, who);
  return LMCB_OK;
}

}  // extern "C"
