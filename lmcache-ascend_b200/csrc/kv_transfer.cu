// kv_transfer.cu -- paged KV-cache <-> LMCache object row transfer for sm_100a.
//
// Two kernels serve every transfer entry point of the reference's c_ops
// surface (csrc/mem_kernels.cpp). Both copy "rows" (one token's hidden_dims
// elements of K, V or the MLA latent) between vLLM-style paged buffers,
// addressed through slot ids, and dense LMCache objects. The entry points
// only differ in how a (kv, layer, slot) triple becomes a paged-side address
// and a (kv, layer, token) triple becomes an LMCache-side address (PagedMode).
//
//   transfer_rows_bulk_kernel  one-warp CTAs stream contiguous row ranges
//       through a shared-memory ring with bulk (TMA engine) copies, merging
//       rows that are contiguous on both sides; device objects only. Used
//       for launches under kVectorMinTraffic whose copies can merge or whose
//       rows are at least kBulkMinUnmergedRow bytes (launch_transfer).
//   transfer_rows_kernel       vectorised loads and stores, below; every
//       other case, pinned-host (zero-copy) objects included.
//
// transfer_rows_kernel's work decomposition: a tile is (kv, layer, TILE
// consecutive tokens). A CTA takes tiles in a grid-stride loop. For each tile
// it
//   1. resolves the tile's rows once: slot id -> paged address, token ->
//      LMCache address, dropping skipped rows (slot < 0 or out of range) and
//      compacting the rest into shared memory;
//   2. moves the surviving rows as a flat array of VEC-byte vectors, UNROLL
//      independent vectors per thread in flight (all loads, then all stores),
//      so consecutive threads touch consecutive 16-byte words of a row and
//      every warp access is fully coalesced, whatever the row length.
// Rows whose addresses are not VEC-aligned (possible only through the device
// pointer array, which the host cannot inspect) are copied byte-wise.
//
// The same kernel serves HBM and pinned-host (device-mapped, zero-copy)
// LMCache objects; for host objects every row crosses PCIe exactly once.

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "lmcache_b200.h"

namespace lmcb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxTileRows = 128;
// Vectors in flight per thread (all loads, then all stores; a template
// parameter of the vectorised kernel). A launch whose tiles all fit one wave
// of CTAs takes 8 (8 x 256 threads x 16 B = 32 KB: a whole target tile in one
// pass), longer launches 4. Measured on B200: a c5 single-layer batched
// launch (256 tiles) 5.7 us with 4, 5.2 us with 8; a whole c2 request in one
// launch (32,768 tiles) 0.94 of the copy roofline with 4, 0.91 with 8.
constexpr int kUnrollShort = 8;
constexpr int kUnrollLong = 4;
constexpr int kTargetTileBytes = 32 * 1024;
constexpr int kMinTilesPerSm = 1;

// How row addresses are formed.
//   kPtrArray: paged base = ptrs_k[layer] (kv == 0) or ptrs_v[layer]
//              (kv == 1), plus kv * page_kv_offset; one LMCache object.
//   kDirect:   paged base = base_k (kv == 0) or base_v (kv == 1); one object.
//   kBatched:  paged side as kPtrArray; many LMCache objects, located through
//              the launch's ObjectTable.
//   kBatchedDirect: paged side as kDirect (one layer); many objects.
enum PagedMode { kPtrArray = 0, kDirect = 1, kBatched = 2, kBatchedDirect = 3 };

__host__ __device__ constexpr bool paged_direct(int mode) {
  return mode == kDirect || mode == kBatchedDirect;
}
__host__ __device__ constexpr bool batched_mode(int mode) {
  return mode == kBatched || mode == kBatchedDirect;
}

struct TransferParams {
  // LMCache side: row(kv, layer, t) = lmc + kv*lmc_kv_stride
  //                                 + layer*lmc_layer_stride + t*lmc_token_stride
  uint8_t* lmc;
  int64_t lmc_kv_stride;
  int64_t lmc_layer_stride;
  int64_t lmc_token_stride;
  // Paged side: row(kv, layer, slot) = base(kv, layer) + slot * paged_row_stride
  const uint64_t* ptrs_k;
  const uint64_t* ptrs_v;
  uint8_t* base_k;
  uint8_t* base_v;
  int64_t page_kv_offset;
  int64_t paged_row_stride;
  int64_t num_paged_rows;  // slot bound; <= 0 means unchecked
  // Slots and shape.
  const void* slots;
  int32_t num_tokens;
  int32_t num_layers;
  int32_t num_kv;
  int32_t tile_rows;       // tokens per tile
  int32_t tiles_per_seq;   // ceil(num_tokens / tile_rows)
  int64_t num_tiles;       // num_kv * num_layers * tiles_per_seq
  int64_t row_bytes;
  FastDiv row_vecs;        // row_bytes / VEC
  int32_t page2L;          // 1: paged -> LMCache, 0: LMCache -> paged
  unsigned int* status;
  // Vector kernel, single object, page2L only: device-mapped alias of the
  // final destination object (same layout as lmc); rows with a skipped slot
  // are copied from it instead of being left untouched. Null otherwise.
  const uint8_t* fallback;
  // Batched modes only: the number of objects in this launch's ObjectTable.
  int32_t num_objects;
  // Object layout: 0 = [kv, num_layers, T_i, hidden];
  //                1 = token-major [T_i, kv, hidden] (single layer).
  int32_t obj_token_major;
  // Vector kernel: 1 when this is a retrieve from device objects, whose rows
  // each CTA prefetches into L2 for its first tile before
  // griddepcontrol.wait (their addresses are parameters, not inputs).
  int32_t prefetch_lmc;
};

// The object table of a batched launch travels in the kernel parameters
// (constant bank, __grid_constant__), so a launch reads no table from global
// memory, needs no host-to-device copy before it and can be captured in a
// CUDA graph. Tokens t are numbered across the launch's objects: object i
// holds t in [offsets[i], offsets[i+1]), is laid out [kv, num_layers, T_i,
// hidden] (or token-major) at ptrs[i], and takes its slot ids from
// slots[slot_starts[i] + (t - offsets[i])]. The host splits batches of more
// than kMaxObjects objects into several launches (5 KB of parameters each).
constexpr int kMaxObjects = 255;

template <bool kBatched>
struct ObjectTable {};  // non-batched launches carry no table

template <>
struct ObjectTable<true> {
  uint64_t ptrs[kMaxObjects];        // base addresses (0 for empty objects)
  int64_t slot_starts[kMaxObjects];  // index of each object's first slot id
  int32_t offsets[kMaxObjects + 1];  // token prefix sums, offsets[0] = 0
};

// A row finds its object by a binary search over the token offsets, about
// log2(num_objects) dependent probes. Each CTA first copies the offsets into
// shared memory (1 KB), so the probes are shared-memory loads instead of
// divergent constant-bank reads; pointers and slot starts, read once per row
// and uniform across most warps, are read from the parameters.
__device__ __forceinline__ void stage_obj_offsets(const TransferParams& p,
                                                  const ObjectTable<true>& tab, int32_t* s,
                                                  int tid, int nthreads) {
  for (int i = tid; i <= p.num_objects; i += nthreads) s[i] = tab.offsets[i];
}

// LMCache-side row address of (kv, layer, t) and the index of t's slot id.
// s_offsets: the staged token offsets of a batched launch.
template <int MODE>
__device__ __forceinline__ uint8_t* lmc_row(const TransferParams& p,
                                            const ObjectTable<batched_mode(MODE)>& tab,
                                            const int32_t* s_offsets, int kv, int layer, int t,
                                            int64_t* slot_index) {
  if constexpr (batched_mode(MODE)) {
    // Last object whose first token is <= t (empty objects are skipped over).
    int lo = 0, hi = p.num_objects;  // offsets[lo] <= t < offsets[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_offsets[mid] <= t) lo = mid; else hi = mid;
    }
    const int64_t first = s_offsets[lo];
    const int64_t count = s_offsets[lo + 1] - first;
    const int64_t j = t - first;
    *slot_index = tab.slot_starts[lo] + j;
    const int64_t row = p.obj_token_major
                            ? j * p.num_kv + kv
                            : (static_cast<int64_t>(kv) * p.num_layers + layer) * count + j;
    return reinterpret_cast<uint8_t*>(tab.ptrs[lo]) + row * p.row_bytes;
  } else {
    (void)tab;
    (void)s_offsets;
    *slot_index = t;
    return p.lmc + kv * p.lmc_kv_stride + layer * p.lmc_layer_stride +
           static_cast<int64_t>(t) * p.lmc_token_stride;
  }
}

template <int VEC>
struct VecType;
template <> struct VecType<16> { using T = uint4; };
template <> struct VecType<8> { using T = uint2; };
template <> struct VecType<4> { using T = uint32_t; };
template <> struct VecType<2> { using T = uint16_t; };

// Programmatic dependent launch: wait for the preceding kernel in the stream
// (and the visibility of its writes) before touching global memory, and let
// the next kernel be scheduled while this one runs. Both are no-ops when the
// launch carries no programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename SlotT, int VEC, int MODE, int kUnroll>
__global__ void __launch_bounds__(kThreads)
transfer_rows_kernel(const TransferParams p,
                     const __grid_constant__ ObjectTable<batched_mode(MODE)> tab) {
  using V = typename VecType<VEC>::T;
  __shared__ const uint8_t* s_src[kMaxTileRows];
  __shared__ uint8_t* s_dst[kMaxTileRows];
  __shared__ int s_warp_count[kMaxTileRows / 32];
  __shared__ int32_t s_objoff[batched_mode(MODE) ? kMaxObjects + 1 : 1];

  const SlotT* __restrict__ slots = static_cast<const SlotT*>(p.slots);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  // The object table's offsets come from the parameters: staged before the
  // wait, like the retrieve prefetch below.
  const int32_t* obj_offsets = s_objoff;
  if constexpr (batched_mode(MODE)) {
    stage_obj_offsets(p, tab, s_objoff, tid, kThreads);
    __syncthreads();
  }
  // A retrieve reads object rows whose addresses come from the parameters
  // (and the staged offsets): the CTA's first tile of them is prefetched into
  // L2, 128-byte line by line, before the wait. A hint: if the previous kernel
  // is still writing those lines, its writes land in L2, where the loads
  // after the wait read them.
  if (p.prefetch_lmc && blockIdx.x < p.num_tiles) {
    const int64_t seq = blockIdx.x / p.tiles_per_seq;
    const int ttile = static_cast<int>(blockIdx.x - seq * p.tiles_per_seq);
    const int kv = static_cast<int>(seq / p.num_layers);
    const int layer = static_cast<int>(seq - static_cast<int64_t>(kv) * p.num_layers);
    const int t0 = ttile * p.tile_rows;
    const int n_tile = min(p.tile_rows, p.num_tokens - t0);
    const int lines = static_cast<int>((p.row_bytes + 127) / 128);
    for (int i = tid; i < n_tile * lines; i += kThreads) {
      const int r = i / lines;
      int64_t slot_index;
      const uint8_t* row = lmc_row<MODE>(p, tab, obj_offsets, kv, layer, t0 + r, &slot_index);
      prefetch_l2(row + static_cast<int64_t>(i - r * lines) * 128);
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  for (int64_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
    // tile -> (kv, layer, token range); token tiles vary fastest so
    // neighbouring CTAs write neighbouring LMCache memory.
    const int64_t seq = tile / p.tiles_per_seq;
    const int ttile = static_cast<int>(tile - seq * p.tiles_per_seq);
    const int kv = static_cast<int>(seq / p.num_layers);
    const int layer = static_cast<int>(seq - static_cast<int64_t>(kv) * p.num_layers);
    const int t0 = ttile * p.tile_rows;
    const int n_tile = min(p.tile_rows, p.num_tokens - t0);

    // ---- 1. resolve and compact the tile's rows -------------------------
    // Thread r (< n_tile <= kMaxTileRows) resolves token t0 + r.
    bool valid = false;
    bool misaligned = false;
    const uint8_t* src = nullptr;
    uint8_t* dst = nullptr;
    if (tid < n_tile) {
      const int t = t0 + tid;
      int64_t slot_index;
      uint8_t* lmc = lmc_row<MODE>(p, tab, obj_offsets, kv, layer, t, &slot_index);
      const int64_t slot = static_cast<int64_t>(slots[slot_index]);
      valid = slot >= 0;
      if (valid && p.num_paged_rows > 0 && slot >= p.num_paged_rows) {
        valid = false;
        raise_flag(p.status, LMCB_DEVICE_FLAG_SLOT_OUT_OF_RANGE);
      }
      if (valid) {
        uint8_t* paged;
        if (!paged_direct(MODE)) {
          const uint64_t* arr = kv == 0 ? p.ptrs_k : p.ptrs_v;
          paged = reinterpret_cast<uint8_t*>(arr[layer]) + kv * p.page_kv_offset;
        } else {
          paged = kv == 0 ? p.base_k : p.base_v;
        }
        paged += slot * p.paged_row_stride;
        if (p.page2L) {
          src = paged;
          dst = lmc;
        } else {
          src = lmc;
          dst = paged;
        }
        misaligned = ((reinterpret_cast<uintptr_t>(src) |
                       reinterpret_cast<uintptr_t>(dst)) & (VEC - 1)) != 0;
      } else if (p.fallback != nullptr && p.page2L) {
        // Staged store: a skipped row of the staging copy takes the row the
        // destination object already holds, so the copy back leaves it as is.
        src = p.fallback + (lmc - p.lmc);
        dst = lmc;
        valid = true;
        misaligned = ((reinterpret_cast<uintptr_t>(src) |
                       reinterpret_cast<uintptr_t>(dst)) & (VEC - 1)) != 0;
      }
    }
    const unsigned ballot = __ballot_sync(0xffffffffu, valid);
    if (lane == 0 && warp < kMaxTileRows / 32) s_warp_count[warp] = __popc(ballot);
    const bool mis = __syncthreads_or(misaligned) != 0;  // also publishes the counts
    if (valid) {
      int pos = __popc(ballot & ((1u << lane) - 1u));
      for (int w = 0; w < warp; ++w) pos += s_warp_count[w];
      s_src[pos] = src;
      s_dst[pos] = dst;
    }
    int n_rows = 0;
#pragma unroll
    for (int w = 0; w < kMaxTileRows / 32; ++w) n_rows += s_warp_count[w];
    __syncthreads();

    // ---- 2. move the rows ------------------------------------------------
    if (!mis) {
      const uint32_t rv = p.row_vecs.d;
      const uint32_t n_items = static_cast<uint32_t>(n_rows) * rv;
      for (uint32_t base = tid; base < n_items; base += kThreads * kUnroll) {
        V buf[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const uint32_t i = base + u * kThreads;
          if (i < n_items) {
            const uint32_t r = p.row_vecs.div(i);
            const uint32_t c = i - r * rv;
            buf[u] = __ldcs(reinterpret_cast<const V*>(s_src[r]) + c);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const uint32_t i = base + u * kThreads;
          if (i < n_items) {
            const uint32_t r = p.row_vecs.div(i);
            const uint32_t c = i - r * rv;
            __stcs(reinterpret_cast<V*>(s_dst[r]) + c, buf[u]);
          }
        }
      }
    } else {
      // Byte-wise fallback for rows whose addresses are not VEC-aligned.
      const int64_t n_bytes = static_cast<int64_t>(n_rows) * p.row_bytes;
      for (int64_t i = tid; i < n_bytes; i += kThreads) {
        const int64_t r = i / p.row_bytes;
        const int64_t c = i - r * p.row_bytes;
        s_dst[r][c] = s_src[r][c];
      }
    }
    __syncthreads();  // the next tile reuses s_src, s_dst and s_warp_count
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy (TMA) path for device-resident objects.
//
// Each CTA is one warp that owns a contiguous, balanced range of rows in
// (kv, layer, token) order and streams it through a ring of shared-memory
// stages with the asynchronous bulk-copy engine:
//   load   cp.async.bulk global -> shared, completion counted in bytes on
//          the stage's mbarrier;
//   store  cp.async.bulk shared -> global (bulk_group), whose smem reads are
//          awaited with cp.async.bulk.wait_group.read before the stage is
//          refilled.
// Lane i of a group handles row i of the group. Consecutive rows whose source
// and destination are both contiguous (consecutive slots in the paged buffer
// and consecutive tokens in the object, e.g. all tokens of one page) are
// merged into one copy issued by the run's first lane. Loads are plain
// (single-CTA) bulk copies; the kernel needs no cluster launch.
// ---------------------------------------------------------------------------

constexpr int kBulkMaxStages = 8;
constexpr int64_t kVectorMinTraffic = int64_t(256) << 20;
// Rows shorter than this whose LMCache side is not contiguous from one token
// to the next (token-major [T, 2, H] objects interleave K and V) never merge
// into longer copies, so the bulk ring would issue one tiny bulk copy per row;
// the vectorised kernel moves them faster. Measured on B200 for 256-byte rows
// (a Llama-3-70B TP-8 shard, the layerwise path): 3.5 against 4.1 us per
// one-chunk launch; 2048-byte rows still favour the bulk ring (3.0 against
// 3.8 us).
constexpr int64_t kBulkMinUnmergedRow = 1024;
// Upper bound of the ring's dynamic shared memory (stages * stage bytes plus
// bookkeeping); the kernels' limit is raised to this once per device.
constexpr size_t kBulkSmemCap = 200 * 1024;
constexpr uint32_t kWaitSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(__cvta_generic_to_global(gsrc)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   __cvta_generic_to_global(gdst)),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_all_but_one() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Waits until every bulk store of this thread has finished reading shared
// memory. The global writes themselves complete with the grid (kernel
// completion orders them before any later work in the stream).
__device__ __forceinline__ void bulk_wait_reads_done() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

constexpr int kBatchRows = 256;   // rows resolved together (8 per lane)
// Bit 63 of a resolved destination marks a row that is not 16-byte aligned
// (user-space addresses never set it).
constexpr uint64_t kMisalignedTag = uint64_t(1) << 63;

struct BulkParams {
  int32_t num_rows;      // num_kv * num_layers * num_tokens (< 2^31)
  int32_t stage_rows;    // rows per stage (<= 32)
  int32_t stages;        // ring depth (<= kBulkMaxStages)
  int32_t stage_bytes;   // bytes per stage (>= stage_rows * row_bytes)
  int32_t batch_rows;    // rows resolved together: a multiple of 32, <= kBatchRows
  int32_t prefetch_lmc;  // 1: prefetch this CTA's first source rows of the object into L2
  FastDiv div_tokens;    // row -> (kv * num_layers + layer, token)
  FastDiv div_layers;    // (kv * num_layers + layer) -> (kv, layer)
};

// Prefetches [src, src + bytes) into L2 with the bulk-copy engine; src and
// bytes are multiples of 16. A hint: it writes nothing and orders nothing.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                   __cvta_generic_to_global(src)),
               "r"(bytes)
               : "memory");
}

template <typename SlotT, int MODE>
__global__ void __launch_bounds__(32)
transfer_rows_bulk_kernel(const TransferParams p, const BulkParams b,
                          const __grid_constant__ ObjectTable<batched_mode(MODE)> tab) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* data = smem;
  // Bookkeeping after the ring, sized by this launch's geometry.
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(b.stages) * b.stage_bytes);
  uint64_t* s_dst = bars + b.stages;                    // [stages][32] store targets
  uint64_t* tab_src = s_dst + b.stages * 32;            // [batch_rows] resolved sources
  uint64_t* tab_dst = tab_src + b.batch_rows;           // [batch_rows] resolved destinations
  uint32_t* s_len = reinterpret_cast<uint32_t*>(tab_dst + b.batch_rows);  // [stages][32]
  int32_t* s_objoff = reinterpret_cast<int32_t*>(s_len + b.stages * 32);  // batched only

  const int lane = threadIdx.x;
  const SlotT* __restrict__ slots = static_cast<const SlotT*>(p.slots);
  const int32_t r_begin = static_cast<int32_t>(static_cast<int64_t>(b.num_rows) * blockIdx.x / gridDim.x);
  const int32_t r_end = static_cast<int32_t>(static_cast<int64_t>(b.num_rows) * (blockIdx.x + 1) / gridDim.x);
  const int32_t n_rows = r_end - r_begin;
  const uint32_t row_bytes = static_cast<uint32_t>(p.row_bytes);
  // Batches: first_batch rows, then batch_rows rows each. The first batch
  // after griddepcontrol.wait is what the ring takes at once (stages x
  // stage_rows, at most batch_rows): the first loads issue after one
  // slot-load latency and no more address arithmetic than they need, and a
  // CTA with few rows resolves them all in that one latency. Later batches are
  // resolved while earlier groups are in flight. Groups never straddle a
  // batch: a batch of n rows holds ceil(n / stage_rows) groups.
  const int32_t batch_rows = b.batch_rows;
  const int32_t groups_per_batch = (batch_rows + b.stage_rows - 1) / b.stage_rows;
  const int32_t first_batch = min(batch_rows, b.stages * b.stage_rows);
  const int32_t first_rows = min(first_batch, n_rows);
  const int32_t rest_rows = n_rows - first_rows;
  const int32_t full_batches = rest_rows / batch_rows;
  const int32_t tail_rows = rest_rows - full_batches * batch_rows;
  const int64_t n_groups = (first_rows + b.stage_rows - 1) / b.stage_rows +
                           static_cast<int64_t>(full_batches) * groups_per_batch +
                           (tail_rows + b.stage_rows - 1) / b.stage_rows;

  if (lane == 0) {
    for (int s = 0; s < b.stages; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  // Batched modes search their object table's token offsets, staged in
  // shared memory (from the kernel parameters) before the first resolution.
  const int32_t* obj_offsets = s_objoff;

  // Resolves rows [b0, b0 + n) of this CTA's range into tab_src / tab_dst
  // (0 for skipped rows). All slot ids and layer bases of the batch are
  // loaded before any is used, so the batch costs one memory latency.
  auto resolve_batch = [&](int32_t b0, int32_t n) {
    constexpr int kPer = kBatchRows / 32;
    int64_t slot[kPer];
    uint8_t* base[kPer];
    uint8_t* lmcs[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int idx = lane + 32 * j;
      slot[j] = -1;
      base[j] = nullptr;
      lmcs[j] = nullptr;
      if (idx < n) {
        const uint32_t r = static_cast<uint32_t>(r_begin + b0 + idx);
        const uint32_t q = b.div_tokens.div(r);
        const int tok = static_cast<int>(r - q * b.div_tokens.d);
        const int kv = static_cast<int>(b.div_layers.div(q));
        const int layer = static_cast<int>(q - kv * b.div_layers.d);
        int64_t slot_index;
        lmcs[j] = lmc_row<MODE>(p, tab, obj_offsets, kv, layer, tok, &slot_index);
        slot[j] = static_cast<int64_t>(slots[slot_index]);
        if (!paged_direct(MODE)) {
          const uint64_t* arr = kv == 0 ? p.ptrs_k : p.ptrs_v;
          base[j] = reinterpret_cast<uint8_t*>(arr[layer]) + kv * p.page_kv_offset;
        } else {
          base[j] = kv == 0 ? p.base_k : p.base_v;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int idx = lane + 32 * j;
      if (idx >= n) continue;
      uint64_t src = 0, dst = 0;
      bool valid = slot[j] >= 0;
      if (valid && p.num_paged_rows > 0 && slot[j] >= p.num_paged_rows) {
        valid = false;
        raise_flag(p.status, LMCB_DEVICE_FLAG_SLOT_OUT_OF_RANGE);
      }
      if (valid) {
        uint8_t* paged = base[j] + slot[j] * p.paged_row_stride;
        uint8_t* s = p.page2L ? paged : lmcs[j];
        uint8_t* d = p.page2L ? lmcs[j] : paged;
        src = reinterpret_cast<uint64_t>(s);
        dst = reinterpret_cast<uint64_t>(d);
        if (((src | dst) & 15) != 0) {
          // Not 16-byte aligned (only possible through the pointer array):
          // tagged here, copied byte-wise when its group is issued.
          dst |= kMisalignedTag;
        }
      }
      tab_src[idx] = src;
      tab_dst[idx] = dst;
    }
    __syncwarp();
  };

  // Group cursor: (batch start, rows in batch, next row in batch).
  int32_t cur_b0 = 0, cur_n = 0, cur_next = 0;

  // Takes the next group of rows from the resolved batch (resolving the next
  // batch first when this one is used up), merges contiguous runs and starts
  // their loads into stage `st`.
  auto issue_load = [&](int st) {
    if (cur_next >= cur_n) {
      cur_b0 += cur_n;
      cur_n = min(cur_b0 == 0 ? first_batch : batch_rows, n_rows - cur_b0);
      cur_next = 0;
      resolve_batch(cur_b0, cur_n);
    }
    const int32_t count = min(b.stage_rows, cur_n - cur_next);
    const uint8_t* src = nullptr;
    uint8_t* dst = nullptr;
    if (lane < count) {
      src = reinterpret_cast<const uint8_t*>(tab_src[cur_next + lane]);
      const uint64_t d = tab_dst[cur_next + lane];
      if (d & kMisalignedTag) {
        // Rows the bulk engine cannot address (16-byte alignment) are copied
        // byte-wise by their lane and left out of the ring.
        uint8_t* dd = reinterpret_cast<uint8_t*>(d & ~kMisalignedTag);
        for (uint32_t i = 0; i < row_bytes; ++i) dd[i] = src[i];
        src = nullptr;
      } else {
        dst = reinterpret_cast<uint8_t*>(d);
      }
    }
    cur_next += count;
    const bool valid = src != nullptr;
    const uintptr_t prev_src =
        __shfl_up_sync(0xffffffffu, reinterpret_cast<uintptr_t>(src), 1);
    const uintptr_t prev_dst =
        __shfl_up_sync(0xffffffffu, reinterpret_cast<uintptr_t>(dst), 1);
    // Row i of the group sits in stage slot i, so rows that are consecutive
    // on one side move with one copy on that side. The two sides merge
    // independently: a store of random slots into an object (MLA) writes each
    // group with one copy, a retrieve from it reads each group with one; when
    // both sides are contiguous (consecutive slots of a page, consecutive
    // tokens of the object) both merge.
    const bool prev_valid = lane > 0 && prev_src != 0;
    const bool cont_src =
        valid && prev_valid && reinterpret_cast<uintptr_t>(src) == prev_src + row_bytes;
    const bool cont_dst =
        valid && prev_valid && reinterpret_cast<uintptr_t>(dst) == prev_dst + row_bytes;
    const uint32_t src_mask = __ballot_sync(0xffffffffu, cont_src);
    const uint32_t dst_mask = __ballot_sync(0xffffffffu, cont_dst);
    // Rows lane, lane + 1, ... while the following lanes continue the run.
    auto run_rows = [&](uint32_t mask) -> uint32_t {
      const uint32_t after = lane == 31 ? 0u : (mask >> (lane + 1));
      return 1 + static_cast<uint32_t>(__ffs(~after) - 1);
    };
    const uint32_t load_bytes = (valid && !cont_src) ? run_rows(src_mask) * row_bytes : 0;
    const uint32_t store_bytes = (valid && !cont_dst) ? run_rows(dst_mask) * row_bytes : 0;
    const uint32_t total = __reduce_add_sync(0xffffffffu, load_bytes);
    if (lane == 0) mbar_arrive_expect_tx(&bars[st], total);
    __syncwarp();
    uint8_t* stage_slot = data + static_cast<size_t>(st) * b.stage_bytes + lane * row_bytes;
    if (load_bytes) bulk_load(stage_slot, src, load_bytes, &bars[st]);
    s_dst[st * 32 + lane] = reinterpret_cast<uint64_t>(dst);
    s_len[st * 32 + lane] = store_bytes;
  };

  // Under programmatic dependent launch this CTA can start while the previous
  // kernel in the stream is still running, and none of that kernel's writes
  // is guaranteed visible before griddepcontrol.wait -- the slot mapping and
  // the layer-base array included, since a caller may build either on the
  // GPU right before the transfer. Before the wait the CTA therefore only
  // prefetches its first batch's slot ids and layer bases into L2 (a hint
  // that loads nothing into registers; L2 sees the previous kernel's writes).
  if (!batched_mode(MODE) && n_rows > 0) {
    constexpr int kPer = kBatchRows / 32;
    const int32_t n0 = min(first_batch, n_rows);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int idx = lane + 32 * j;
      if (idx < n0) {
        const uint32_t r = static_cast<uint32_t>(r_begin + idx);
        const uint32_t q = b.div_tokens.div(r);
        const int tok = static_cast<int>(r - q * b.div_tokens.d);
        const int kv = static_cast<int>(b.div_layers.div(q));
        const int layer = static_cast<int>(q - kv * b.div_layers.d);
        prefetch_l2(slots + tok);
        if (!paged_direct(MODE)) prefetch_l2((kv == 0 ? p.ptrs_k : p.ptrs_v) + layer);
      }
    }
  }
  // A retrieve from a device object reads the object's rows in this CTA's
  // order, and those addresses come from the kernel parameters, not from
  // memory: the CTA's first ring-full of source bytes is prefetched into L2
  // before the wait (a hint; the previous kernel's writes to those lines
  // still land in L2, which the bulk loads read). The launch's first loads
  // then hit L2 while DRAM serves them during the previous kernel's tail.
  if (!batched_mode(MODE) && b.prefetch_lmc && n_rows > 0) {
    const uint64_t bytes = static_cast<uint64_t>(first_rows) * row_bytes;
    constexpr uint32_t kPiece = 16384;
    const uint8_t* base = p.lmc + static_cast<int64_t>(r_begin) * row_bytes;
    for (uint64_t off = static_cast<uint64_t>(lane) * kPiece; off < bytes; off += 32 * kPiece) {
      const uint64_t left = bytes - off;
      bulk_prefetch_l2(base + off, static_cast<uint32_t>(left < kPiece ? left : kPiece));
    }
  }
  if constexpr (batched_mode(MODE)) {
    stage_obj_offsets(p, tab, s_objoff, lane, 32);  // parameters, not an input in memory
    __syncwarp();
  }
  pdl_wait();
  pdl_launch_dependents();

  int64_t issued = 0;
  for (; issued < n_groups && issued < b.stages; ++issued) issue_load(static_cast<int>(issued));

  bool timed_out = false;
  for (int64_t g = 0; g < n_groups; ++g) {
    const int st = static_cast<int>(g % b.stages);
    const uint32_t parity = static_cast<uint32_t>((g / b.stages) & 1);
    uint32_t spins = 0;
    while (!mbar_try_wait(&bars[st], parity)) {
      if (++spins >= kWaitSpinLimit) {
        timed_out = true;
        break;
      }
    }
    if (__any_sync(0xffffffffu, timed_out)) {
      if (lane == 0) raise_flag(p.status, LMCB_DEVICE_FLAG_WAIT_TIMEOUT);
      // Give the loads still in flight a bounded chance to land before the
      // CTA (and its shared memory) goes away.
      for (int64_t g2 = g + 1; g2 < issued; ++g2) {
        const int st2 = static_cast<int>(g2 % b.stages);
        const uint32_t par2 = static_cast<uint32_t>((g2 / b.stages) & 1);
        for (uint32_t k = 0; k < kWaitSpinLimit && !mbar_try_wait(&bars[st2], par2); ++k) {
        }
      }
      break;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const uint32_t len = s_len[st * 32 + lane];
    if (len) {
      bulk_store(reinterpret_cast<void*>(s_dst[st * 32 + lane]),
                 data + static_cast<size_t>(st) * b.stage_bytes + lane * row_bytes, len);
    }
    bulk_commit();
    if (g >= 1 && issued < n_groups) {
      // The previous group's stage is free once its store has read it.
      bulk_wait_read_all_but_one();
      issue_load(static_cast<int>(issued % b.stages));
      ++issued;
    }
  }
  bulk_wait_reads_done();
}

struct BulkConfig {
  int stages;
  int stage_kb;
  int ctas_per_sm;
};

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == 0) return dflt;
  return std::atoi(v);
}

// Ring geometry; LMCB_BULK_STAGES / LMCB_BULK_STAGE_KB / LMCB_BULK_CTAS_PER_SM
// override the defaults (tuning only; read on every call so a process can
// compare settings). Defaults from sweeps on B200 (median of three, fraction
// of the copy roofline, one stream / two streams):
//   rows of 512 B or less (a Llama-3-70B TP-8 shard, 10 MB launches): many
//   small CTAs, 12/SM x 2 stages x 8 KB: 0.59 / 0.84, against 0.55 / 0.63
//   for 4/SM x 6 x 8 KB;
//   longer rows, launches under 24 MB (random 1152-byte MLA rows, 18 MB):
//   4/SM x 3 x 16 KB: 0.70 / 0.81, against 0.67 / 0.75 for 3/SM x 4 x 16 KB;
//   longer rows, larger launches (2 KB rows, 32 MB and more): 3/SM x 4 x
//   16 KB: 0.85 / 0.97.
// A short launch is the fixed chain of slot loads, first bulk loads, stores
// and drain: more, smaller CTAs shorten each CTA's chain, and their small
// shared-memory footprint lets the next launch's CTAs be resident (waiting
// in griddepcontrol.wait) while this one runs.
BulkConfig bulk_config(int64_t row_bytes, int64_t launch_bytes) {
  const bool short_rows = row_bytes <= 512;
  const bool small_launch = launch_bytes < (int64_t(24) << 20);
  BulkConfig c;
  const int d_stages = short_rows ? 2 : (small_launch ? 3 : 4);
  const int d_kb = short_rows ? 8 : 16;
  const int d_ctas = short_rows ? 12 : (small_launch ? 4 : 3);
  c.stages = env_int("LMCB_BULK_STAGES", d_stages);
  c.stage_kb = env_int("LMCB_BULK_STAGE_KB", d_kb);
  c.ctas_per_sm = env_int("LMCB_BULK_CTAS_PER_SM", d_ctas);
  if (c.stages < 2) c.stages = 2;
  if (c.stages > kBulkMaxStages) c.stages = kBulkMaxStages;
  if (c.stage_kb < 4) c.stage_kb = 4;
  if (c.stage_kb > 64) c.stage_kb = 64;
  while (c.stages * c.stage_kb > 192 && c.stages > 2) --c.stages;  // per-CTA smem cap
  if (c.ctas_per_sm < 1) c.ctas_per_sm = 1;
  if (c.ctas_per_sm > 16) c.ctas_per_sm = 16;
  return c;
}

size_t bulk_smem_bytes(const BulkParams& b, bool batched) {
  return static_cast<size_t>(b.stages) * b.stage_bytes + b.stages * sizeof(uint64_t) +
         b.stages * 32 * (sizeof(uint64_t) + sizeof(uint32_t)) +
         2 * static_cast<size_t>(b.batch_rows) * sizeof(uint64_t) +
         (batched ? (kMaxObjects + 1) * sizeof(int32_t) : 0);
}

// LMCB_PDL=0 launches without the programmatic-serialization attribute.
bool pdl_enabled() {
  const char* v = std::getenv("LMCB_PDL");
  return v == nullptr || std::strcmp(v, "0") != 0;
}

template <typename Kernel, typename... Args>
cudaError_t launch_ex(Kernel* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The table argument of a launch: the batched table, or the empty one.
template <int MODE>
const ObjectTable<batched_mode(MODE)>& table_arg(const ObjectTable<true>* tab) {
  static const ObjectTable<false> kNone{};
  if constexpr (batched_mode(MODE)) {
    return *tab;
  } else {
    (void)tab;
    return kNone;
  }
}

template <typename SlotT, int MODE>
cudaError_t launch_bulk_mode(const TransferParams& p, const BulkParams& b,
                             const ObjectTable<true>* tab, int grid, cudaStream_t stream) {
  const size_t smem = bulk_smem_bytes(b, batched_mode(MODE));
  cudaError_t err = ensure_smem_limit<&transfer_rows_bulk_kernel<SlotT, MODE>>(smem, kBulkSmemCap);
  if (err != cudaSuccess) return err;
  return launch_ex(&transfer_rows_bulk_kernel<SlotT, MODE>, dim3(grid), dim3(32), smem, stream,
                   p, b, table_arg<MODE>(tab));
}

template <typename SlotT>
cudaError_t launch_bulk(const TransferParams& p, const BulkParams& b,
                        const ObjectTable<true>* tab, int mode, int grid, cudaStream_t stream) {
  switch (mode) {
    case kPtrArray: return launch_bulk_mode<SlotT, kPtrArray>(p, b, tab, grid, stream);
    case kDirect: return launch_bulk_mode<SlotT, kDirect>(p, b, tab, grid, stream);
    case kBatched: return launch_bulk_mode<SlotT, kBatched>(p, b, tab, grid, stream);
    default: return launch_bulk_mode<SlotT, kBatchedDirect>(p, b, tab, grid, stream);
  }
}

// True when `ptr` is device memory (not a host mapping); bulk copies are
// used only between device buffers. Registered host ranges are recognised
// without a driver call.
bool is_device_memory(const void* ptr) {
  if (lmcb_host_get_device_ptr(const_cast<void*>(ptr)) != nullptr) return false;
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeDevice;
}

// Largest power of two <= 16 dividing every value in `vals`.
int pick_vec(std::initializer_list<uint64_t> vals) {
  uint64_t g = 0;
  for (uint64_t v : vals) g |= v;
  if (g % 16 == 0) return 16;
  if (g % 8 == 0) return 8;
  if (g % 4 == 0) return 4;
  if (g % 2 == 0) return 2;
  return 1;
}

template <typename SlotT, int VEC, int MODE>
cudaError_t launch_vec_mode(const TransferParams& p, const ObjectTable<true>* tab, int grid,
                            cudaStream_t stream) {
  if (p.num_tiles <= grid) {  // one wave: every tile has its own CTA
    return launch_ex(&transfer_rows_kernel<SlotT, VEC, MODE, kUnrollShort>, dim3(grid),
                     dim3(kThreads), 0, stream, p, table_arg<MODE>(tab));
  }
  return launch_ex(&transfer_rows_kernel<SlotT, VEC, MODE, kUnrollLong>, dim3(grid),
                   dim3(kThreads), 0, stream, p, table_arg<MODE>(tab));
}

template <typename SlotT, int VEC>
cudaError_t launch_vec(const TransferParams& p, const ObjectTable<true>* tab, int mode, int grid,
                       cudaStream_t stream) {
  switch (mode) {
    case kPtrArray: return launch_vec_mode<SlotT, VEC, kPtrArray>(p, tab, grid, stream);
    case kDirect: return launch_vec_mode<SlotT, VEC, kDirect>(p, tab, grid, stream);
    case kBatched: return launch_vec_mode<SlotT, VEC, kBatched>(p, tab, grid, stream);
    default: return launch_vec_mode<SlotT, VEC, kBatchedDirect>(p, tab, grid, stream);
  }
}

template <typename SlotT>
cudaError_t launch_slot(const TransferParams& p, const ObjectTable<true>* tab, int vec, int mode,
                        int grid, cudaStream_t stream) {
  switch (vec) {
    case 16: return launch_vec<SlotT, 16>(p, tab, mode, grid, stream);
    case 8: return launch_vec<SlotT, 8>(p, tab, mode, grid, stream);
    case 4: return launch_vec<SlotT, 4>(p, tab, mode, grid, stream);
    default: return launch_vec<SlotT, 2>(p, tab, mode, grid, stream);
  }
}

// Validates the common arguments, fills the derived fields of `p` and
// launches. `alignment_terms` are the host-known addresses and strides that
// must all be multiples of the vector width.
int launch_transfer(TransferParams p, int type, int slot_type, int mode,
                    std::initializer_list<uint64_t> alignment_terms,
                    cudaStream_t stream, const char* who, bool objects_on_device = false,
                    bool force_vector = false, const ObjectTable<true>* tab = nullptr) {
  const int esz = dtype_size(type);
  if (esz == 0) {
    return fail(LMCB_ERR_UNSUPPORTED_DTYPE, std::string(who) + ": ScalarType not supported.");
  }
  if (slot_type != LMCB_DTYPE_INT64 && slot_type != LMCB_DTYPE_INT32) {
    return fail(LMCB_ERR_UNSUPPORTED_DTYPE,
                std::string(who) + ": slot ids must be int64 or int32.");
  }
  if (p.num_tokens < 0 || p.num_layers < 0 || p.row_bytes <= 0) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": negative size.");
  }
  if (p.num_tokens == 0 || p.num_layers == 0) return LMCB_OK;
  if ((!batched_mode(mode) && p.lmc == nullptr) || p.slots == nullptr) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL pointer.");
  }
  if (batched_mode(mode) && (tab == nullptr || p.num_objects <= 0 ||
                             p.num_objects > kMaxObjects)) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": bad object table.");
  }
  if (!paged_direct(mode) && (p.ptrs_k == nullptr || p.ptrs_v == nullptr)) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL pointer array.");
  }
  if (paged_direct(mode) && (p.base_k == nullptr || (p.num_kv > 1 && p.base_v == nullptr))) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL cache pointer.");
  }
  p.status = device_status_ptr();
  if (p.status == nullptr) return LMCB_ERR_CUDA;

  int vec = pick_vec(alignment_terms);
  if (vec < 2) vec = 2;  // every supported element is >= 2 bytes

  // Path choice: bulk copies when both sides are device memory, rows are
  // 16-byte multiples and fit a stage; LMCB_TRANSFER_PATH=vector|bulk forces
  // one (bulk still requires those conditions).
  const int forced = [] {
    const char* v = std::getenv("LMCB_TRANSFER_PATH");
    if (v == nullptr) return 0;
    if (std::strcmp(v, "vector") == 0) return 1;
    if (std::strcmp(v, "bulk") == 0) return 2;
    return 0;
  }();
  const int64_t total_rows = static_cast<int64_t>(p.num_kv) * p.num_layers * p.num_tokens;
  const BulkConfig bc = bulk_config(p.row_bytes, total_rows * p.row_bytes);
  const int64_t stage_bytes = static_cast<int64_t>(bc.stage_kb) * 1024;
  const bool lmc_on_device = batched_mode(mode) ? objects_on_device : is_device_memory(p.lmc);
  const bool bulk_ok = vec == 16 && p.row_bytes % 16 == 0 && p.row_bytes <= stage_bytes &&
                       lmc_on_device;
  // Launches moving at least kVectorMinTraffic bytes stream slightly better on
  // the vectorised kernel (full occupancy, no per-launch ramp to hide); the
  // bulk ring wins below it, where its shorter ramp dominates. Measured on
  // B200: 64 MB (one c2 chunk) bulk 12.1 us vs vector 13.6 us; 2 GB (a
  // request's chunks in one launch) vector 0.92 vs bulk 0.90 of the copy
  // roofline, and 0.80 vs 0.72 for random 1152-byte MLA rows.
  const bool large = 2 * total_rows * p.row_bytes >= kVectorMinTraffic;
  const bool token_contiguous =
      batched_mode(mode) ? p.obj_token_major == 0 : p.lmc_token_stride == p.row_bytes;
  const bool unmerged_short = !token_contiguous && p.row_bytes < kBulkMinUnmergedRow;
  if (bulk_ok && forced != 1 && !force_vector && total_rows < (int64_t(1) << 31) &&
      (forced == 2 || (!large && !unmerged_short))) {
    BulkParams b;
    b.num_rows = static_cast<int32_t>(total_rows);
    int64_t rows = stage_bytes / p.row_bytes;
    b.stage_rows = static_cast<int32_t>(rows > 32 ? 32 : rows);
    b.stages = bc.stages;
    b.stage_bytes = static_cast<int32_t>(stage_bytes);
    b.div_tokens = FastDiv(static_cast<uint32_t>(p.num_tokens));
    b.div_layers = FastDiv(static_cast<uint32_t>(p.num_layers));
    int64_t grid = static_cast<int64_t>(current_sm_count()) * bc.ctas_per_sm;
    const int64_t groups = (total_rows + b.stage_rows - 1) / b.stage_rows;
    if (grid > groups) grid = groups;
    if (grid < 1) grid = 1;
    // The resolution table holds what one CTA resolves at once: at most
    // kBatchRows rows, and no more than a CTA's whole range (short launches
    // then need less shared memory per CTA).
    const int64_t rows_per_cta = (total_rows + grid - 1) / grid;
    b.batch_rows = static_cast<int32_t>(std::min<int64_t>(kBatchRows, (rows_per_cta + 31) / 32 * 32));
    // Retrieves from a dense device object prefetch their first source rows
    // before griddepcontrol.wait (LMCB_BULK_PREFETCH=0 turns it off).
    const int64_t T = p.num_tokens, L = p.num_layers;
    const bool lmc_dense = !batched_mode(mode) && p.lmc_token_stride == p.row_bytes &&
                           (L == 1 || p.lmc_layer_stride == p.row_bytes * T) &&
                           (p.num_kv == 1 || p.lmc_kv_stride == p.row_bytes * T * L);
    b.prefetch_lmc = (!p.page2L && lmc_dense && env_int("LMCB_BULK_PREFETCH", 1) != 0) ? 1 : 0;
    cudaError_t err = slot_type == LMCB_DTYPE_INT64
                          ? launch_bulk<int64_t>(p, b, tab, mode, static_cast<int>(grid), stream)
                          : launch_bulk<int32_t>(p, b, tab, mode, static_cast<int>(grid), stream);
    if (err != cudaSuccess) return cuda_fail(err, who);
    return LMCB_OK;
  }

  const int64_t row_vecs = p.row_bytes / vec;
  int64_t tile_rows = kTargetTileBytes / p.row_bytes;
  if (tile_rows < 1) tile_rows = 1;
  if (tile_rows > kMaxTileRows) tile_rows = kMaxTileRows;
  // The flat item index (rows * row_vecs) must stay below 2^31.
  while (tile_rows > 1 && tile_rows * row_vecs >= (int64_t(1) << 31)) tile_rows >>= 1;
  if (row_vecs >= (int64_t(1) << 31)) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": row too long.");
  }
  // Tiny launches (one chunk of one layer: 512 rows) would leave most SMs
  // without a tile: smaller tiles, down to 32 rows, until every SM has
  // kMinTilesPerSm of them (LMCB_VEC_MIN_TILES_PER_SM overrides). Measured on
  // B200: a c5 single-layer chunk launch 3.6 -> 2.4 us. Going further costs
  // more than it gains: a c5 single-layer batched launch (32,768 rows of
  // 256 B) takes 6.5 us with 128-row tiles (1.7 per SM) and 7.4 us with
  // 64-row tiles (3.5 per SM).
  {
    const int64_t want = static_cast<int64_t>(current_sm_count()) *
                         env_int("LMCB_VEC_MIN_TILES_PER_SM", kMinTilesPerSm);
    const int64_t seqs = static_cast<int64_t>(p.num_kv) * p.num_layers;
    while (tile_rows > 32 && seqs * ((p.num_tokens + tile_rows - 1) / tile_rows) < want) {
      tile_rows >>= 1;
    }
  }
  p.tile_rows = static_cast<int32_t>(tile_rows);
  p.tiles_per_seq = static_cast<int32_t>((p.num_tokens + tile_rows - 1) / tile_rows);
  p.prefetch_lmc =
      (!p.page2L && lmc_on_device && env_int("LMCB_BULK_PREFETCH", 1) != 0) ? 1 : 0;
  p.num_tiles = static_cast<int64_t>(p.num_kv) * p.num_layers * p.tiles_per_seq;
  p.row_vecs = FastDiv(static_cast<uint32_t>(row_vecs));

  const int64_t max_grid = static_cast<int64_t>(current_sm_count()) * 8;
  const int grid = static_cast<int>(p.num_tiles < max_grid ? p.num_tiles : max_grid);

  cudaError_t err = slot_type == LMCB_DTYPE_INT64
                        ? launch_slot<int64_t>(p, tab, vec, mode, grid, stream)
                        : launch_slot<int32_t>(p, tab, vec, mode, grid, stream);
  if (err != cudaSuccess) return cuda_fail(err, who);
  return LMCB_OK;
}

// Launches a batched transfer whose object table is in host memory: checks
// the table, then issues one launch per group of at most kMaxObjects objects,
// each carrying its part of the table (token offsets rebased to 0) in its
// kernel parameters. `p` holds every other field.
int launch_batched(TransferParams p, int type, int slot_type, int mode,
                   std::initializer_list<uint64_t> alignment_terms, cudaStream_t stream,
                   const char* who, bool objects_on_device, const uint64_t* object_ptrs,
                   const int64_t* token_offsets, const int64_t* slot_starts, int32_t num_objects,
                   int64_t total_tokens) {
  if (object_ptrs == nullptr || token_offsets == nullptr || slot_starts == nullptr) {
    return fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL object table.");
  }
  if (token_offsets[num_objects] - token_offsets[0] != total_tokens) {
    return fail(LMCB_ERR_INVALID_ARGUMENT,
                std::string(who) + ": token offsets do not add up to the token count.");
  }
  for (int32_t i = 0; i < num_objects; ++i) {
    if (token_offsets[i + 1] < token_offsets[i] || slot_starts[i] < 0 ||
        (token_offsets[i + 1] > token_offsets[i] && object_ptrs[i] == 0)) {
      return fail(LMCB_ERR_INVALID_ARGUMENT,
                  std::string(who) + ": object " + std::to_string(i) + " is malformed.");
    }
  }
  ObjectTable<true> tab;
  for (int32_t g0 = 0; g0 < num_objects; g0 += kMaxObjects) {
    const int32_t g1 = std::min(num_objects, g0 + kMaxObjects);
    const int64_t base = token_offsets[g0];
    const int64_t tokens = token_offsets[g1] - base;
    if (tokens == 0) continue;
    for (int32_t i = g0; i < g1; ++i) {
      tab.ptrs[i - g0] = object_ptrs[i];
      tab.slot_starts[i - g0] = slot_starts[i];
      tab.offsets[i - g0] = static_cast<int32_t>(token_offsets[i] - base);
    }
    tab.offsets[g1 - g0] = static_cast<int32_t>(tokens);
    p.num_objects = g1 - g0;
    p.num_tokens = static_cast<int32_t>(tokens);
    const int rc = launch_transfer(p, type, slot_type, mode, alignment_terms, stream, who,
                                   objects_on_device, false, &tab);
    if (rc != LMCB_OK) return rc;
  }
  return LMCB_OK;
}

}  // namespace
}  // namespace lmcb

using lmcb::TransferParams;

extern "C" {

int lmcb_multi_layer_kv_transfer_kernel(int type, int slotType, void* stream,
                                        const uint64_t* pagedKVCaches,
                                        void* dstCacheTensor,
                                        const void* slotmappings,
                                        int64_t hiddenDims, int32_t kvs,
                                        int32_t numLayers, int64_t pageBuffSize,
                                        int32_t numTokensChunk, int page2L) {
  lmcb::clear_error();
  const char* who = "multi_layer_kv_transfer";
  if (kvs != 1 && kvs != 2) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": kvs must be 1 or 2.");
  }
  if (kvs == 2 && pageBuffSize <= 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      std::string(who) + ": page_buffer_size must be positive for K/V caches.");
  }
  const int64_t esz = lmcb::dtype_size(type);
  const int64_t row = hiddenDims * esz;
  TransferParams p{};
  p.lmc = static_cast<uint8_t*>(dstCacheTensor);
  p.lmc_token_stride = row;
  p.lmc_layer_stride = row * numTokensChunk;
  p.lmc_kv_stride = p.lmc_layer_stride * numLayers;
  p.ptrs_k = pagedKVCaches;
  p.ptrs_v = pagedKVCaches;
  p.page_kv_offset = pageBuffSize * row;
  p.paged_row_stride = row;
  p.num_paged_rows = pageBuffSize;
  p.slots = slotmappings;
  p.num_tokens = numTokensChunk;
  p.num_layers = numLayers;
  p.num_kv = kvs;
  p.row_bytes = row;
  p.page2L = page2L ? 1 : 0;
  if (esz == 0) p.row_bytes = 1;  // rejected in launch_transfer
  return lmcb::launch_transfer(
      p, type, slotType, lmcb::kPtrArray,
      {reinterpret_cast<uint64_t>(dstCacheTensor), static_cast<uint64_t>(row),
       static_cast<uint64_t>(p.page_kv_offset)},
      static_cast<cudaStream_t>(stream), who);
}

int lmcb_multi_layer_kv_transfer_unilateral_kernel(
    int type, int slotType, void* stream, const uint64_t* keyPtrs,
    const uint64_t* valuePtrs, void* dstCacheTensor, const void* slotmappings,
    int64_t hiddenDims, int32_t numLayers, int64_t pageBuffSize,
    int32_t numTokensChunk, int page2L) {
  lmcb::clear_error();
  const char* who = "multi_layer_kv_transfer_unilateral";
  const int64_t esz = lmcb::dtype_size(type);
  const int64_t row = hiddenDims * esz;
  TransferParams p{};
  p.lmc = static_cast<uint8_t*>(dstCacheTensor);
  p.lmc_token_stride = row;
  p.lmc_layer_stride = row * numTokensChunk;
  p.lmc_kv_stride = p.lmc_layer_stride * numLayers;
  p.ptrs_k = keyPtrs;
  p.ptrs_v = valuePtrs;
  p.page_kv_offset = 0;
  p.paged_row_stride = row;
  p.num_paged_rows = pageBuffSize;
  p.slots = slotmappings;
  p.num_tokens = numTokensChunk;
  p.num_layers = numLayers;
  p.num_kv = 2;
  p.row_bytes = esz == 0 ? 1 : row;
  p.page2L = page2L ? 1 : 0;
  return lmcb::launch_transfer(
      p, type, slotType, lmcb::kPtrArray,
      {reinterpret_cast<uint64_t>(dstCacheTensor), static_cast<uint64_t>(row)},
      static_cast<cudaStream_t>(stream), who);
}

int lmcb_single_layer_kv_transfer_kernel(int type, int slotType, void* stream,
                                         void* dstCacheTensor, void* keyCachePtr,
                                         void* valueCachePtr,
                                         const void* slotmappings,
                                         int64_t hiddenDims, int32_t numTokens,
                                         int page2L, int tokenMajor, int isMLA,
                                         int64_t pagedRowStride,
                                         int64_t numPagedRows) {
  lmcb::clear_error();
  const char* who = "single_layer_kv_transfer";
  const int64_t esz = lmcb::dtype_size(type);
  const int64_t row = hiddenDims * esz;
  const int kvs = isMLA ? 1 : 2;
  TransferParams p{};
  p.lmc = static_cast<uint8_t*>(dstCacheTensor);
  if (isMLA) {
    p.lmc_token_stride = row;
    p.lmc_kv_stride = 0;
  } else if (tokenMajor) {
    p.lmc_token_stride = 2 * row;  // [T, 2, H]
    p.lmc_kv_stride = row;
  } else {
    p.lmc_token_stride = row;      // [2, T, H]
    p.lmc_kv_stride = row * numTokens;
  }
  p.lmc_layer_stride = 0;
  p.base_k = static_cast<uint8_t*>(keyCachePtr);
  p.base_v = static_cast<uint8_t*>(valueCachePtr);
  p.paged_row_stride = pagedRowStride > 0 ? pagedRowStride : row;
  p.num_paged_rows = numPagedRows;
  p.slots = slotmappings;
  p.num_tokens = numTokens;
  p.num_layers = 1;
  p.num_kv = kvs;
  p.row_bytes = esz == 0 ? 1 : row;
  p.page2L = page2L ? 1 : 0;
  return lmcb::launch_transfer(
      p, type, slotType, lmcb::kDirect,
      {reinterpret_cast<uint64_t>(dstCacheTensor), static_cast<uint64_t>(row),
       reinterpret_cast<uint64_t>(keyCachePtr),
       isMLA ? 0 : reinterpret_cast<uint64_t>(valueCachePtr),
       static_cast<uint64_t>(p.paged_row_stride)},
      static_cast<cudaStream_t>(stream), who);
}

int lmcb_load_and_reshape_flash_kernel(int type, int slotType, void* stream,
                                       void* dstCacheTensor, void* keyCachePtr,
                                       void* valueCachePtr,
                                       const void* slotmappings,
                                       int64_t hiddenDims, int64_t numPages,
                                       int32_t pagedSize, int32_t numTokens,
                                       int32_t numLayers, int32_t layerIdx,
                                       int page2L, int64_t pagedRowStride) {
  lmcb::clear_error();
  const char* who = page2L ? "load_and_reshape_flash" : "reshape_and_cache_back_flash";
  if (layerIdx < 0 || layerIdx >= numLayers) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      std::string(who) + ": layer_idx out of range.");
  }
  const int64_t esz = lmcb::dtype_size(type);
  const int64_t row = hiddenDims * esz;
  TransferParams p{};
  // Layer `layerIdx` of a [2, numLayers, numTokens, H] object.
  p.lmc = static_cast<uint8_t*>(dstCacheTensor) +
          static_cast<int64_t>(layerIdx) * numTokens * row;
  p.lmc_token_stride = row;
  p.lmc_layer_stride = 0;
  p.lmc_kv_stride = row * numTokens * numLayers;
  p.base_k = static_cast<uint8_t*>(keyCachePtr);
  p.base_v = static_cast<uint8_t*>(valueCachePtr);
  p.paged_row_stride = pagedRowStride > 0 ? pagedRowStride : row;
  p.num_paged_rows = numPages * static_cast<int64_t>(pagedSize);
  p.slots = slotmappings;
  p.num_tokens = numTokens;
  p.num_layers = 1;
  p.num_kv = 2;
  p.row_bytes = esz == 0 ? 1 : row;
  p.page2L = page2L ? 1 : 0;
  return lmcb::launch_transfer(
      p, type, slotType, lmcb::kDirect,
      {reinterpret_cast<uint64_t>(p.lmc), static_cast<uint64_t>(row),
       static_cast<uint64_t>(p.lmc_kv_stride),
       reinterpret_cast<uint64_t>(keyCachePtr), reinterpret_cast<uint64_t>(valueCachePtr),
       static_cast<uint64_t>(p.paged_row_stride)},
      static_cast<cudaStream_t>(stream), who);
}

int lmcb_multi_layer_kv_transfer_batched_kernel(
    int type, int slotType, void* stream, const uint64_t* pagedKVCaches,
    const uint64_t* objectPtrs, const int64_t* tokenOffsets, const int64_t* slotStarts,
    int32_t numObjects, int objectsOnDevice, const void* slotmappings, int64_t hiddenDims,
    int32_t kvs, int32_t numLayers, int64_t pageBuffSize, int32_t totalTokens, int page2L) {
  lmcb::clear_error();
  const char* who = "multi_layer_kv_transfer_batched";
  if (kvs != 1 && kvs != 2) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": kvs must be 1 or 2.");
  }
  if (kvs == 2 && pageBuffSize <= 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      std::string(who) + ": page_buffer_size must be positive for K/V caches.");
  }
  if (numObjects < 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": negative object count.");
  }
  if (numObjects == 0 || totalTokens == 0) return LMCB_OK;
  const int64_t esz = lmcb::dtype_size(type);
  const int64_t row = hiddenDims * esz;
  TransferParams p{};
  p.ptrs_k = pagedKVCaches;
  p.ptrs_v = pagedKVCaches;
  p.page_kv_offset = pageBuffSize * row;
  p.paged_row_stride = row;
  p.num_paged_rows = pageBuffSize;
  p.slots = slotmappings;
  p.num_tokens = totalTokens;
  p.num_layers = numLayers;
  p.num_kv = kvs;
  p.row_bytes = esz == 0 ? 1 : row;
  p.page2L = page2L ? 1 : 0;
  return lmcb::launch_batched(
      p, type, slotType, lmcb::kBatched,
      {static_cast<uint64_t>(row), static_cast<uint64_t>(p.page_kv_offset)},
      static_cast<cudaStream_t>(stream), who, objectsOnDevice != 0, objectPtrs, tokenOffsets,
      slotStarts, numObjects, totalTokens);
}

int lmcb_single_layer_kv_transfer_batched_kernel(
    int type, int slotType, void* stream, const uint64_t* objectPtrs,
    const int64_t* tokenOffsets, const int64_t* slotStarts, int32_t numObjects,
    int objectsOnDevice, void* keyCachePtr, void* valueCachePtr, const void* slotmappings,
    int64_t hiddenDims, int32_t totalTokens, int page2L, int tokenMajor,
    int64_t pagedRowStride, int64_t numPagedRows) {
  lmcb::clear_error();
  const char* who = "single_layer_kv_transfer_batched";
  if (numObjects < 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": negative object count.");
  }
  if (numObjects == 0 || totalTokens == 0) return LMCB_OK;
  const int64_t esz = lmcb::dtype_size(type);
  const int64_t row = hiddenDims * esz;
  TransferParams p{};
  p.base_k = static_cast<uint8_t*>(keyCachePtr);
  p.base_v = static_cast<uint8_t*>(valueCachePtr);
  p.paged_row_stride = pagedRowStride > 0 ? pagedRowStride : row;
  p.num_paged_rows = numPagedRows;
  p.slots = slotmappings;
  p.num_tokens = totalTokens;
  p.num_layers = 1;
  p.num_kv = 2;
  p.row_bytes = esz == 0 ? 1 : row;
  p.page2L = page2L ? 1 : 0;
  p.obj_token_major = tokenMajor ? 1 : 0;
  return lmcb::launch_batched(
      p, type, slotType, lmcb::kBatchedDirect,
      {static_cast<uint64_t>(row), reinterpret_cast<uint64_t>(keyCachePtr),
       reinterpret_cast<uint64_t>(valueCachePtr), static_cast<uint64_t>(p.paged_row_stride)},
      static_cast<cudaStream_t>(stream), who, objectsOnDevice != 0, objectPtrs, tokenOffsets,
      slotStarts, numObjects, totalTokens);
}

int lmcb_multi_layer_kv_store_staged(int type, int slotType, void* stream,
                                     const uint64_t* pagedKVCaches, void* hostCacheTensor,
                                     const void* hostCacheDevice, void* staging,
                                     size_t stagingBytes, const void* slotmappings,
                                     int64_t hiddenDims, int32_t kvs, int32_t numLayers,
                                     int64_t pageBuffSize, int32_t numTokensChunk) {
  lmcb::clear_error();
  const char* who = "multi_layer_kv_store_staged";
  const int64_t esz = lmcb::dtype_size(type);
  if (esz == 0) {
    return lmcb::fail(LMCB_ERR_UNSUPPORTED_DTYPE, std::string(who) + ": ScalarType not supported.");
  }
  if (kvs != 1 && kvs != 2) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": kvs must be 1 or 2.");
  }
  if (kvs == 2 && pageBuffSize <= 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      std::string(who) + ": page_buffer_size must be positive for K/V caches.");
  }
  if (numTokensChunk <= 0 || numLayers <= 0) return LMCB_OK;
  const int64_t row = hiddenDims * esz;
  if (hostCacheTensor == nullptr || hostCacheDevice == nullptr || staging == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL pointer.");
  }
  uint64_t bytes = 0;
  if (!lmcb::object_bytes(kvs, numLayers, numTokensChunk, hiddenDims, esz, &bytes)) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": object size overflows.");
  }
  if (stagingBytes < bytes) {
    return lmcb::fail(LMCB_ERR_CAPACITY,
                      std::string(who) + ": staging buffer holds " + std::to_string(stagingBytes) +
                          " bytes, the object needs " + std::to_string(bytes));
  }
  TransferParams p{};
  p.lmc = static_cast<uint8_t*>(staging);
  p.lmc_token_stride = row;
  p.lmc_layer_stride = row * numTokensChunk;
  p.lmc_kv_stride = p.lmc_layer_stride * numLayers;
  p.ptrs_k = pagedKVCaches;
  p.ptrs_v = pagedKVCaches;
  p.page_kv_offset = pageBuffSize * row;
  p.paged_row_stride = row;
  p.num_paged_rows = pageBuffSize;
  p.slots = slotmappings;
  p.num_tokens = numTokensChunk;
  p.num_layers = numLayers;
  p.num_kv = kvs;
  p.row_bytes = row;
  p.page2L = 1;
  p.fallback = static_cast<const uint8_t*>(hostCacheDevice);
  // The gather reads skipped rows from host memory, so it runs on the
  // vectorised kernel (the bulk-copy path only addresses device memory).
  const int rc = lmcb::launch_transfer(
      p, type, slotType, lmcb::kPtrArray,
      {reinterpret_cast<uint64_t>(staging), static_cast<uint64_t>(row),
       static_cast<uint64_t>(p.page_kv_offset), reinterpret_cast<uint64_t>(hostCacheDevice)},
      static_cast<cudaStream_t>(stream), who, false, /*force_vector=*/true);
  if (rc != LMCB_OK) return rc;
  LMCB_CUDA_TRY(cudaMemcpyAsync(hostCacheTensor, staging, bytes, cudaMemcpyDeviceToHost,
                                static_cast<cudaStream_t>(stream)));
  return LMCB_OK;
}

int lmcb_multi_layer_kv_retrieve_staged(int type, int slotType, void* stream,
                                        const uint64_t* pagedKVCaches,
                                        const void* hostCacheTensor,
                                        void* staging, size_t stagingBytes,
                                        const void* slotmappings,
                                        int64_t hiddenDims, int32_t kvs,
                                        int32_t numLayers, int64_t pageBuffSize,
                                        int32_t numTokensChunk) {
  lmcb::clear_error();
  const char* who = "multi_layer_kv_retrieve_staged";
  // Every argument the scatter would reject is rejected here, before the
  // copy into the staging buffer is queued: a failed call leaves the buffer
  // as it was.
  const int64_t esz = lmcb::dtype_size(type);
  if (esz == 0) {
    return lmcb::fail(LMCB_ERR_UNSUPPORTED_DTYPE, std::string(who) + ": ScalarType not supported.");
  }
  if (slotType != LMCB_DTYPE_INT64 && slotType != LMCB_DTYPE_INT32) {
    return lmcb::fail(LMCB_ERR_UNSUPPORTED_DTYPE,
                      std::string(who) + ": slot ids must be int64 or int32.");
  }
  if (kvs != 1 && kvs != 2) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": kvs must be 1 or 2.");
  }
  if (kvs == 2 && pageBuffSize <= 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT,
                      std::string(who) + ": page_buffer_size must be positive for K/V caches.");
  }
  if (hiddenDims <= 0 || numTokensChunk < 0 || numLayers < 0) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": negative size.");
  }
  if (numTokensChunk == 0 || numLayers == 0) return LMCB_OK;
  if (hostCacheTensor == nullptr || staging == nullptr || pagedKVCaches == nullptr ||
      slotmappings == nullptr) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL pointer.");
  }
  uint64_t bytes = 0;
  if (!lmcb::object_bytes(kvs, numLayers, numTokensChunk, hiddenDims, esz, &bytes)) {
    return lmcb::fail(LMCB_ERR_INVALID_ARGUMENT, std::string(who) + ": object size overflows.");
  }
  if (stagingBytes < bytes) {
    return lmcb::fail(LMCB_ERR_CAPACITY,
                      "multi_layer_kv_retrieve_staged: staging buffer holds " +
                          std::to_string(stagingBytes) + " bytes, the object needs " +
                          std::to_string(bytes));
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LMCB_CUDA_TRY(cudaMemcpyAsync(staging, hostCacheTensor, bytes, cudaMemcpyHostToDevice, s));
  return lmcb_multi_layer_kv_transfer_kernel(type, slotType, stream, pagedKVCaches, staging,
                                             slotmappings, hiddenDims, kvs, numLayers,
                                             pageBuffSize, numTokensChunk, 0);
}

}  // extern "C"
