/*
 * lmcache_b200.h -- C ABI of the B200 (sm_100a) paged KV-cache transfer library.
 *
 * Plain pointers, sizes and enums only: no torch or pybind types cross this
 * boundary. Every entry point returns an lmcb_status (0 = success); on failure a
 * thread-local message is available from lmcb_last_error().
 *
 * The transfer entry points are the B200 replacements of the device-kernel
 * launch functions that LMCache-Ascend's host launchers bind:
 *   kvcache_ops::multi_layer_kv_transfer_kernel   csrc/mem_kernels.h:8-12
 *   kvcache_ops::single_layer_kv_transfer_kernel  csrc/mem_kernels.h:14-18
 *   kvcache_ops::load_and_reshape_flash_kernel    csrc/mem_kernels.h:20-24
 * with the same argument meaning and order, minus the Ascend `blockDim`
 * (the library sizes its own grid from the SM count of the current device).
 * Pointers may be device pointers or device-mapped pinned host pointers
 * (see lmcb_host_register). Launches are asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream).
 *
 * Address rules shared by the transfer entry points (a "row" is one token's
 * hidden_dims elements of one of K, V or the MLA latent):
 *   paged side   row(layer, kv, slot) = pagedKVCaches[layer]
 *                                        + (kv * pageBuffSize + slot) * row_bytes
 *   LMCache side row(kv, layer, t)    = dstCacheTensor
 *                                        + ((kv * numLayers + layer) * numTokens + t) * row_bytes
 *   page2L != 0 copies paged -> LMCache (store / offload);
 *   page2L == 0 copies LMCache -> paged (retrieve / load back).
 *   A slot < 0 is skipped: the destination row is left unchanged.
 *   A slot >= the paged side's row count (when the entry point knows it)
 *   is skipped and sets LMCB_DEVICE_FLAG_SLOT_OUT_OF_RANGE in the device's
 *   status word (lmcb_device_status), so no access leaves the buffers.
 */
#ifndef LMCACHE_B200_H_
#define LMCACHE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LMCB_API __attribute__((visibility("default")))
#else
#define LMCB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
typedef enum {
  LMCB_OK = 0,
  LMCB_ERR_INVALID_ARGUMENT = 1,
  LMCB_ERR_UNSUPPORTED_DTYPE = 2,
  LMCB_ERR_CUDA = 3,
  LMCB_ERR_NOT_REGISTERED = 4,
  LMCB_ERR_NOT_IMPLEMENTED = 5,
  LMCB_ERR_CAPACITY = 6
} lmcb_status;

/* Element / slot types. Same set and meaning as the reference's dtype map
 * (csrc/utils.h:22-38: FP32, BF16, FP16 data; INT64, INT32 slot ids). */
typedef enum {
  LMCB_DTYPE_FP32 = 0,
  LMCB_DTYPE_BF16 = 1,
  LMCB_DTYPE_FP16 = 2,
  LMCB_DTYPE_INT64 = 3,
  LMCB_DTYPE_INT32 = 4
} lmcb_dtype;

/* Bits of the per-device status word. */
#define LMCB_DEVICE_FLAG_SLOT_OUT_OF_RANGE 0x1u
#define LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE 0x2u
#define LMCB_DEVICE_FLAG_STREAM_OVERFLOW 0x4u
#define LMCB_DEVICE_FLAG_WAIT_TIMEOUT 0x8u
#define LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE 0x10u

/* Library version, "major.minor.patch". */
LMCB_API const char* lmcb_version(void);

/* Message of the last failing call on this thread ("" if none). */
LMCB_API const char* lmcb_last_error(void);

/* Short name of a status code. */
LMCB_API const char* lmcb_status_string(int status);

/* Size in bytes of one element of `dtype`, or 0 if unknown. */
LMCB_API int lmcb_dtype_size(int dtype);

/* ------------------------------------------------------------------------- */
/* Paged KV transfer                                                          */
/* ------------------------------------------------------------------------- */

/* All layers of one chunk in one launch.
 * Replaces kvcache_ops::multi_layer_kv_transfer_kernel (csrc/mem_kernels.h:8-12),
 * launched by multi_layer_kv_transfer (csrc/mem_kernels.cpp:48-92).
 *   type            element type of both sides (lmcb_dtype)
 *   slotType        LMCB_DTYPE_INT64 or LMCB_DTYPE_INT32
 *   stream          cudaStream_t
 *   pagedKVCaches   device-readable array of numLayers uint64 base addresses,
 *                   each a [kvs, pageBuffSize, hiddenDims] buffer
 *   dstCacheTensor  LMCache object [kvs, numLayers, numTokensChunk, hiddenDims]
 *   slotmappings    device-readable [numTokensChunk] slot ids
 *   hiddenDims      elements per row
 *   kvs             2 (K and V) or 1 (MLA latent)
 *   pageBuffSize    rows per K or V half of a layer buffer (num_blocks *
 *                   block_size). With kvs == 1 it may be 0 (unknown, as the
 *                   reference's MLA callers pass it); then no slot bound is checked.
 *   page2L          non-zero: paged -> LMCache; zero: LMCache -> paged */
LMCB_API int lmcb_multi_layer_kv_transfer_kernel(int type, int slotType, void* stream,
                                        const uint64_t* pagedKVCaches,
                                        void* dstCacheTensor,
                                        const void* slotmappings,
                                        int64_t hiddenDims, int32_t kvs,
                                        int32_t numLayers, int64_t pageBuffSize,
                                        int32_t numTokensChunk, int page2L);

/* As lmcb_multi_layer_kv_transfer_kernel with separate K and V base-address
 * arrays (each [numLayers] uint64; a layer's K rows at keyPtrs[layer] +
 * slot * row_bytes, V rows at valuePtrs[layer] + slot * row_bytes).
 * Implements multi_layer_kv_transfer_unilateral, which the reference leaves
 * unimplemented (csrc/mem_kernels.cpp:95-105). pageBuffSize bounds the slot
 * (0 = unchecked). */
LMCB_API int lmcb_multi_layer_kv_transfer_unilateral_kernel(
    int type, int slotType, void* stream, const uint64_t* keyPtrs,
    const uint64_t* valuePtrs, void* dstCacheTensor, const void* slotmappings,
    int64_t hiddenDims, int32_t numLayers, int64_t pageBuffSize,
    int32_t numTokensChunk, int page2L);

/* Many chunks in one launch: the objects of a request that LMCache stores or
 * retrieves together (upstream LMCache drives them through the connector's
 * batched_from_gpu / batched_to_gpu, one multi_layer_kv_transfer per chunk;
 * this moves all of them with one kernel). Object i is a
 * [kvs, numLayers, T_i, hiddenDims] LMCache object at objectPtrs[i] and
 * holds T_i = tokenOffsets[i+1] - tokenOffsets[i] tokens whose slot ids are
 * slotmappings[slotStarts[i] ... slotStarts[i] + T_i). Per row the result is
 * that of lmcb_multi_layer_kv_transfer_kernel on each object in turn.
 *   objectPtrs, tokenOffsets ([numObjects + 1], ascending,
 *   tokenOffsets[numObjects] - tokenOffsets[0] = totalTokens), slotStarts:
 *   HOST arrays, read during the call. The table travels in the kernel
 *   parameters (up to 255 objects per launch; larger batches are split into
 *   several launches), so nothing is copied to the device before the launch
 *   and the call can be captured in a CUDA graph.
 *   objectsOnDevice  1 if every object is device memory (the bulk-copy kernel
 *                    may then be chosen), 0 if any is host memory (zero-copy) */
LMCB_API int lmcb_multi_layer_kv_transfer_batched_kernel(
    int type, int slotType, void* stream, const uint64_t* pagedKVCaches,
    const uint64_t* objectPtrs, const int64_t* tokenOffsets, const int64_t* slotStarts,
    int32_t numObjects, int objectsOnDevice, const void* slotmappings, int64_t hiddenDims,
    int32_t kvs, int32_t numLayers, int64_t pageBuffSize, int32_t totalTokens, int page2L);

/* single_layer_kv_transfer for many objects in one launch (the layerwise
 * connector moves every chunk of a request for one layer this way, where the
 * reference issues one call per chunk, npu_connector.py:227-252). Object i
 * (at objectPtrs[i]) holds T_i = tokenOffsets[i+1] - tokenOffsets[i] tokens
 * with slot ids slotmappings[slotStarts[i] ... + T_i), laid out [T_i, 2,
 * hiddenDims] if tokenMajor else [2, T_i, hiddenDims]. Caches, strides and
 * bounds as in lmcb_single_layer_kv_transfer_kernel; the object table (host
 * arrays) and objectsOnDevice as in lmcb_multi_layer_kv_transfer_batched_kernel. */
LMCB_API int lmcb_single_layer_kv_transfer_batched_kernel(
    int type, int slotType, void* stream, const uint64_t* objectPtrs,
    const int64_t* tokenOffsets, const int64_t* slotStarts, int32_t numObjects,
    int objectsOnDevice, void* keyCachePtr, void* valueCachePtr, const void* slotmappings,
    int64_t hiddenDims, int32_t totalTokens, int page2L, int tokenMajor,
    int64_t pagedRowStride, int64_t numPagedRows);

/* One layer, separate K and V caches.
 * Replaces kvcache_ops::single_layer_kv_transfer_kernel (csrc/mem_kernels.h:14-18),
 * launched by single_layer_kv_transfer (csrc/mem_kernels.cpp:108-152).
 *   dstCacheTensor  [numTokens, 2, hiddenDims] if tokenMajor else
 *                   [2, numTokens, hiddenDims]  (isMLA: [numTokens, hiddenDims])
 *   keyCachePtr     K rows; row `slot` at keyCachePtr + slot * pagedRowStride bytes
 *   valueCachePtr   V rows, same addressing (ignored when isMLA)
 *   pagedRowStride  bytes between consecutive slots of the caches (0 = row_bytes)
 *   numPagedRows    rows in each cache (num_blocks * block_size; 0 = unchecked) */
LMCB_API int lmcb_single_layer_kv_transfer_kernel(int type, int slotType, void* stream,
                                         void* dstCacheTensor, void* keyCachePtr,
                                         void* valueCachePtr,
                                         const void* slotmappings,
                                         int64_t hiddenDims, int32_t numTokens,
                                         int page2L, int tokenMajor, int isMLA,
                                         int64_t pagedRowStride,
                                         int64_t numPagedRows);

/* One layer `layerIdx` of a [2, numLayers, numTokens, hiddenDims] LMCache object
 * against [numPages, pagedSize, heads, head_dim] K and V caches.
 * Replaces kvcache_ops::load_and_reshape_flash_kernel (csrc/mem_kernels.h:20-24),
 * launched by load_and_reshape_flash (page2L = 1, csrc/mem_kernels.cpp:154-198)
 * and reshape_and_cache_back_flash (page2L = 0, csrc/mem_kernels.cpp:200-245).
 *   pagedRowStride  bytes between consecutive slots of the caches (0 = row_bytes) */
LMCB_API int lmcb_load_and_reshape_flash_kernel(int type, int slotType, void* stream,
                                       void* dstCacheTensor, void* keyCachePtr,
                                       void* valueCachePtr,
                                       const void* slotmappings,
                                       int64_t hiddenDims, int64_t numPages,
                                       int32_t pagedSize, int32_t numTokens,
                                       int32_t numLayers, int32_t layerIdx,
                                       int page2L, int64_t pagedRowStride);

/* Retrieve (LMCache -> paged) from a pinned host LMCache object through one
 * host-to-device DMA into a caller-provided device staging buffer, followed
 * by an HBM scatter. Same result as lmcb_multi_layer_kv_transfer_kernel with
 * page2L == 0; the staging buffer must hold the whole object
 * (kvs * numLayers * numTokensChunk * hiddenDims elements). Every argument is
 * checked before the copy is queued, so a call that returns an error leaves
 * the staging buffer untouched.
 *   hostCacheTensor  pinned host address of the LMCache object
 *   staging          device scratch, stagingBytes long, 16-byte aligned */
LMCB_API int lmcb_multi_layer_kv_retrieve_staged(int type, int slotType, void* stream,
                                        const uint64_t* pagedKVCaches,
                                        const void* hostCacheTensor,
                                        void* staging, size_t stagingBytes,
                                        const void* slotmappings,
                                        int64_t hiddenDims, int32_t kvs,
                                        int32_t numLayers, int64_t pageBuffSize,
                                        int32_t numTokensChunk);

/* Store (paged -> LMCache) into a pinned host LMCache object through a
 * caller-provided device staging buffer and one device-to-host DMA, instead of
 * zero-copy kernel writes. Same result as lmcb_multi_layer_kv_transfer_kernel
 * with page2L != 0: a row whose slot is skipped is first read from the host
 * object (through hostCacheDevice, its device-mapped alias) into the staging
 * buffer, so the copy back leaves it unchanged.
 *   hostCacheTensor  host address of the object (DMA destination)
 *   hostCacheDevice  device-mapped alias of the same object (lmcb_host_register)
 *   staging          device scratch of stagingBytes >= the object's size */
LMCB_API int lmcb_multi_layer_kv_store_staged(int type, int slotType, void* stream,
                                              const uint64_t* pagedKVCaches,
                                              void* hostCacheTensor,
                                              const void* hostCacheDevice, void* staging,
                                              size_t stagingBytes, const void* slotmappings,
                                              int64_t hiddenDims, int32_t kvs,
                                              int32_t numLayers, int64_t pageBuffSize,
                                              int32_t numTokensChunk);

/* Size of the staging area that lmcb_multi_layer_kv_retrieve_staged_noalloc
 * keeps on every GPU where the library is loaded (64 MiB). */
#define LMCB_NOALLOC_STAGING_BYTES (64u << 20)

/* The staged retrieve of lmcb_multi_layer_kv_retrieve_staged for callers
 * that cannot allocate device memory when they retrieve. Examples: an engine
 * that reserved almost all HBM for its paged KV cache up front, or a native
 * host without a caching allocator, where a cudaMalloc / cudaFree per chunk
 * would synchronise the device. No reference counterpart: the reference has
 * no staged retrieve.
 * Instead of a caller buffer it uses a staging area of
 * LMCB_NOALLOC_STAGING_BYTES built into the library (a device array that every
 * GPU loading the library holds until exit); it calls no allocator.
 * Objects larger than the area are rejected with LMCB_ERR_CAPACITY before
 * any work is queued. The first call on each device looks up the area's
 * device address (with that device current); make that first call before any
 * stream capture. All calls share the one area: calls whose copies and
 * scatters overlap on the GPU (different streams, no ordering between them)
 * race on it, so order them, for example by issuing them on one stream.
 * Nothing needs to be cleared between calls: each call writes every staging
 * byte it later reads. The area's address is kept per device ordinal for the
 * life of the process, so calling cudaDeviceReset while the library is in use
 * is not supported. */
LMCB_API int lmcb_multi_layer_kv_retrieve_staged_noalloc(
    int type, int slotType, void* stream, const uint64_t* pagedKVCaches,
    const void* hostCacheTensor, const void* slotmappings, int64_t hiddenDims, int32_t kvs,
    int32_t numLayers, int64_t pageBuffSize, int32_t numTokensChunk);

/* Reads and clears the status word of `device` (LMCB_DEVICE_FLAG_* bits).
 * Synchronous with respect to that device's legacy default stream. */
LMCB_API int lmcb_device_status(int device, uint32_t* flags_out);

/* ------------------------------------------------------------------------- */
/* Host memory registration                                                   */
/* ------------------------------------------------------------------------- */

/* Registers [hostPtr, hostPtr + bytes) for device access and returns the
 * device-side alias. Already CUDA-pinned memory is recorded as is; pageable
 * memory is page-locked and mapped. Registering the same pointer twice returns
 * the first record. Replaces HostRegisteredMemoryManager::registerHostPtr
 * (csrc/managed_mem.h:44, csrc/managed_mem.cpp:59-77). */
LMCB_API int lmcb_host_register(void* hostPtr, size_t bytes, void** devPtrOut);

/* Drops the record of hostPtr (and unpins it if this library pinned it).
 * Replaces HostRegisteredMemoryManager::unregisterMemory
 * (csrc/managed_mem.cpp:118-125). Unknown pointers are not an error. */
LMCB_API int lmcb_host_unregister(void* hostPtr);

/* Device alias of any address inside a registered range, or NULL.
 * Replaces get_device_ptr / HostRegisteredMemoryManager::getDevicePtr
 * (csrc/managed_mem.h:69, csrc/managed_mem.cpp:134-155). */
LMCB_API void* lmcb_host_get_device_ptr(void* hostPtr);

/* Size of the registered range containing hostPtr, or 0.
 * Replaces HostRegisteredMemoryManager::getRecordSize
 * (csrc/managed_mem.cpp:158-174). */
LMCB_API size_t lmcb_host_record_size(void* hostPtr);

/* Drops every record. Replaces HostRegisteredMemoryManager::unregisterAll
 * (csrc/managed_mem.cpp:43-55). */
LMCB_API int lmcb_host_unregister_all(void);

/* ------------------------------------------------------------------------- */
/* CacheGen codec                                                             */
/* ------------------------------------------------------------------------- */
/* Symbols are int8 values in [0, maxBins), laid out [numLayers, numTokens,
 * numChannels]. A CDF is int16 [numLayers, numChannels, maxBins + 1] holding
 * unsigned 16-bit values: cdf[0] = 0, cdf[maxBins] = 1 << 15, every symbol's
 * frequency cdf[s+1] - cdf[s] >= 1. Each (layer, channel) stream is coded
 * independently with a carry-less byte-oriented range coder over 15-bit
 * frequencies. The reference entry points are unimplemented stubs
 * (csrc/cachegen_kernels.cpp:7-32); the format is defined by this library. */

/* Replaces calculate_cdf (csrc/cachegen_kernels.h:16). cdfOut is device
 * int16 [numLayers, numChannels, maxBins + 1]. 1 <= maxBins <= 256. */
LMCB_API int lmcb_calculate_cdf(const int8_t* input, int16_t* cdfOut, int32_t numLayers,
                       int32_t numTokens, int32_t numChannels, int32_t maxBins,
                       void* stream);

/* Replaces encode_cuda_new (csrc/cachegen_kernels.h:7-8).
 *   outputBuffer   uint8 [numLayers, numChannels, bufferStride]
 *   outputLengths  int32 [numLayers, numChannels] bytes written per stream
 * A stream that does not fit in bufferStride bytes is truncated, its length
 * is reported as -1 and LMCB_DEVICE_FLAG_STREAM_OVERFLOW is set. */
LMCB_API int lmcb_encode(const int16_t* cdf, const int8_t* inputSym, uint8_t* outputBuffer,
                int32_t* outputLengths, int32_t numLayers, int32_t numTokens,
                int32_t numChannels, int32_t maxBins, int64_t bufferStride,
                void* stream);

/* Replaces decode_cuda_new (csrc/cachegen_kernels.h:10-11).
 *   bytestreams  uint8 [numLayers, numChannels, bufferStride]
 *   lengths      int32 [numLayers, numChannels]
 *   output       int8 [numLayers, numTokens, numChannels] */
LMCB_API int lmcb_decode(const int16_t* cdf, const uint8_t* bytestreams,
                const int32_t* lengths, int8_t* output, int32_t numLayers,
                int32_t numTokens, int32_t numChannels, int32_t maxBins,
                int64_t bufferStride, void* stream);

/* Replaces decode_cuda_prefsum (csrc/cachegen_kernels.h:13-14): the streams
 * are concatenated in (layer, channel) order in a buffer of streamBytes
 * bytes; stream i spans [i == 0 ? 0 : endOffsets[i-1], endOffsets[i])
 * (inclusive prefix sums of the stream lengths, int64
 * [numLayers * numChannels]). Offsets are clamped to [0, streamBytes]. */
LMCB_API int lmcb_decode_prefsum(const int16_t* cdf, const uint8_t* bytestreams,
                                 int64_t streamBytes, const int64_t* endOffsets,
                                 int8_t* output, int32_t numLayers, int32_t numTokens,
                                 int32_t numChannels, int32_t maxBins, void* stream);

/* ------------------------------------------------------------------------- */
/* CacheBlend: fused K re-rotation                                            */
/* ------------------------------------------------------------------------- */

/* Replaces rotary_embedding_k_fused (csrc/pos_kernels.h:7-10; unimplemented
 * in the reference, csrc/pos_kernels.cpp:7-14). Rotates, in place, the rotary
 * dims of every head of every token of `key` from the angles of
 * oldPositions[t] to those of newPositions[t]: the same result as undoing the
 * rotary embedding at the old position and applying it at the new one, with
 * one rounding to the key's type.
 *   key          [numTokens, numHeads, headSize] elements of keyType; tokens
 *                keyTokenStride elements apart, heads headSize apart
 *   cosSinCache  [maxPosition, rotDim] of cacheType, each row [cos | sin]
 *   isNeox       non-zero: pairs (i, i + rotDim/2); zero: pairs (2i, 2i + 1)
 * Positions outside [0, maxPosition) leave their token unchanged and set
 * LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE. */
LMCB_API int lmcb_rotary_embedding_k_fused(const void* oldPositions, const void* newPositions,
                                           int posType, void* key, int keyType,
                                           int64_t numTokens, int64_t numHeads,
                                           int64_t headSize, int64_t keyTokenStride,
                                           const void* cosSinCache, int cacheType,
                                           int64_t rotDim, int64_t maxPosition, int isNeox,
                                           void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* LMCACHE_B200_H_ */
