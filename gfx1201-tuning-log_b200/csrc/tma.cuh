// Tensor-memory-accelerator helpers: host-side tensor-map encoding (through the
// driver entry point, no libcuda link dependency) and the device-side tiled
// load.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200kv_common.cuh"

namespace b200kv {

// Encodes a 2-D uint8 tensor map over a row-major [rows, row_bytes] matrix with
// row pitch `pitch` bytes and box [box_x bytes, box_y rows].  Returns false when
// the driver entry point is unavailable or the driver rejects the map.
bool encode_u8_2d(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                  uint64_t pitch, uint32_t box_x, uint32_t box_y, bool swizzle128);

// Encodes a 2-D tensor map over packed e2m1 codes [rows, row_elems] (two codes
// a byte, row pitch `pitch` bytes) that the TMA unpacks on the way into shared
// memory: every 8 bytes (16 codes) land in a 16-byte chunk, the operand layout
// of 4-bit types in tcgen05 kind::f8f6f4 / mxf8f6f4 MMAs.  Box [128 codes, box_rows
// rows] with 128-byte swizzle: 128 bytes of shared memory per row, of which the
// TMA signals the 64 packed bytes on the mbarrier.  x coordinates count codes.
bool encode_e2m1_unpacked_2d(CUtensorMap* map, const void* base, uint64_t row_elems, uint64_t rows,
                             uint64_t pitch, uint32_t box_rows);

// 2-D tiled TMA load of the box at (x bytes, y rows) into shared memory,
// completion counted on `bar`.  x must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Encodes a 4-D uint8 tensor map over a paged KV cache [blocks][tokens][heads][row]
// (row = one head's `row_bytes`, byte strides s_head < s_tok < s_blk) with box
// [row_bytes, 1 head, `tokens` tokens, 1 block] and 128-byte swizzle, so one
// load brings one head's rows of one page into shared memory as a swizzled
// [tokens][row_bytes] tile.  row_bytes must be 128.  Out-of-range block ids
// read as zeros.
bool encode_paged_kv(CUtensorMap* map, const void* base, uint32_t row_bytes, uint32_t heads,
                     uint32_t tokens, uint64_t blocks, uint64_t s_head, uint64_t s_tok,
                     uint64_t s_blk);


// 4-D tiled TMA load of the box at (c0 bytes, c1, c2, c3), completion counted on
// `bar`.  c0 must be a multiple of 16.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

// Prefetch of the 4-D box at (c0, c1, c2, c3) into L2 (no shared memory, no
// barrier).  L2 is the point of coherence for device memory, so a prefetch
// issued before a producer kernel's writes land can never serve stale data.
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2,
                                                   int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Prefetch of the 2-D box at (x, y) into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// Prefetch of `bytes` (a multiple of 16) at a 16-byte-aligned global address into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace b200kv
