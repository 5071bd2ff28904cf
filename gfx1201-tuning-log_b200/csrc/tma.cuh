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

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace b200kv
