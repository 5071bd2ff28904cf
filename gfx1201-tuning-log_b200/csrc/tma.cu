// Host side of tma.cuh: tensor-map encoding through cudaGetDriverEntryPoint.
#include <cudaTypedefs.h>
#include <mutex>

#include "tma.cuh"

namespace b200kv {
namespace {

PFN_cuTensorMapEncodeTiled get_encode() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

}  // namespace

bool encode_u8_2d(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                  uint64_t pitch, uint32_t box_x, uint32_t box_y, bool swizzle128) {
  PFN_cuTensorMapEncodeTiled enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_x, box_y};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_e2m1_unpacked_2d(CUtensorMap* map, const void* base, uint64_t row_elems, uint64_t rows,
                             uint64_t pitch, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled enc = get_encode();
  if (!enc || row_elems % 128 || (pitch & 15) || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[2] = {row_elems, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_paged_kv(CUtensorMap* map, const void* base, uint32_t row_bytes, uint32_t heads,
                     uint32_t tokens, uint64_t blocks, uint64_t s_head, uint64_t s_tok,
                     uint64_t s_blk) {
  PFN_cuTensorMapEncodeTiled enc = get_encode();
  if (!enc || row_bytes != 128 || tokens == 0 || tokens > 256 || blocks == 0) return false;
  if ((s_head | s_tok | s_blk) & 15) return false;
  const cuuint64_t dims[4] = {row_bytes, heads, tokens, blocks};
  const cuuint64_t strides[3] = {s_head, s_tok, s_blk};
  const cuuint32_t box[4] = {row_bytes, 1, tokens, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace b200kv
