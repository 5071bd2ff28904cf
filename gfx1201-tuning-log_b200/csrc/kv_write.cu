// Paged KV-cache write for sm_100a: bf16 K/V rows of the new tokens ->
// per-tensor-scaled fp8 e4m3 (or bf16) slots of the paged cache.
//
// The reference relies on vLLM's reshape_and_cache_flash for this step
// (profiling/prof_h4mv.txt:9); the contract kept here is that op's:
// slot = slot_mapping[t] (negative = padding token, skipped), block = slot /
// block_size, offset = slot % block_size, and the fp8 value is
// cvt.rn.satfinite.e4m3(float(x) / scale) -- IEEE fp32 division, round to
// nearest even, saturation to +-448.  For |x / scale| <= 448 this is bit-exact
// with torch's (x.float() / scale).to(torch.float8_e4m3fn).
//
// HBM-bound streaming: one CTA per token, each thread moves 16 output bytes
// (16 fp8 from 32 bytes of bf16) with 128-bit loads and stores.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace b200kv {
namespace {

struct KvWriteParams {
  const __nv_bfloat16* key;
  const __nv_bfloat16* value;
  int64_t k_st, k_sh, v_st, v_sh;  // elements
  uint8_t* kc;
  uint8_t* vc;
  int64_t sk0, sk1, sk2, sv0, sv1, sv2;  // bytes
  const int64_t* slots;
  const float* k_scale;
  const float* v_scale;
  int hkv, head_dim, block_size;
};

__device__ __forceinline__ uint32_t quant4(const __nv_bfloat16* x, float scale) {
  // 4 bf16 -> 4 e4m3 bytes
  float f[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = __fdiv_rn(__bfloat162float(x[i]), scale);
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[0], f[1]), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f[2], f[3]), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

template <bool FP8>
__global__ void __launch_bounds__(256) kv_write_kernel(const KvWriteParams p) {
  const int t = blockIdx.x;
  const int64_t slot = p.slots[t];
  if (slot < 0) return;
  const int64_t blk = slot / p.block_size;
  const int64_t off = slot % p.block_size;
  constexpr int EPT = FP8 ? 16 : 8;  // elements per thread (16 output bytes)
  const int per_head = p.head_dim / EPT;
  const int per_tensor = p.hkv * per_head;
  const float ks = FP8 ? __ldg(p.k_scale) : 1.f;
  const float vs = FP8 ? __ldg(p.v_scale) : 1.f;
  for (int i = threadIdx.x; i < 2 * per_tensor; i += blockDim.x) {
    const bool is_v = i >= per_tensor;
    const int j = is_v ? i - per_tensor : i;
    const int h = j / per_head;
    const int d0 = (j % per_head) * EPT;
    const __nv_bfloat16* src = is_v ? p.value + (int64_t)t * p.v_st + (int64_t)h * p.v_sh + d0
                                    : p.key + (int64_t)t * p.k_st + (int64_t)h * p.k_sh + d0;
    uint8_t* dst = is_v ? p.vc + blk * p.sv0 + off * p.sv1 + h * p.sv2 + d0 * (FP8 ? 1 : 2)
                        : p.kc + blk * p.sk0 + off * p.sk1 + h * p.sk2 + d0 * (FP8 ? 1 : 2);
    if constexpr (FP8) {
      __align__(16) __nv_bfloat16 x[16];
      *reinterpret_cast<uint4*>(x) = *reinterpret_cast<const uint4*>(src);
      *reinterpret_cast<uint4*>(x + 8) = *reinterpret_cast<const uint4*>(src + 8);
      const float sc = is_v ? vs : ks;
      uint4 o;
      o.x = quant4(x, sc);
      o.y = quant4(x + 4, sc);
      o.z = quant4(x + 8, sc);
      o.w = quant4(x + 12, sc);
      *reinterpret_cast<uint4*>(dst) = o;
    } else {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }
}

}  // namespace

int kv_write_launch(const void* key, int64_t k_st, int64_t k_sh, const void* value, int64_t v_st,
                    int64_t v_sh, void* k_cache, void* v_cache, int64_t sk0, int64_t sk1,
                    int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, const int64_t* slots,
                    const float* k_scale, const float* v_scale, int num_tokens, int hkv,
                    int head_dim, int block_size, int kv_dtype, void* stream) {
  if (!key || !value || !k_cache || !v_cache || !slots) return B200KV_ERR_INVALID_ARG;
  if (num_tokens < 0 || hkv <= 0 || head_dim <= 0 || block_size <= 0) return B200KV_ERR_INVALID_ARG;
  if (kv_dtype != B200KV_KV_FP8_E4M3 && kv_dtype != B200KV_KV_BF16) return B200KV_ERR_UNSUPPORTED;
  const bool fp8 = kv_dtype == B200KV_KV_FP8_E4M3;
  if (fp8 && (!k_scale || !v_scale)) return B200KV_ERR_INVALID_ARG;
  if (head_dim % 16) return B200KV_ERR_UNSUPPORTED;
  const int esz = fp8 ? 1 : 2;
  const int64_t cs[6] = {sk0, sk1, sk2, sv0, sv1, sv2};
  for (int i = 0; i < 6; ++i)
    if ((cs[i] * esz) % 16) return B200KV_ERR_MISALIGNED;
  const int64_t xs[4] = {k_st, k_sh, v_st, v_sh};
  for (int i = 0; i < 4; ++i)
    if (xs[i] % 8) return B200KV_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
       reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return B200KV_ERR_MISALIGNED;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  if (num_tokens == 0) return B200KV_OK;
  KvWriteParams p;
  p.key = static_cast<const __nv_bfloat16*>(key);
  p.value = static_cast<const __nv_bfloat16*>(value);
  p.k_st = k_st; p.k_sh = k_sh; p.v_st = v_st; p.v_sh = v_sh;
  p.kc = static_cast<uint8_t*>(k_cache);
  p.vc = static_cast<uint8_t*>(v_cache);
  p.sk0 = sk0 * esz; p.sk1 = sk1 * esz; p.sk2 = sk2 * esz;
  p.sv0 = sv0 * esz; p.sv1 = sv1 * esz; p.sv2 = sv2 * esz;
  p.slots = slots;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.hkv = hkv;
  p.head_dim = head_dim;
  p.block_size = block_size;
  const int work = 2 * hkv * head_dim / (fp8 ? 16 : 8);
  const int threads = work >= 256 ? 256 : ((work + 31) / 32) * 32;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fp8)
    kv_write_kernel<true><<<num_tokens, threads, 0, st>>>(p);
  else
    kv_write_kernel<false><<<num_tokens, threads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
