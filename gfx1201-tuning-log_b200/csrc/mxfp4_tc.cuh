// Shared pieces of the MXFP4 kernels on block-scaled tcgen05 MMAs (sm_100a):
// the kind::mxf8f6f4 instruction (A = e2m1 weights, B = e4m3 activation terms,
// e8m0 scales from tensor memory), the 512-byte scale-factor atom and its copy
// to tensor memory, and the exact two-term e4m3 split of bf16 activations.
//
// Scale-factor atom: 128 rows x 4 groups of 32 k, byte 16 (row % 32) +
// 4 (row / 32) + group (the tcgen05 scale-factor layout for block32, copied
// with tcgen05.cp 32x128b.warpx4 into 4 tensor-memory columns).
//
// Two-term split of a 32-element block of bf16 values (B operand):
//   x = t0 * 2^(s0-127) + t1 * 2^(s1-127),  t0, t1 e4m3,
// where s0 maps the block maximum into [128, 256) and t0 = RN_e4m3(x / 2^(s0-127))
// keeps the top four significant bits of every element; the remainder has at most
// four more (a bf16 value has eight) and t1 takes it with its own scale.  Both
// terms are exact for every element within 2^-13 of the block maximum; below
// that the product loses at most 2^-21 of the block maximum.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "b200kv_common.cuh"

namespace b200kv {
namespace mx {

constexpr int kAtom = 512;  // scale-factor atom bytes

// instruction descriptor, kind::mxf8f6f4 block-scaled: A e2m1 (format 5 of this
// kind), B e4m3 (format 0), both K-major, e8m0 scales, scale-factor byte ids
// (0..3: one byte per MMA, K = 32)
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(int M, int N, uint32_t sf_id) {
  return (sf_id << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | (sf_id << 29);
}

// shared-memory descriptor of a 512-byte scale atom (32 rows x 16 B, no swizzle)
__device__ __forceinline__ uint64_t sdesc_atom(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16 >> 4) << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

__device__ __forceinline__ void tmem_cp_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void mma_mxf8f6f4(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t acc, uint32_t sfa, uint32_t sfb) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

// (lo, hi) -> two e4m3 codes, lo in the low byte (round to nearest even, saturating)
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return (uint32_t)r;
}
// two e4m3 codes (low byte first) -> their values
__device__ __forceinline__ float2 e4m3x2_val(uint32_t codes) {
  uint32_t h;
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(h) : "r"(codes));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// e8m0 byte of the scale that maps a block maximum mx into [128, 256)
// (127 = 2^0 for an all-zero block)
__device__ __forceinline__ int term_scale(float mx) {
  if (mx == 0.f) return 127;
  const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);
  return max(E - 7, 0);
}

// 2^-(sb-127) and 2^(sb-127) as fp32 (sb = 0 gives 2^-127, a subnormal)
__device__ __forceinline__ float term_inv(int sb) { return __uint_as_float((uint32_t)(254 - sb) << 23); }
__device__ __forceinline__ float term_val(int sb) {
  return sb ? __uint_as_float((uint32_t)sb << 23) : 0x1p-127f;
}

// One term of E elements (E % 4 == 0) held in r[]: codes into w[E / 4] (four
// e4m3 per word, element 4k + e in byte e of word k), and r[] reduced by the
// term's value.  The block maximum behind sb is the caller's (reduced over the
// threads that share a block).
template <int E>
__device__ __forceinline__ void term_codes(float (&r)[E], int sb, uint32_t (&w)[E / 4]) {
  const float inv = term_inv(sb), scl = term_val(sb);
#pragma unroll
  for (int k = 0; k < E / 4; ++k) {
    const uint32_t c0 = e4m3x2(r[4 * k] * inv, r[4 * k + 1] * inv);
    const uint32_t c1 = e4m3x2(r[4 * k + 2] * inv, r[4 * k + 3] * inv);
    const float2 v0 = e4m3x2_val(c0), v1 = e4m3x2_val(c1);
    r[4 * k] = fmaf(-v0.x, scl, r[4 * k]);
    r[4 * k + 1] = fmaf(-v0.y, scl, r[4 * k + 1]);
    r[4 * k + 2] = fmaf(-v1.x, scl, r[4 * k + 2]);
    r[4 * k + 3] = fmaf(-v1.y, scl, r[4 * k + 3]);
    w[k] = c0 | (c1 << 16);
  }
}

// bf16 pairs of a 16-byte load -> 8 floats
__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float* r) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    r[2 * e] = __uint_as_float(u[e] << 16);
    r[2 * e + 1] = __uint_as_float(u[e] & 0xFFFF0000u);
  }
}

}  // namespace mx
}  // namespace b200kv
