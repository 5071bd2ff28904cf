// ORACLE -- test infrastructure, not product code.
//
// Host stand-in for <hip/hip_runtime.h>, just enough to compile the
// reference's MXFP4 matvec kernel h4mv_t<MT> (h4mv/h4mv.cu:43-104) unmodified
// with g++ and run it on the CPU, so its exact arithmetic (per-lane group
// partials, the scale multiply, the wave's xor-shuffle reduction and its
// manual round-to-bf16) can pin the repo's oracle.  oracle/Makefile feeds the
// kernel's source to g++ from where it lies; nothing of it is copied.
//
// Execution model: every thread of a block is a coroutine (ucontext);
// __syncthreads() and __shfl_xor() hand control back to a scheduler that runs
// each thread up to its next barrier or shuffle and resolves a shuffle once
// every live lane of the wave (warpSize 32, as gfx1201's wave32) offered its
// value.  __shared__ arrays become function statics, shared by all threads.
//
// The one instruction g++ cannot take is the kernel's inline
// "v_dot2_f32_bf16" (h4mv.cu:26-31); it is replaced by dot2_bf16_f32 below:
// the two bf16 x bf16 products (exact) and the fp32 addend summed in double
// and rounded once to fp32, the result of a fused two-term dot product with a
// single rounding.  That is a modelling choice (the gfx1201 instruction's
// internal rounding is not documented in the reference); products of an e2m1
// code and a bf16 value have at most 10 significant bits, so for the data
// here the double sum is exact and only the final rounding remains.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ucontext.h>
#include <vector>

namespace hiphost {

struct Dim3 {
  unsigned x, y, z;
};

struct Lane {
  Dim3 tid;
  ucontext_t ctx;
  int state;  // 0 runnable, 1 at __syncthreads, 2 at a shuffle, 3 finished
  float val;  // value offered to a shuffle
  int off;    // its xor offset
  float got;  // value received
};

inline Dim3 g_block_idx = {0, 0, 0}, g_block_dim = {1, 1, 1};
inline Lane* g_cur = nullptr;
inline ucontext_t g_sched;

inline void yield_to_scheduler() { swapcontext(&g_cur->ctx, &g_sched); }

inline void syncthreads() {
  g_cur->state = 1;
  yield_to_scheduler();
}

inline float shfl_xor(float v, int off) {
  g_cur->val = v;
  g_cur->off = off;
  g_cur->state = 2;
  yield_to_scheduler();
  return g_cur->got;
}

inline float f32_of_bits(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// fused two-term bf16 dot product with fp32 accumulate, one rounding
inline float dot2_bf16_f32(uint32_t a, uint32_t b, float c) {
  const double p = (double)f32_of_bits(a << 16) * (double)f32_of_bits(b << 16) +
                   (double)f32_of_bits(a & 0xFFFF0000u) * (double)f32_of_bits(b & 0xFFFF0000u) + (double)c;
  return (float)p;
}

}  // namespace hiphost

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(n)
#define __shared__ static
#define threadIdx (hiphost::g_cur->tid)
#define blockIdx (hiphost::g_block_idx)
#define blockDim (hiphost::g_block_dim)
#define warpSize 32

inline void __syncthreads() { hiphost::syncthreads(); }
inline float __shfl_xor(float v, int off) { return hiphost::shfl_xor(v, off); }
inline float __uint_as_float(uint32_t u) { return hiphost::f32_of_bits(u); }
inline uint32_t __float_as_uint(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
struct uint4 {
  uint32_t x, y, z, w;
};
typedef void* hipStream_t;

// The kernel's only inline-asm statement is its dot2 (operands named a, b, c,
// result d); every system header is included above, before this definition.
#define __asm__(...) (d = hiphost::dot2_bf16_f32(a, b, c))
