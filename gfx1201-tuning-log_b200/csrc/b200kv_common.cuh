// Shared device/host helpers for libb200kv (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace b200kv {

// ---- device status word ------------------------------------------------------
// Written (atomicExch) by a kernel that gave up on a bounded wait.  Codes:
enum DeviceStatus : int {
  kDevOk = 0,
  kDevMbarrierTimeout = 0x101,   // a bulk copy never completed on its mbarrier
  kDevSplitOverflow = 0x102,     // seq_len larger than the context bound given
  kDevPeerTimeout = 0x103,       // a peer GPU's flag did not arrive in time
  kDevChainTimeout = 0x104,      // a chained GEMV's input tile was not ready in time
  kDevIndexRange = 0x105,        // a token id or position outside its table
};
extern __device__ int g_device_status;

// ---- host helpers ------------------------------------------------------------
int num_sms_current_device();     // cached per device; 0 when no device
int sm_major_current_device();
bool pdl_enabled();               // B200KV_PDL=0 turns programmatic launches off

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// ---- device helpers ----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// SiLU of a bf16 value g, rounded to bf16: the activation of HF Llama's
// act_fn(gate) * up as the decoder rounds it (every SwiGLU in this library
// uses it, so fused and separate paths agree bit for bit).  g / (1 + e^-g)
// with the fast division: within 2 ulp of the fp32 quotient before the bf16
// rounding, and 0 for g < -87 (where 1 + e^-g passes 2^126 and SiLU(g) is
// below 1e-36 in magnitude).  An IEEE division here made the SwiGLU epilogue
// of the wide GEMM five times as long.
__device__ __forceinline__ float silu_bf16(float g) {
  return __bfloat162float(__float2bfloat16_rn(__fdividef(g, 1.f + __expf(-g))));
}

// Neox rotary embedding of one pair (x1 at dim j, x2 at dim j + d/2 of a head;
// c, s the cosine and sine of the pair's angle), the products rounded before
// the sum (no fused multiply-add): the arithmetic of the RoPE + KV-write
// kernel and of the qkv GEMV's RoPE epilogue, which so agree bit for bit.
__device__ __forceinline__ void rope_pair(float x1, float x2, float c, float s, float& y1, float& y2) {
  y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ANDs a predicate over its `count` threads: every
// thread gets the same answer, so all of them can leave a loop together.
__device__ __forceinline__ bool named_bar_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records the device
// status) when the phase did not complete within `max_tries` polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t max_tries = (1u << 22)) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < max_tries; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicExch(&g_device_status, kDevMbarrierTimeout);
  return false;
}

// Global nanosecond timer (bounded spins on flags in global memory).
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One non-blocking test of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// One-dimensional bulk copy global -> shared (TMA engine), completion counted
// in bytes on `bar`.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Ampere-style 16-byte asynchronous global -> shared copy (L2 only) and its
// commit / wait-group pair.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- thread-block clusters: push into a peer's shared memory -----------------------
// A rank that pushes with st.async must know the target's mbarrier is
// initialised: every thread calls cluster_arrive_relaxed() after the barriers
// are set up and the pushing threads call cluster_wait() before their first
// push.  The target waits on its mbarrier for the bytes it expects, so no rank
// reads another's shared memory and none waits on a cluster barrier at the end.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// 4-byte store into a peer CTA's shared memory, counted in bytes on the peer's
// mbarrier (both addresses from map_to_rank)
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
               : "memory");
}

// 16-byte store (four floats) into a peer CTA's shared memory, counted on the
// peer's mbarrier; raddr 16-byte aligned
__device__ __forceinline__ void st_async_v4_f32(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   raddr),
               "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
               "r"(__float_as_uint(v.w)), "r"(rbar)
               : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------
// A kernel launched with programmatic stream serialization may start while the
// kernel before it in the stream still runs (once every CTA of that kernel has
// called griddep_launch_dependents or exited).  Whatever it reads that the
// previous kernel may write, and everything it writes, comes after
// griddep_wait(), which returns once the previous grid has completed and its
// memory is visible.  Every CTA of every kernel here passes griddep_wait()
// before it exits, so a grid's completion implies its predecessors'.  Both are
// no-ops for a plain launch.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace b200kv
