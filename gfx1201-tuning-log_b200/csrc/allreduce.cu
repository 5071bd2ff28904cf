// One-shot allreduce (sum) of a small bf16 vector over the GPUs of one node,
// through peer memory over NVLink / NVSwitch: the collective after the
// row-parallel o and down projections of the tensor-parallel 7B step (one
// [M, 4096] partial per rank, M <= 8).
//
// The buffer layout and the line protocol are in peer_comm.cuh; here the
// vector is split into chunks of kLinesPerCta lines, one CTA each (the grid
// depends only on n, so every call of a size uses the same chunks and
// counters).  No multicast objects, no NCCL.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "peer_comm.cuh"

namespace b200kv {
namespace {

constexpr int kMaxRanks = kCommMaxRanks;
constexpr int kMaxElems = kCommMaxElems;
constexpr int kArThreads = 256;
constexpr int kLinesPerCta = 256;        // one line per thread
constexpr int kMaxCtas = kMaxElems / 2 / kLinesPerCta;
constexpr size_t kBufBytes = kCommBufBytes;
static_assert(kMaxCtas <= kCommCounters, "one counter per CTA in the control block");
constexpr unsigned long long kTimeoutNs = kCommTimeoutNs;

__device__ __forceinline__ uint2* lines(uint8_t* buf, int parity, int r) { return comm_lines(buf, parity, r); }
__device__ __forceinline__ void st_line(uint2* p, uint32_t data, uint32_t flag) { comm_st_line(p, data, flag); }
__device__ __forceinline__ uint2 ld_line(const uint2* p) { return comm_ld_line(p); }
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kArThreads, 1)
    allreduce_oneshot_kernel(const __nv_bfloat16* in, __nv_bfloat16* out, int n,
                             const __grid_constant__ PeerBufs peers,
                             int rank, int tp) {
  __shared__ uint32_t call;
  const int tid = threadIdx.x;
  if (tid == 0) griddep_launch_dependents();
  uint8_t* mine = peers.p[rank];
  volatile uint32_t* counter = reinterpret_cast<volatile uint32_t*>(mine) + blockIdx.x;
  // `in` is the previous kernel's output, and the counter was advanced by the
  // previous call, which may still have been running when this grid started
  griddep_wait();
  if (tid == 0) call = *counter;
  __syncthreads();
  const uint32_t flag = call + 1;
  const int par = (int)(call & 1u);
  const int nl = min(n / 2, (int)(blockIdx.x + 1) * kLinesPerCta);  // lines (2 bf16 each)
  const int i0 = blockIdx.x * kLinesPerCta;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(in);

  // push: this rank's chunk into slot `rank` of every rank's buffer
  for (int i = i0 + tid; i < nl; i += kArThreads) {
    const uint32_t d = src[i];
    for (int r = 0; r < tp; ++r) st_line(lines(peers.p[r], par, rank) + i, d, flag);
  }

  // poll the local slots, fixed-order sum (identical on every rank): the
  // first load of every rank's line is issued at once (one round trip for
  // all of them), only lines not yet written are loaded again
  bool late = false;
  for (int i = i0 + tid; i < nl; i += kArThreads) {
    uint2 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < tp) v[r] = ld_line(lines(mine, par, r) + i);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= tp) continue;
      if (v[r].y != flag && !late) {
        const uint2* l = lines(mine, par, r) + i;
        const unsigned long long t0 = globaltimer();
        while ((v[r] = ld_line(l)).y != flag) {
          if (globaltimer() - t0 > kTimeoutNs) {
            atomicExch(&g_device_status, kDevPeerTimeout);
            late = true;
            break;
          }
        }
      }
      a0 += __uint_as_float(v[r].x << 16);
      a1 += __uint_as_float(v[r].x & 0xFFFF0000u);
    }
    const __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
    reinterpret_cast<uint32_t*>(out)[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  __syncthreads();
  if (tid == 0) *counter = flag;
}

}  // namespace

size_t comm_buffer_bytes() { return kBufBytes; }

int comm_alloc(void** buf, void* ipc_handle) {
  if (!buf || !ipc_handle) return B200KV_ERR_INVALID_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, kBufBytes) != cudaSuccess) return B200KV_ERR_LAUNCH;
  if (cudaMemset(p, 0, kBufBytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p) != cudaSuccess) {
    cudaFree(p);
    return B200KV_ERR_LAUNCH;
  }
  *buf = p;
  return B200KV_OK;
}

int comm_open(const void* ipc_handle, void** peer) {
  if (!ipc_handle || !peer) return B200KV_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(peer, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? B200KV_OK : B200KV_ERR_LAUNCH;
}

int comm_close(void* peer) {
  return cudaIpcCloseMemHandle(peer) == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

int comm_free(void* buf) { return cudaFree(buf) == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH; }

int allreduce_oneshot_launch(const void* in, void* out, int n, void* const* bufs, int rank, int tp,
                             void* stream) {
  if (!in || !out || !bufs || n <= 0) return B200KV_ERR_INVALID_ARG;
  if (tp < 1 || tp > kMaxRanks || rank < 0 || rank >= tp) return B200KV_ERR_INVALID_ARG;
  if (n > kMaxElems || n % 8) return B200KV_ERR_UNSUPPORTED;  // 16-byte rows of 8 bf16
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return B200KV_ERR_MISALIGNED;
  PeerBufs pb = {};
  for (int r = 0; r < tp; ++r) {
    if (!bufs[r]) return B200KV_ERR_INVALID_ARG;
    pb.p[r] = static_cast<uint8_t*>(bufs[r]);
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((n / 2 + kLinesPerCta - 1) / kLinesPerCta, 1, 1);
  lc.blockDim = dim3(kArThreads, 1, 1);
  lc.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&lc, allreduce_oneshot_kernel,
                                           static_cast<const __nv_bfloat16*>(in),
                                           static_cast<__nv_bfloat16*>(out), n, pb, rank, tp);
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
