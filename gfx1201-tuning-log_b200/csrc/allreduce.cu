// One-shot allreduce (sum) of a small bf16 vector over the GPUs of one node,
// through peer memory over NVLink / NVSwitch: the collective after the
// row-parallel o and down projections of the tensor-parallel 7B step (one
// [M, 4096] partial per rank, M <= 8).
//
// Every rank owns a communication buffer (cudaMalloc, shared with the peers
// through CUDA IPC handles):
//   [0, 256)       call counters, one per CTA (read and advanced only by it)
//   [256, ...)     lines[2][8][kMaxElems / 2] of 8 bytes: {4 data bytes, flag}
// The vector is split into chunks of kLinesPerCta lines, one CTA each (the
// grid depends only on n, so every call of a size uses the same chunks and
// counters).  Call k of a chunk (its counter value k, parity p = k & 1) on
// rank r: the CTA writes its chunk into lines[p][r] of every rank, two bf16
// and the flag k + 1 per
// 8-byte store (one NVLink transaction, so a reader that sees the flag sees the
// data: no fence and no separate flag round trip -- the "low-latency" line
// format), then polls its own lines[p][*] until every flag reads k + 1
// (bounded by %globaltimer) and writes the sum over ranks in rank order (fp32,
// then bf16): every rank produces identical bytes.
// Reusing parity p at call k + 2 is safe: rank r starts call k + 2 only after
// its call k + 1 saw every peer's lines of call k + 1, which each peer wrote
// after it had finished reading its lines of call k.  No multicast objects, no
// NCCL.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace b200kv {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxElems = 8 * 4096;     // bf16 elements per partial
constexpr int kArThreads = 256;
constexpr int kLinesPerCta = 256;        // one line per thread
constexpr int kMaxCtas = kMaxElems / 2 / kLinesPerCta;
constexpr size_t kCtrlBytes = 256;
constexpr size_t kLines = kMaxElems / 2;  // 8-byte lines per rank slot
constexpr size_t kBufBytes = kCtrlBytes + (size_t)2 * kMaxRanks * kLines * 8;
static_assert(kMaxCtas * 4 <= (int)kCtrlBytes, "one counter per CTA in the control block");
constexpr unsigned long long kTimeoutNs = 200ull * 1000 * 1000;  // 200 ms

struct PeerBufs {
  uint8_t* p[kMaxRanks];
};

__device__ __forceinline__ uint2* lines(uint8_t* buf, int parity, int r) {
  return reinterpret_cast<uint2*>(buf + kCtrlBytes) + ((size_t)parity * kMaxRanks + r) * kLines;
}
__device__ __forceinline__ void st_line(uint2* p, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(flag) : "memory");
}
__device__ __forceinline__ uint2 ld_line(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
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

  // poll the local slots, fixed-order sum (identical on every rank)
  bool late = false;
  for (int i = i0 + tid; i < nl; i += kArThreads) {
    float a0 = 0.f, a1 = 0.f;
    for (int r = 0; r < tp; ++r) {
      const uint2* l = lines(mine, par, r) + i;
      uint2 v = ld_line(l);
      if (v.y != flag && !late) {
        const unsigned long long t0 = globaltimer();
        while ((v = ld_line(l)).y != flag) {
          if (globaltimer() - t0 > kTimeoutNs) {
            atomicExch(&g_device_status, kDevPeerTimeout);
            late = true;
            break;
          }
        }
      }
      a0 += __uint_as_float(v.x << 16);
      a1 += __uint_as_float(v.x & 0xFFFF0000u);
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
