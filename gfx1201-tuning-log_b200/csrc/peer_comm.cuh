// Communication buffers for the peer-memory allreduces (one-shot kernel,
// allreduce.cu; the GEMV with an allreduce epilogue, mxfp4_mma.cu).
//
// Every rank owns one buffer (cudaMalloc, shared with the peers through CUDA
// IPC handles, zeroed once):
//   [0, 256)     call counters (u32): per CTA of the one-shot kernel, or per
//                128-row output tile of the fused GEMV; read and advanced only
//                by the one CTA that handles that chunk or tile in a call
//   [256, ...)   lines[2][kCommMaxRanks][kCommLines] of 8 bytes: {two bf16 of
//                the flattened [M, N] partial, flag}
// Call k of a chunk (counter value k, parity p = k & 1) on rank r writes its
// partial into lines[p][r] of every rank with flag k + 1, one 8-byte store per
// line (one NVLink transaction, so a reader that sees the flag sees the data),
// then polls its own lines[p][*] until every flag reads k + 1 and sums over
// the ranks in rank order (fp32, then bf16): every rank gets identical bytes.
// Reusing parity p at call k + 2 is safe: rank r starts call k + 2 of a chunk
// only after its call k + 1 saw every peer's lines of call k + 1, which each
// peer wrote after it had finished reading its lines of call k.  Buffers are
// plain device memory: no multicast objects.
#pragma once

#include <stdint.h>

namespace b200kv {

constexpr int kCommMaxRanks = 8;
constexpr int kCommMaxElems = 8 * 4096;  // bf16 elements of one rank's partial
constexpr size_t kCommCtrlBytes = 256;
constexpr int kCommCounters = (int)(kCommCtrlBytes / 4);
constexpr size_t kCommLines = kCommMaxElems / 2;  // 8-byte lines per rank slot
constexpr size_t kCommBufBytes = kCommCtrlBytes + (size_t)2 * kCommMaxRanks * kCommLines * 8;
constexpr unsigned long long kCommTimeoutNs = 200ull * 1000 * 1000;  // 200 ms

struct PeerBufs {
  uint8_t* p[kCommMaxRanks];
};

__device__ __forceinline__ uint2* comm_lines(uint8_t* buf, int parity, int r) {
  return reinterpret_cast<uint2*>(buf + kCommCtrlBytes) + ((size_t)parity * kCommMaxRanks + r) * kCommLines;
}
__device__ __forceinline__ void comm_st_line(uint2* p, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(flag) : "memory");
}
__device__ __forceinline__ uint2 comm_ld_line(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

}  // namespace b200kv
