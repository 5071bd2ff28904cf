// Greedy-decoding argmax over fp32 logits rows (sm_100a).
//
// The decode step's last op: [rows, cols] fp32 logits -> per row the largest
// value and the lowest index holding it.  A thread-block cluster of kCs CTAs
// shares a row (cols = 128256 for the 7B vocabulary, 513 KB per row): each CTA
// scans one contiguous chunk with coalesced loads, reduces (value, index)
// pairs through warp shuffles and shared memory, and rank 0 merges the kCs
// results read from its peers' shared memory.  No global scratch, one launch,
// programmatic dependent launch like the other kernels here (the logits are
// read after griddep_wait()).

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace cg = cooperative_groups;

namespace b200kv {
namespace {

constexpr int kCs = 8;          // CTAs per row (a portable cluster)
constexpr int kArgThreads = 512;

// a beats b: larger value, or the same value at a lower index (NaN-free rows)
__device__ __forceinline__ bool better(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

__global__ void __cluster_dims__(kCs, 1, 1) __launch_bounds__(kArgThreads)
    argmax_rows_kernel(const float* __restrict__ x, int64_t ld, int cols, float* max_val, int64_t* max_idx) {
  __shared__ float s_val[kArgThreads / 32];
  __shared__ int64_t s_idx[kArgThreads / 32];
  __shared__ float c_val;
  __shared__ int64_t c_idx;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int row = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) griddep_launch_dependents();
  const int chunk = (cols + kCs - 1) / kCs;
  const int lo = rank * chunk, hi = min(cols, lo + chunk);
  griddep_wait();  // the logits are the previous kernel's output
  const float* xr = x + (int64_t)row * ld;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
#pragma unroll 8
  for (int i = lo + tid; i < hi; i += kArgThreads) {
    const float v = __ldg(xr + i);
    if (v > bv) {  // ascending indices per thread: the first of equal values stays
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_val[warp] = bv;
    s_idx[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kArgThreads / 32; ++w)
      if (better(s_val[w], s_idx[w], bv, bi)) {
        bv = s_val[w];
        bi = s_idx[w];
      }
    c_val = bv;
    c_idx = bi;
  }
  cluster.sync();  // every rank's result is in its shared memory
  if (rank == 0 && tid == 0) {
    float v = c_val;
    int64_t ix = c_idx;
    for (int r = 1; r < kCs; ++r) {
      const float rv = *cluster.map_shared_rank(&c_val, r);
      const int64_t ri = *cluster.map_shared_rank(&c_idx, r);
      if (better(rv, ri, v, ix)) {
        v = rv;
        ix = ri;
      }
    }
    if (max_val) max_val[row] = v;
    max_idx[row] = ix == INT64_MAX ? 0 : ix;
  }
  cluster.sync();  // peers keep their shared memory until rank 0 has read it
}

}  // namespace

int argmax_rows_launch(const float* x, int64_t ld, int rows, int cols, float* max_val, int64_t* max_idx,
                       void* stream) {
  if (!x || !max_idx) return B200KV_ERR_INVALID_ARG;
  if (rows <= 0 || cols <= 0 || ld < cols || rows > 65535) return B200KV_ERR_INVALID_ARG;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(kCs, rows, 1);
  lc.blockDim = dim3(kArgThreads, 1, 1);
  lc.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&lc, argmax_rows_kernel, x, ld, cols, max_val, max_idx);
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
