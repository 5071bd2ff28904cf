// MXFP4 (e2m1 + e8m0) W4A16 matvec / skinny GEMM for sm_100a, 1 <= M <= 8.
//
// Computes out[m, n] = bf16_rn( sum_g scale(St[n,g]) * sum_{j<32} e2m1(W[n,32g+j]) * x[m,32g+j] )
// with fp32 accumulation -- the arithmetic of the reference kernel
// h4mv/h4mv.cu:43-104 (h4mv_t<MT>), re-designed for B200:
//
//  * Work unit: a CTA owns 16*RT consecutive weight rows and one K-slice; the
//    K-slices of a row tile form a thread-block cluster (up to 8 CTAs along y)
//    that reduce their fp32 partials through distributed shared memory, so a
//    small-N layer still puts several CTAs on every SM without global scratch.
//  * Inside a CTA, NW warps split the K-slice further; each warp step covers 4
//    consecutive e8m0 groups (128 k): lane (r0 = lane/4, c = lane%4) streams one
//    16-byte group (32 weights) of row r0 and of row r0+8 per row tile with
//    128-bit evict-first loads -- a 16-byte load is exactly one scale group, as
//    in the reference (h4mv.cu:7-8).
//  * Dequant happens in registers: a nibble's sign goes to the bf16 sign bit and
//    its 3 magnitude bits to bf16 bits [8:6], which is the e2m1 value times
//    2^-126 for every code (zero and the 0.5 subnormal included); one packed
//    bf16x2 multiply by 2^(s-1) then applies the 2^126 renormalisation and the
//    group scale 2^(s-127) exactly (two multiplies when s > 128).
//  * The products and the fp32 accumulation run on the tensor pipe through
//    mma.sync m16n8k16 (A = 16 weight rows x 16 k, B = 16 k x 8 activation rows),
//    used here purely as a wide fp32-accumulating dot-product engine: a matvec
//    needs 2*M multiply-adds per weight byte, which would saturate the FP32 pipe
//    and the issue slots long before HBM does.  The reference made the same move
//    on gfx1201 with v_dot2_f32_bf16 (h4mv.cu:26-31).
//  * The activation pairs are permuted with byte_perm so that the k-order of the
//    B fragment matches the (nibble j, nibble j+4) pairing of the dequant.
//
// Edge semantics follow the reference kernel: scale byte 0 -> 0.0, 255 -> inf.
// The output rounding is fp32 -> bf16 round-to-nearest-even.

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdlib.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace cg = cooperative_groups;

namespace b200kv {
namespace {

// 8 e2m1 codes (nibble i = k offset i) -> 4 bf16x2 words, value * 2^-126.
// d[j] = { lo: nibble j, hi: nibble j+4 }.  The shift moves nibble j to bits
// 12..15 and nibble j+4 to bits 28..31, the top nibble of each 16-bit half.
__device__ __forceinline__ void e2m1x8_to_bf16x2_lowexp(uint32_t q, uint32_t (&d)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t qs = q << (4 * (3 - j));
    d[j] = (qs & 0x80008000u) | ((qs & 0x70007000u) >> 6);
  }
}

// d = a * b for packed bf16x2 (one rounding; exact here since one factor is a
// power of two and no result underflows).  fma with -0 keeps the sign of zero.
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(0x80008000u));
  return d;
}

__device__ __forceinline__ void mma_16816_bf16(float (&c)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Dequantise one 16-byte group (32 weights of one row) into 16 bf16x2 words
// a[p], p = 4*t + j  <->  k offsets (8t + j, 8t + j + 4) inside the group.
__device__ __forceinline__ void dequant_group(const uint4& w, uint32_t s, uint32_t (&a)[16]) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  // s in [1,128]: one multiply by 2^(s-1); s == 0: scale 0; s > 128: 2^126 then 2^(s-127).
  const bool two_step = s > 128u;
  const uint32_t e1 = (s == 0u) ? 0u : (two_step ? 0x7E80u : ((s + 126u) << 7));
  const uint32_t m1 = e1 | (e1 << 16);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    uint32_t d[4];
    e2m1x8_to_bf16x2_lowexp(words[t], d);
#pragma unroll
    for (int j = 0; j < 4; ++j) a[4 * t + j] = bf16x2_mul(d[j], m1);
  }
  if (two_step) {
    const uint32_t e2 = s << 7;  // 2^(s-127); s == 255 gives inf like the reference
    const uint32_t m2 = e2 | (e2 << 16);
#pragma unroll
    for (int p = 0; p < 16; ++p) a[p] = bf16x2_mul(a[p], m2);
  }
}

template <int RT, int NW>
__global__ void __launch_bounds__(NW * 32)
    mxfp4_gemv_kernel(const uint8_t* __restrict__ W, const uint8_t* __restrict__ St,
                      const __nv_bfloat16* __restrict__ X, __nv_bfloat16* __restrict__ Out,
                      int N, int K, int M, int groups_per_split) {
  constexpr int ROWS = 16 * RT;
  __shared__ float red[NW][ROWS][8];
  __shared__ float cta_part[ROWS][8];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int r0 = lane >> 2;
  const int c = lane & 3;
  const int ngroups = K >> 5;
  const int row_base = blockIdx.x * ROWS;
  const int g_begin = blockIdx.y * groups_per_split;
  const int g_end = min(ngroups, g_begin + groups_per_split);
  const size_t row_bytes = (size_t)(K >> 1);

  const int xn = min(r0, M - 1);
  const uint4* xrow = reinterpret_cast<const uint4*>(X + (size_t)xn * K);

  const uint8_t* wrow[RT][2];
  const uint8_t* srow[RT][2];
#pragma unroll
  for (int t = 0; t < RT; ++t) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = min(row_base + 16 * t + 8 * h + r0, N - 1);
      wrow[t][h] = W + (size_t)r * row_bytes;
      srow[t][h] = St + (size_t)r * ngroups;
    }
  }

  float acc[RT][4];
#pragma unroll
  for (int t = 0; t < RT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;

  const int q_begin = g_begin >> 2;               // g_begin is a multiple of 4
  const int q_end = (g_end + 3) >> 2;
#pragma unroll 2
  for (int qd = q_begin + warp; qd < q_end; qd += NW) {
    const int g = qd * 4 + c;
    const bool valid = g < g_end;
    uint4 wv[RT][2];
    uint32_t sv[RT][2];
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        wv[t][h] = valid ? ldg_stream_u4(wrow[t][h] + (size_t)g * 16) : make_uint4(0, 0, 0, 0);
        sv[t][h] = valid ? (uint32_t)__ldg(srow[t][h] + g) : 0u;
      }
    uint4 xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) xv[i] = valid ? __ldg(xrow + (size_t)g * 4 + i) : make_uint4(0, 0, 0, 0);

    // B fragments: pair (x[8t+j], x[8t+j+4]) for p = 4t + j.
    uint32_t xp[16];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      xp[4 * t + 0] = __byte_perm(xv[t].x, xv[t].z, 0x5410);
      xp[4 * t + 1] = __byte_perm(xv[t].x, xv[t].z, 0x7632);
      xp[4 * t + 2] = __byte_perm(xv[t].y, xv[t].w, 0x5410);
      xp[4 * t + 3] = __byte_perm(xv[t].y, xv[t].w, 0x7632);
    }

#pragma unroll
    for (int t = 0; t < RT; ++t) {
      uint32_t a_lo[16], a_hi[16];
      dequant_group(wv[t][0], sv[t][0], a_lo);
      dequant_group(wv[t][1], sv[t][1], a_hi);
#pragma unroll
      for (int mi = 0; mi < 8; ++mi)
        mma_16816_bf16(acc[t], a_lo[2 * mi], a_hi[2 * mi], a_lo[2 * mi + 1], a_hi[2 * mi + 1],
                       xp[2 * mi], xp[2 * mi + 1]);
    }
  }

  // ---- reduce the NW warps of this CTA --------------------------------------
#pragma unroll
  for (int t = 0; t < RT; ++t) {
    red[warp][16 * t + r0][2 * c] = acc[t][0];
    red[warp][16 * t + r0][2 * c + 1] = acc[t][1];
    red[warp][16 * t + r0 + 8][2 * c] = acc[t][2];
    red[warp][16 * t + r0 + 8][2 * c + 1] = acc[t][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ROWS * 8; i += NW * 32) {
    const int r = i >> 3, m = i & 7;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) s += red[w][r][m];
    cta_part[r][m] = s;
  }

  if (gridDim.y == 1) {
    __syncthreads();
    for (int i = threadIdx.x; i < ROWS * M; i += NW * 32) {
      const int m = i / ROWS, r = i % ROWS;
      const int n = row_base + r;
      if (n < N) Out[(size_t)m * N + n] = __float2bfloat16_rn(cta_part[r][m]);
    }
    return;
  }

  // ---- reduce the K-slices of the cluster through distributed shared memory --
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const int nranks = (int)cluster.num_blocks();
    for (int i = threadIdx.x; i < ROWS * M; i += NW * 32) {
      const int m = i / ROWS, r = i % ROWS;
      float s = cta_part[r][m];
      for (int q = 1; q < nranks; ++q) {
        const float* peer = cluster.map_shared_rank(&cta_part[0][0], q);
        s += peer[r * 8 + m];
      }
      const int n = row_base + r;
      if (n < N) Out[(size_t)m * N + n] = __float2bfloat16_rn(s);
    }
  }
  cluster.sync();  // keep every peer's shared memory alive until rank 0 is done
}

struct GemvConfig {
  int rt, nw, ksplit;
};

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return atoi(v);
}

GemvConfig choose_config(int N, int K, int M) {
  const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
  GemvConfig cfg;
  cfg.rt = M <= 2 ? 1 : 2;
  cfg.nw = 4;
  const int ngroups = K / 32;
  const int tiles = cdiv(N, 16 * cfg.rt);
  cfg.ksplit = 1;
  while (cfg.ksplit < 8 && tiles * cfg.ksplit < 2 * sms && ngroups / (cfg.ksplit * 2) >= 16)
    cfg.ksplit *= 2;
  // explicit overrides for tuning sweeps
  cfg.rt = env_int("B200KV_GEMV_RT", cfg.rt);
  cfg.nw = env_int("B200KV_GEMV_NW", cfg.nw);
  cfg.ksplit = env_int("B200KV_GEMV_KSPLIT", cfg.ksplit);
  return cfg;
}

template <int RT, int NW>
cudaError_t launch_gemv(const GemvConfig& cfg, const uint8_t* W, const uint8_t* St,
                        const __nv_bfloat16* X, __nv_bfloat16* Out, int N, int K, int M,
                        cudaStream_t stream) {
  const int ngroups = K / 32;
  int gps = cdiv(ngroups, cfg.ksplit);
  gps = (gps + 3) & ~3;  // split boundaries on 4-group steps
  const int ksplit = cdiv(ngroups, gps);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(cdiv(N, 16 * RT), ksplit, 1);
  lc.blockDim = dim3(NW * 32, 1, 1);
  lc.dynamicSmemBytes = 0;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ksplit;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, mxfp4_gemv_kernel<RT, NW>, W, St, X, Out, N, K, M, gps);
}

}  // namespace

int mxfp4_gemv_launch(const void* W, const void* St, const void* X, void* out, int N, int K,
                      int M, void* stream) {
  if (!W || !St || !X || !out) return B200KV_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || M <= 0) return B200KV_ERR_INVALID_ARG;
  if (M > 8 || (K % 32) != 0) return B200KV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(X) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 1))
    return B200KV_ERR_MISALIGNED;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  const GemvConfig cfg = choose_config(N, K, M);
  if (cfg.ksplit < 1 || cfg.ksplit > 8) return B200KV_ERR_INVALID_ARG;
  const uint8_t* w = static_cast<const uint8_t*>(W);
  const uint8_t* s = static_cast<const uint8_t*>(St);
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(X);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  const int key = cfg.rt * 100 + cfg.nw;
  switch (key) {
    case 104: e = launch_gemv<1, 4>(cfg, w, s, x, o, N, K, M, st); break;
    case 108: e = launch_gemv<1, 8>(cfg, w, s, x, o, N, K, M, st); break;
    case 204: e = launch_gemv<2, 4>(cfg, w, s, x, o, N, K, M, st); break;
    case 208: e = launch_gemv<2, 8>(cfg, w, s, x, o, N, K, M, st); break;
    case 404: e = launch_gemv<4, 4>(cfg, w, s, x, o, N, K, M, st); break;
    default: return B200KV_ERR_INVALID_ARG;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
