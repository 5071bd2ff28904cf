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
//  * Warp-specialised CTA: one producer warp streams the weight tile through a
//    4-stage ring of ~8 KB K-chunks with bulk copies (TMA engine, one copy per
//    row per stage, mbarrier full/empty handshake), so loads of later chunks
//    overlap the math on earlier ones; the activation slice is staged once.
//  * The activations are converted once per CTA to f16 with an exact per-row
//    power-of-two prescale (the row maximum lands in [2^4, 2^5)): every bf16
//    value within 2^-18 of its row's maximum keeps its 8-bit significand
//    exactly, smaller ones are rounded to f16 subnormals (their products are
//    below 2^-18 of the largest and vanish in the fp32 sum), and no value can
//    overflow f16.  The prescale is undone exactly on the fp32 result; it can
//    only push a partial sum past fp32's range when the reference's own result
//    is within a factor 2^5 of it (scale bytes near 255).
//  * Weights are decoded with the Blackwell hardware convert
//    cvt.rn.f16x2.e2m1x2 (one instruction per byte, exact), and the products
//    and fp32 accumulation run on the tensor pipe through mma.sync m16n8k16
//    (A = 16 weight rows x 16 k, B = 16 k x 8 activation rows), used as a wide
//    fp32-accumulating dot-product engine: a matvec needs 2*M multiply-adds per
//    weight byte, which would saturate the FP32 pipe and the issue slots long
//    before HBM does.  The reference made the same move on gfx1201 with
//    v_dot2_f32_bf16 (h4mv.cu:26-31).
//  * The fragments are group-aligned: lane (r0 = lane/4, c = lane%4) takes bytes
//    4c..4c+3 of one 16-byte group (32 weights = one e8m0 group) of rows r0 and
//    r0+8, so the two MMAs of a group cover exactly that group, and the group
//    scale 2^(s-127) multiplies the group's fp32 partial -- the reference's
//    per-group structure (h4mv.cu:72-90), exact for every scale byte.
//
// Edge semantics follow the reference kernel: the scale is the fp32 bit pattern
// s << 23, so byte 0 -> 0.0 and 255 -> inf.  Output rounding: fp32 -> bf16 RN-even.

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace cg = cooperative_groups;

namespace b200kv {
namespace {

// 4 bytes = 8 e2m1 codes -> 4 f16x2 words (exact); word b holds byte b, low
// nibble (even k) in the low half.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n"
      " mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      " cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      " cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

__device__ __forceinline__ void mma_16816_f16(float (&c)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory layout.  Weight rows of a stage: pitch == 16 (mod 128) bytes,
// so the 8 rows x 4 lanes of a 32-bit load hit 32 distinct banks.  Activation
// rows: pitch == 64 (mod 128), so the 8-lane phases of a 128-bit load hit
// distinct 16-byte bank groups.  Scale rows: pitch == 4 (mod 8) words apart.
constexpr int kStages = 4;
__host__ __device__ constexpr int w_pitch(int kc) { return kc * 16 + 16; }
__host__ __device__ constexpr int x_pitch(int slice_k) { return ((slice_k * 2 + 127) & ~127) + 64; }
__host__ __device__ constexpr int s_pitch(int gps) { return ((gps + 15) & ~15) + 4; }

struct GemvLayout {
  int rows, gps, kc, m;
  __host__ __device__ int wp() const { return w_pitch(kc); }
  __host__ __device__ int xp() const { return x_pitch(gps * 32); }
  __host__ __device__ int sp() const { return s_pitch(gps); }
  __host__ __device__ size_t ring_off() const { return 0; }
  __host__ __device__ size_t x_off() const { return (size_t)kStages * rows * wp(); }
  __host__ __device__ size_t s_off() const { return x_off() + (size_t)m * xp(); }
  __host__ __device__ size_t bytes() const { return s_off() + (((size_t)rows * sp() + 15) & ~(size_t)15); }
};

// Warp-specialised: NW consumer warps do the math, one producer warp streams
// the weight tile through a kStages-deep ring of K-chunks (kc groups each).
template <int RT, int NW>
__global__ void __launch_bounds__((NW + 1) * 32)
    mxfp4_gemv_kernel(const uint8_t* __restrict__ W, const uint8_t* __restrict__ St,
                      const __nv_bfloat16* __restrict__ X, __nv_bfloat16* __restrict__ Out,
                      int N, int K, int M, int gps, int kc) {
  constexpr int ROWS = 16 * RT;
  constexpr int NC = NW * 32;        // consumer threads
  constexpr int NT = NC + 32;
  __shared__ float red[NW][ROWS][8];
  __shared__ float cta_part[ROWS][8];
  __shared__ float xunscale[8];
  __shared__ float xmax_part[NW][8];
  __shared__ uint64_t full_bar[kStages], empty_bar[kStages], x_bar;
  extern __shared__ __align__(128) uint8_t dsm[];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool producer = warp == NW;
  const int r0 = lane >> 2;
  const int c = lane & 3;
  const int ngroups = K >> 5;
  const int row_base = blockIdx.x * ROWS;
  const int g_begin = blockIdx.y * gps;
  const int g_end = min(ngroups, g_begin + gps);
  const int ng = g_end - g_begin;
  const int nst = (ng + kc - 1) / kc;
  const GemvLayout L{ROWS, gps, kc, M};
  const int wp = L.wp(), xp = L.xp(), sp = L.sp();
  uint8_t* ring = dsm + L.ring_off();   // [kStages][ROWS][wp]
  uint8_t* xsm = dsm + L.x_off();       // [M][xp]: bf16 staged, f16 after convert
  uint8_t* ssm = dsm + L.s_off();       // [ROWS][sp] scale bytes
  const int nrows = min(ROWS, N - row_base);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], NW);
    }
    mbar_init(&x_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  if (producer) {
    // ---- activation slice (once), then the weight ring ----------------------
    if (lane == 0) mbar_arrive_expect_tx(&x_bar, (uint32_t)(M * ng * 64));
    __syncwarp();
    if (lane < M)
      bulk_g2s(xsm + lane * xp, X + (size_t)lane * K + (size_t)g_begin * 32, (uint32_t)(ng * 64), &x_bar);
    for (int st = 0; st < nst && !failed; ++st) {
      const int slot = st % kStages;
      if (st >= kStages) failed = !mbar_wait_bounded(&empty_bar[slot], ((st / kStages) - 1) & 1);
      const int g0 = st * kc;
      const int kcs = min(kc, ng - g0);
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], (uint32_t)(nrows * kcs * 16));
      __syncwarp();
      for (int r = lane; r < nrows; r += 32)
        bulk_g2s(ring + (size_t)(slot * ROWS + r) * wp,
                 W + (size_t)(row_base + r) * (K >> 1) + (size_t)(g_begin + g0) * 16,
                 (uint32_t)(kcs * 16), &full_bar[slot]);
    }
  } else {
    // ---- scales of the whole slice into padded rows ---------------------------
    for (int i = tid; i < nrows * ng; i += NC) {
      const int r = i / ng, g = i % ng;
      ssm[r * sp + g] = __ldg(St + (size_t)(row_base + r) * ngroups + g_begin + g);
    }
    // ---- activations: exact per-row power-of-two prescale into f16 ------------
    failed = !mbar_wait_bounded(&x_bar, 0);
    const int per_row = ng * 4;  // uint4 per row
    for (int m = 0; m < M; ++m) {
      const uint4* row = reinterpret_cast<const uint4*>(xsm + m * xp);
      float mx = 0.f;
      for (int i = tid; i < per_row; i += NC) {
        const uint4 v = row[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(w[j] << 16)),
                               fabsf(__uint_as_float(w[j] & 0xFFFF0000u))));
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) xmax_part[warp][m] = mx;
    }
    named_bar_sync(1, NC);
    for (int m = 0; m < M; ++m) {
      float mx = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) mx = fmaxf(mx, xmax_part[w][m]);
      const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);
      int sh = (E == 0xFF || mx == 0.f) ? 0 : 131 - E;  // max * 2^sh in [2^4, 2^5)
      sh = max(-126, min(127, sh));
      const float up = __uint_as_float((uint32_t)(sh + 127) << 23);
      if (tid == 0) xunscale[m] = __uint_as_float((uint32_t)(127 - sh) << 23);
      uint4* row = reinterpret_cast<uint4*>(xsm + m * xp);
      for (int i = tid; i < per_row; i += NC) {
        const uint4 v = row[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2 h = __floats2half2_rn(__uint_as_float(w[j] << 16) * up,
                                              __uint_as_float(w[j] & 0xFFFF0000u) * up);
          o[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        row[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    named_bar_sync(1, NC);
  }

  float acc[RT][4];
#pragma unroll
  for (int t = 0; t < RT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;

  if (!producer) {
    const uint8_t* xrow = xsm + min(r0, M - 1) * xp + 16 * c;
    int lrow[RT][2];
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) lrow[t][h] = min(16 * t + 8 * h + r0, nrows - 1);
    for (int st = 0; st < nst; ++st) {
      const int slot = st % kStages;
      if (!failed) failed = !mbar_wait_bounded(&full_bar[slot], (st / kStages) & 1);
      const int g0 = st * kc;
      const int kcs = failed ? 0 : min(kc, ng - g0);
      const uint8_t* stage = ring + (size_t)slot * ROWS * wp;
#pragma unroll 2
      for (int gl = warp; gl < kcs; gl += NW) {
        const int g = g0 + gl;
        const uint4 xv = *reinterpret_cast<const uint4*>(xrow + g * 64);
#pragma unroll
        for (int t = 0; t < RT; ++t) {
          const uint32_t w_lo = *reinterpret_cast<const uint32_t*>(stage + lrow[t][0] * wp + gl * 16 + 4 * c);
          const uint32_t w_hi = *reinterpret_cast<const uint32_t*>(stage + lrow[t][1] * wp + gl * 16 + 4 * c);
          uint32_t a_lo[4], a_hi[4];
          e2m1x8_to_f16x2(w_lo, a_lo);
          e2m1x8_to_f16x2(w_hi, a_hi);
          float part[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816_f16(part, a_lo[0], a_hi[0], a_lo[1], a_hi[1], xv.x, xv.y);
          mma_16816_f16(part, a_lo[2], a_hi[2], a_lo[3], a_hi[3], xv.z, xv.w);
          const float s_lo = __uint_as_float((uint32_t)ssm[lrow[t][0] * sp + g] << 23);
          const float s_hi = __uint_as_float((uint32_t)ssm[lrow[t][1] * sp + g] << 23);
          acc[t][0] = fmaf(part[0], s_lo, acc[t][0]);
          acc[t][1] = fmaf(part[1], s_lo, acc[t][1]);
          acc[t][2] = fmaf(part[2], s_hi, acc[t][2]);
          acc[t][3] = fmaf(part[3], s_hi, acc[t][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[slot]);
    }
#pragma unroll
    for (int t = 0; t < RT; ++t) {
      red[warp][16 * t + r0][2 * c] = acc[t][0];
      red[warp][16 * t + r0][2 * c + 1] = acc[t][1];
      red[warp][16 * t + r0 + 8][2 * c] = acc[t][2];
      red[warp][16 * t + r0 + 8][2 * c + 1] = acc[t][3];
    }
  }
  __syncthreads();  // all warps, the producer included, meet here

  // ---- reduce the NW warps of this CTA (and undo the activation prescale) ----
  for (int i = tid; i < ROWS * 8; i += NT) {
    const int r = i >> 3, m = i & 7;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) s += red[w][r][m];
    cta_part[r][m] = m < M ? s * xunscale[m] : 0.f;
  }

  if (gridDim.y == 1) {
    __syncthreads();
    for (int i = tid; i < ROWS * M; i += NT) {
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
    for (int i = tid; i < ROWS * M; i += NT) {
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
  int rt, nw, ksplit, kc;
};

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return atoi(v);
}

// Row tile 16*RT (RT grows with M so the activation slice is amortised over
// more weight rows); K-split (a cluster) so that the activation slice stays
// <= 16 KB and there are >= 2 CTAs per SM; kc groups per pipeline stage so a
// stage is ~8 KB of weights.
GemvConfig choose_config(int N, int K, int M) {
  const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
  GemvConfig cfg;
  cfg.rt = M <= 2 ? 1 : (M <= 4 ? 2 : 4);
  cfg.nw = 4;
  const int ngroups = K / 32;
  const int tiles = cdiv(N, 16 * cfg.rt);
  cfg.ksplit = 1;
  while (cfg.ksplit < 8 && ngroups / (cfg.ksplit * 2) >= 8 &&
         ((size_t)M * 2 * K / cfg.ksplit > 16384 || tiles * cfg.ksplit < 2 * sms))
    cfg.ksplit *= 2;
  cfg.kc = 32 / cfg.rt;  // groups per stage: 16*RT rows x kc*16 bytes = 8 KB
  // explicit overrides for tuning sweeps
  cfg.rt = env_int("B200KV_GEMV_RT", cfg.rt);
  cfg.nw = env_int("B200KV_GEMV_NW", cfg.nw);
  cfg.ksplit = env_int("B200KV_GEMV_KSPLIT", cfg.ksplit);
  cfg.kc = env_int("B200KV_GEMV_KC", cfg.kc);
  return cfg;
}

template <int RT, int NW>
cudaError_t launch_gemv(const GemvConfig& cfg, const uint8_t* W, const uint8_t* St,
                        const __nv_bfloat16* X, __nv_bfloat16* Out, int N, int K, int M,
                        cudaStream_t stream) {
  const int ngroups = K / 32;
  const int gps = cdiv(ngroups, cfg.ksplit);
  const int ksplit = cdiv(ngroups, gps);
  const int kc = cfg.kc < gps ? cfg.kc : gps;
  const GemvLayout L{16 * RT, gps, kc, M};
  const size_t smem = L.bytes();
  if (smem > 200 * 1024 || kc < 1 || ksplit > 8) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(mxfp4_gemv_kernel<RT, NW>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(cdiv(N, 16 * RT), ksplit, 1);
  lc.blockDim = dim3((NW + 1) * 32, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ksplit;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, mxfp4_gemv_kernel<RT, NW>, W, St, X, Out, N, K, M, gps, kc);
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
