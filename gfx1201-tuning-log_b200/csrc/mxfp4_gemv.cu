// MXFP4 (e2m1 + e8m0) W4A16 matvec / skinny GEMM for sm_100a, 1 <= M <= 8.
//
// Computes out[m, n] = bf16_rn( sum_g scale(St[n,g]) * sum_{j<32} e2m1(W[n,32g+j]) * x[m,32g+j] )
// with fp32 accumulation -- the arithmetic of the reference kernel
// h4mv/h4mv.cu:43-104 (h4mv_t<MT>), re-designed for B200:
//
//  * Persistent thread-block clusters.  The ks CTAs of a cluster (ks in
//    {1,2,4,8}) split K; the clusters split the 16-row weight tiles round-robin.
//    ks is chosen to balance the tiles over the clusters (148 SMs rarely divide
//    N/16) and to keep the activation slice small.  Each CTA keeps its tiles'
//    fp32 partials in shared memory and the cluster reduces them once, at the
//    end, through distributed shared memory: no global scratch, one launch.
//  * Warp-specialised: one producer warp streams (tile, K-chunk) stages
//    through a 4- to 6-deep ring with TMA tensor-map loads -- the weights as
//    128-byte-swizzled 16-row boxes (2 KB per request) and the scales as a
//    [kc groups x 16 rows] box -- with a full/empty mbarrier handshake, so HBM
//    sees a continuous stream of large requests (small bulk requests were
//    measured to cap at ~2 TB/s on this part).
//  * The activation slice is staged once per CTA and converted to f16 with an
//    exact per-row power-of-two prescale (row maximum in [2^4, 2^5)): every bf16
//    value within 2^-18 of its row's maximum keeps its 8-bit significand,
//    smaller ones round to f16 subnormals (their products vanish in the fp32
//    sum), none can overflow.  The prescale is undone exactly at the end.
//  * Weights are decoded with the Blackwell hardware convert
//    cvt.rn.f16x2.e2m1x2 (one instruction per byte, exact) and multiplied on
//    the tensor pipe through mma.sync m16n8k16 (A = 16 weight rows x 16 k,
//    B = 16 k x 8 activation rows), used as a wide fp32-accumulating dot
//    product engine -- a matvec needs 2*M multiply-adds per weight byte, which
//    would saturate the FP32 pipe and the issue slots long before HBM does.
//    The reference made the same move on gfx1201 with v_dot2_f32_bf16
//    (h4mv.cu:26-31).
//  * Group-aligned fragments: lane (r0 = lane/4, c = lane%4) takes bytes
//    4c..4c+3 of one 16-byte group (32 weights = one e8m0 group) of rows r0 and
//    r0+8, so the two MMAs of a group cover exactly that group and the group
//    scale multiplies the group's fp32 partial -- the reference's per-group
//    structure (h4mv.cu:72-90), exact for every scale byte.
//
// Edge semantics follow the reference kernel: the scale is the fp32 bit pattern
// s << 23, so byte 0 -> 0.0 and 255 -> inf.  The activation prescale can push
// a partial sum past fp32's range only when the reference's own result is
// within a factor 2^5 of it.  Output rounding: fp32 -> bf16 RN-even.

#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace b200kv {
namespace {

constexpr int kTileRows = 16;
constexpr int kMaxStages = 8;
constexpr int kMaxClusterK = 8;

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

struct GemvArgs {
  const uint8_t* St;  // scale bytes [N, K/32] (read directly when not staged by TMA)
  const __nv_bfloat16* X;
  __nv_bfloat16* Out;
  int N, K, M;
  int gps;        // groups per K-slice (multiple of 16)
  int kc;         // groups per stage (multiple of 16)
  int nstages;    // ring depth (<= kMaxStages)
  int ntiles;     // cdiv(N, 16)
  int nclusters;  // clusters (each owns tiles cid, cid + nclusters, ...)
  int tmax;       // cdiv(ntiles, nclusters): partial slots per CTA
};

// Shared-memory layout.  Stage = kc/8 weight boxes of [128 B x 16 rows]
// (128B-swizzled, 2 KB each) + one scale box [kc B x 16 rows]; stages are
// 1024-byte aligned as the swizzle pattern requires.  Activation rows: pitch
// == 64 (mod 128) so the 8-lane phases of a 128-bit load hit distinct 16-byte
// bank groups.  kc is a divisor of the slice's groups (no wasted loads).
struct GemvLayout {
  int kc, gps, m, tmax, nw, nstages;
  __host__ __device__ int w_bytes() const { return kc * 16 * kTileRows; }
  __host__ __device__ int stage_bytes() const { return (w_bytes() + kTileRows * kc + 1023) & ~1023; }
  __host__ __device__ int xp() const { return ((gps * 64 + 127) & ~127) + 64; }
  __host__ __device__ size_t x_off() const { return (size_t)nstages * stage_bytes(); }
  __host__ __device__ size_t part_off() const { return x_off() + (((size_t)m * xp() + 15) & ~(size_t)15); }
  __host__ __device__ size_t red_off() const { return part_off() + (size_t)tmax * kTileRows * 8 * 4; }
  __host__ __device__ size_t bytes() const { return red_off() + (size_t)nw * kTileRows * 8 * 4 + 1024; }
};

// STMA: scales through the TMA ring (needs K/32 to be a multiple of 16 bytes);
// otherwise each lane reads its scale bytes from global memory (L1-cached).
template <int NW, bool STMA>
__global__ void __launch_bounds__((NW + 1) * 32)
    mxfp4_gemv_kernel(const __grid_constant__ CUtensorMap wmap,
                      const __grid_constant__ CUtensorMap smap, const GemvArgs a) {
  constexpr int NC = NW * 32;  // consumer threads
  constexpr int NT = NC + 32;
  __shared__ float xunscale[8];
  __shared__ float xmax_part[NW][8];
  __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], x_bar;
  extern __shared__ uint8_t dsm_raw[];
  // 1024-byte align the dynamic region (the 128-byte swizzle needs it)
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool producer = warp == NW;
  const int r0 = lane >> 2;
  const int c = lane & 3;
  const int M = a.M;
  const int ngroups = a.K >> 5;
  const int rank = blockIdx.x;  // K-slice = rank in the cluster
  const int cid = blockIdx.y;
  const int g_begin = rank * a.gps;
  const int ng = max(0, min(ngroups, g_begin + a.gps) - g_begin);
  const int kc = a.kc;
  const int nch = (ng + kc - 1) / kc;
  const int my_tiles = cid < a.ntiles ? (a.ntiles - cid + a.nclusters - 1) / a.nclusters : 0;
  const int nstages = a.nstages;
  const GemvLayout L{kc, a.gps, M, a.tmax, NW, nstages};
  const int stage_bytes = L.stage_bytes();
  const int xp = L.xp();
  uint8_t* xsm = dsm + L.x_off();
  float* part = reinterpret_cast<float*>(dsm + L.part_off());  // [tmax][16][8]
  float* red = reinterpret_cast<float*>(dsm + L.red_off());    // [NW][16][8]

  if (tid == 0) {
    for (int i = 0; i < nstages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], NW);
    }
    mbar_init(&x_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  if (producer) {
    if (lane == 0) {
      tma_prefetch_desc(&wmap);
      tma_prefetch_desc(&smap);
      mbar_arrive_expect_tx(&x_bar, (uint32_t)(M * ng * 64));
    }
    __syncwarp();
    if (lane < M && ng > 0)
      bulk_g2s(xsm + lane * xp, a.X + (size_t)lane * a.K + (size_t)g_begin * 32,
               (uint32_t)(ng * 64), &x_bar);
    // ---- (tile, chunk) stages through the ring --------------------------------
    if (lane == 0) {
      const uint32_t tx = (uint32_t)(L.w_bytes() + (STMA ? kTileRows * kc : 0));
      int s = 0;
      for (int i = 0; i < my_tiles && !failed; ++i) {
        const int row0 = (cid + i * a.nclusters) * kTileRows;
        for (int j = 0; j < nch && !failed; ++j, ++s) {
          const int slot = s % nstages;
          if (s >= nstages) failed = !mbar_wait_bounded(&empty_bar[slot], ((s / nstages) - 1) & 1);
          if (failed) break;
          uint8_t* st = dsm + (size_t)slot * stage_bytes;
          mbar_arrive_expect_tx(&full_bar[slot], tx);
          const int gx = g_begin + j * kc;
          for (int b = 0; b < kc / 8; ++b)
            tma_load_2d(st + b * 2048, &wmap, (gx + 8 * b) * 16, row0, &full_bar[slot]);
          if (STMA) tma_load_2d(st + L.w_bytes(), &smap, gx, row0, &full_bar[slot]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---- activations: exact per-row power-of-two prescale into f16 ------------
    if (ng > 0) failed = !mbar_wait_bounded(&x_bar, 0);
    const int per_row = ng * 4;  // uint4 per row
    for (int m = 0; m < M; ++m) {
      const uint4* row = reinterpret_cast<const uint4*>(xsm + m * xp);
      float mx = 0.f;
      for (int i = tid; i < per_row && !failed; i += NC) {
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
      for (int i = tid; i < per_row && !failed; i += NC) {
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

    // ---- math: consumer warp w takes 4-group steps w, w+NW, ... of a chunk ----
    const uint8_t* xrow = xsm + min(r0, M - 1) * xp + 16 * c;
    const int swz = r0 & 7;  // 128-byte swizzle of rows r0 and r0+8
    int s = 0;
    for (int i = 0; i < my_tiles; ++i) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int row0 = (cid + i * a.nclusters) * kTileRows;
      const uint8_t* sg_lo = a.St + (size_t)min(row0 + r0, a.N - 1) * ngroups + g_begin;
      const uint8_t* sg_hi = a.St + (size_t)min(row0 + r0 + 8, a.N - 1) * ngroups + g_begin;
      for (int j = 0; j < nch; ++j, ++s) {
        const int slot = s % nstages;
        if (!failed) failed = !mbar_wait_bounded(&full_bar[slot], (s / nstages) & 1);
        const int kcs = failed ? 0 : min(kc, ng - j * kc);
        const uint8_t* st = dsm + (size_t)slot * stage_bytes;
        const uint8_t* ssc = st + L.w_bytes();
        for (int q = warp; q * 4 < kcs; q += NW) {
          uint32_t s4_lo, s4_hi;
          if constexpr (STMA) {
            s4_lo = *reinterpret_cast<const uint32_t*>(ssc + r0 * kc + 4 * q);
            s4_hi = *reinterpret_cast<const uint32_t*>(ssc + (r0 + 8) * kc + 4 * q);
          } else {
            s4_lo = s4_hi = 0u;
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (4 * q + u < kcs) {
                s4_lo |= (uint32_t)__ldg(sg_lo + j * kc + 4 * q + u) << (8 * u);
                s4_hi |= (uint32_t)__ldg(sg_hi + j * kc + 4 * q + u) << (8 * u);
              }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int gl = 4 * q + u;
            if (gl < kcs) {
              const uint4 xv = *reinterpret_cast<const uint4*>(xrow + (j * kc + gl) * 64);
              const uint8_t* box = st + (gl >> 3) * 2048 + (((gl & 7) ^ swz) << 4) + 4 * c;
              const uint32_t w_lo = *reinterpret_cast<const uint32_t*>(box + r0 * 128);
              const uint32_t w_hi = *reinterpret_cast<const uint32_t*>(box + (r0 + 8) * 128);
              uint32_t a_lo[4], a_hi[4];
              e2m1x8_to_f16x2(w_lo, a_lo);
              e2m1x8_to_f16x2(w_hi, a_hi);
              float pr[4] = {0.f, 0.f, 0.f, 0.f};
              mma_16816_f16(pr, a_lo[0], a_hi[0], a_lo[1], a_hi[1], xv.x, xv.y);
              mma_16816_f16(pr, a_lo[2], a_hi[2], a_lo[3], a_hi[3], xv.z, xv.w);
              const float sl = __uint_as_float(((s4_lo >> (8 * u)) & 0xFFu) << 23);
              const float sh = __uint_as_float(((s4_hi >> (8 * u)) & 0xFFu) << 23);
              acc[0] = fmaf(pr[0], sl, acc[0]);
              acc[1] = fmaf(pr[1], sl, acc[1]);
              acc[2] = fmaf(pr[2], sh, acc[2]);
              acc[3] = fmaf(pr[3], sh, acc[3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[slot]);
      }
      // ---- fold the consumer warps: tile partial (activation prescale undone) --
      red[(warp * kTileRows + r0) * 8 + 2 * c] = acc[0];
      red[(warp * kTileRows + r0) * 8 + 2 * c + 1] = acc[1];
      red[(warp * kTileRows + r0 + 8) * 8 + 2 * c] = acc[2];
      red[(warp * kTileRows + r0 + 8) * 8 + 2 * c + 1] = acc[3];
      named_bar_sync(1, NC);
      if (tid < kTileRows * 8) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) v += red[w * kTileRows * 8 + tid];
        const int m = tid & 7;
        part[i * kTileRows * 8 + tid] = m < M ? v * xunscale[m] : 0.f;
      }
      named_bar_sync(1, NC);
    }
  }

  // ---- reduce the cluster's K-slices through distributed shared memory -------
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int ks = (int)cluster.num_blocks();
  for (int i = rank; i < my_tiles; i += ks) {
    const int row0 = (cid + i * a.nclusters) * kTileRows;
    for (int e = tid; e < kTileRows * M; e += NT) {
      const int m = e / kTileRows, r = e % kTileRows;
      float v = 0.f;
      for (int q = 0; q < ks; ++q) v += cluster.map_shared_rank(part, q)[(i * kTileRows + r) * 8 + m];
      const int n = row0 + r;
      if (n < a.N) a.Out[(size_t)m * a.N + n] = __float2bfloat16_rn(v);
    }
  }
  cluster.sync();  // peers' shared memory stays alive until every rank is done
}

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return atoi(v);
}

struct GemvPlan {
  int ks, nclusters, gps, kc, nstages, tmax;
  size_t smem;
};

// K-split ks in {1,2,4,8}: 1 unless there are too few 16-row tiles for the
// CTAs (then the best-balanced split), subject to an activation slice of at
// most 64 KB and at least 32 groups per slice.  Stage = kc groups (the largest
// of 64/48/32/16 dividing the slice); 4 stages with two CTAs per SM when they
// fit, else one CTA with 6 stages.  (Measured on B200: 64-group stages with 8
// consumer warps beat better-balanced splits with smaller stages.)
bool plan_gemv(int N, int K, int M, int nw, GemvPlan* P) {
  const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
  const int ngroups = K / 32;
  const int ntiles = cdiv(N, kTileRows);
  const int forced = env_int("B200KV_GEMV_KSPLIT", 0);
  const int kc_env = env_int("B200KV_GEMV_KC", 0);
  const int st_env = env_int("B200KV_GEMV_STAGES", 0);
  double best = -1.0;
  bool ok = false;
  for (int ks = 1; ks <= kMaxClusterK; ks *= 2) {
    if (forced && ks != forced) continue;
    int gps = cdiv(ngroups, ks);
    gps = (gps + 15) & ~15;
    if (cdiv(ngroups, gps) != ks) continue;  // would leave a rank without groups
    if (!forced && ks > 1 && (gps < 32 || ntiles >= 4 * sms)) continue;
    if (!forced && (size_t)M * gps * 64 > 65536 && ks < kMaxClusterK) continue;
    int kc = 16;
    for (int cand : {64, 48, 32, 16})
      if (gps % cand == 0) { kc = cand; break; }
    if (kc_env) kc = kc_env;
    if (kc < 16 || kc % 16 || kc > 256) return false;
    for (int cps = 2; cps >= 1; --cps) {
      int ncl = sms * cps / ks;
      if (ncl > ntiles) ncl = ntiles;
      if (ncl < 1) ncl = 1;
      const int tmax = cdiv(ntiles, ncl);
      int nst = st_env ? st_env : (cps == 2 ? 4 : 6);
      if (nst > kMaxStages) nst = kMaxStages;
      const GemvLayout L{kc, gps, M, tmax, nw, nst};
      const size_t smem = L.bytes();
      if (smem * cps > 220 * 1024) continue;
      const double bal = (double)ntiles / ncl / tmax + (ks == 1 ? 1e-3 : 0.0) + cps * 1e-4;
      if (bal > best) {
        best = bal;
        *P = GemvPlan{ks, ncl, gps, kc, nst, tmax, smem};
        ok = true;
      }
      break;  // the larger cps that fits is preferred
    }
  }
  return ok;
}

template <int NW, bool STMA>
cudaError_t launch_gemv(const GemvPlan& P, const CUtensorMap& wmap, const CUtensorMap& smap,
                        const uint8_t* St, const __nv_bfloat16* X, __nv_bfloat16* Out, int N,
                        int K, int M, cudaStream_t stream) {
  static int attr_set = 0;  // largest dynamic smem already enabled for this instantiation
  cudaError_t e = cudaSuccess;
  if ((int)P.smem > attr_set) {
    e = cudaFuncSetAttribute(mxfp4_gemv_kernel<NW, STMA>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem);
    if (e != cudaSuccess) return e;
    attr_set = (int)P.smem;
  }
  GemvArgs a;
  a.St = St;
  a.X = X;
  a.Out = Out;
  a.N = N;
  a.K = K;
  a.M = M;
  a.gps = P.gps;
  a.kc = P.kc;
  a.nstages = P.nstages;
  a.ntiles = cdiv(N, kTileRows);
  a.nclusters = P.nclusters;
  a.tmax = P.tmax;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(P.ks, P.nclusters, 1);
  lc.blockDim = dim3((NW + 1) * 32, 1, 1);
  lc.dynamicSmemBytes = P.smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, mxfp4_gemv_kernel<NW, STMA>, wmap, smap, a);
}

}  // namespace

int mxfp4_gemv_launch(const void* W, const void* St, const void* X, void* out, int N, int K,
                      int M, void* stream) {
  if (!W || !St || !X || !out) return B200KV_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || M <= 0) return B200KV_ERR_INVALID_ARG;
  if (M > 8 || (K % 32) != 0) return B200KV_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and row pitches (K/2 and K/32 bytes)
  if ((reinterpret_cast<uintptr_t>(W) & 15) ||
      ((K / 32) % 16 == 0 && (reinterpret_cast<uintptr_t>(St) & 15)) ||
      (reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(out) & 1))
    return B200KV_ERR_MISALIGNED;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  const bool stma = (K / 32) % 16 == 0;  // scale rows are 16-byte multiples
  const int nw = env_int("B200KV_GEMV_NW", 8);
  GemvPlan P;
  if (!plan_gemv(N, K, M, nw, &P)) return B200KV_ERR_UNSUPPORTED;
  CUtensorMap wmap, smap;
  if (!encode_u8_2d(&wmap, W, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, 128, kTileRows, true))
    return B200KV_ERR_LAUNCH;
  if (stma) {
    if (!encode_u8_2d(&smap, St, (uint64_t)K / 32, (uint64_t)N, (uint64_t)K / 32, (uint32_t)P.kc,
                      kTileRows, false))
      return B200KV_ERR_LAUNCH;
  } else {
    smap = wmap;  // unused
  }
  const uint8_t* sb = static_cast<const uint8_t*>(St);
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(X);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (nw * 2 + (stma ? 1 : 0)) {
    case 9: e = launch_gemv<4, true>(P, wmap, smap, sb, x, o, N, K, M, st); break;
    case 8: e = launch_gemv<4, false>(P, wmap, smap, sb, x, o, N, K, M, st); break;
    case 17: e = launch_gemv<8, true>(P, wmap, smap, sb, x, o, N, K, M, st); break;
    case 16: e = launch_gemv<8, false>(P, wmap, smap, sb, x, o, N, K, M, st); break;
    case 33: e = launch_gemv<16, true>(P, wmap, smap, sb, x, o, N, K, M, st); break;
    case 32: e = launch_gemv<16, false>(P, wmap, smap, sb, x, o, N, K, M, st); break;
    default: return B200KV_ERR_INVALID_ARG;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
