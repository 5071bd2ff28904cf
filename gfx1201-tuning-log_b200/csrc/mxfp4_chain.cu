// A chain of dependent MXFP4 (e2m1 + e8m0) W4A16 matvecs, 1 <= M <= 8, in one
// persistent launch on block-scaled tcgen05 MMAs (sm_100a).
//
// Each op is the product of mxfp4_mma.cu (the reference kernel h4mv_t,
// h4mv/h4mv.cu:43-104, per op):
//   out_j[m, n] = bf16_rn( sum_g 2^(S[n,g]-127) * sum_{k<32} e2m1(W_j[n,32g+k]) * x_j[m,32g+k] )
// with the same arithmetic (kind::mxf8f6f4, weights unpacked by TMA, x as two
// exact e4m3 terms, fp32 accumulation).  What the chain adds is the schedule:
// a decode step is a sequence of such products where each one reads the
// previous one's output (o -> gate_up -> down -> the next layer's qkv), and as
// separate launches every product pays a pipeline fill, its x split and a
// cross-CTA reduction on the critical path while HBM idles.  Here one CTA per
// SM runs the whole list:
//  * work: op j's weight boxes (128 rows x 128 k, tile-major) are split evenly
//    over the G CTAs, CTA c taking boxes [c T_j / G, (c + 1) T_j / G) of
//    T_j = tiles x K/128; the part of that range inside one 128-row tile is a
//    segment (a contiguous K range of that tile);
//  * warp 0 streams every box of the CTA's list, op after op, through a
//    ring of 5 stages of 2 boxes (TMA, unpacked e2m1 + the boxes' scale atoms;
//    one box per stage streams at ~3.7 TB/s on this part, two at ~5.3) -- weights are
//    load-time data, so it never waits on a dependency and runs ahead across
//    op boundaries as far as the ring allows;
//  * four activation warps write, for each box, x's 128-element slice as two
//    e4m3 terms into an 18-slot ring, in waves of 14 boxes whose (box, row,
//    32-element block) items are dealt to all 128 threads, so a wave's loads
//    and flag waits are in flight together.  When x is op d's output, the
//    slice's producing tiles of op d must be finished first: the thread spins
//    (bounded, %globaltimer, acquire loads) on their ready flags;
//  * four issuing warps take every fourth box into accumulators of their own
//    (one thread issues a block-scaled MMA about every 127 cycles);
//  * two groups of four epilogue warps take alternate segments (four
//    accumulator buffers) and drain a segment's accumulators.  A tile split over
//    several CTAs is reduced through global memory: each segment writes its
//    fp32 partial, counts itself on the tile's counter, and the last to arrive
//    adds the partials in segment order (so the result does not depend on
//    arrival order), stores the bf16 row (or the SwiGLU of a gate/up row
//    pair), and publishes the tile's ready flag.
// Flags and counters are monotonic across launches: each CTA keeps a
// generation count in the workspace, a tile is ready for launch g when its
// flag reaches g + 1, and the last arriver is the one that brings the counter
// to a multiple of the tile's segment count.  All CTAs must be resident at
// once (they wait on each other's tiles): the launch is cooperative.
//
// SwiGLU epilogue: the op's weight rows are interleaved in blocks of 64 --
// tile t holds gate rows 64 t .. 64 t + 63, then the up rows of the same
// indices -- and the op stores act[m, 64 t + r] = bf16(bf16(silu(g)) * u)
// (HF Llama's act_fn(gate) * up in bf16, the rounding of b200kv_swiglu).

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "mxfp4_tc.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200kv {
namespace {

constexpr int kMaxOps = 8;
constexpr int kTile = 128;            // weight rows per tile (MMA M)
constexpr int kStep = 128;            // K per box
constexpr int kBox = kTile * 128;     // unpacked e2m1 box in shared memory
constexpr int kBoxTx = kTile * 64;    // packed bytes the TMA signals for it
constexpr int kAtom = mx::kAtom;
constexpr int kNB = 16;               // B rows: term t of activation row m is row 8 t + m
constexpr int kBBox = kNB * 128;
constexpr int kMaxM = 8;
constexpr int kNS = 10;               // weight ring box slots
constexpr int kSB = 2;                // boxes per ring stage (one mbarrier): DRAM streams 128 B of a row per request pair
constexpr int kNST = kNS / kSB;       // ring stages
constexpr int kNXS = 18;              // activation-term ring slots
constexpr int kNI = 4;                // MMA-issuing warps
constexpr int kXW = 4;                // activation-split warps
constexpr int kEG = 2;                // epilogue warpgroups (alternate segments)
constexpr int kND = 4;                // accumulator buffers (segment sigma uses sigma % 4)
constexpr int kEw0 = 1 + kNI + kXW;   // first of the 4 kEG epilogue warps
constexpr int kThreads = 32 * (kEw0 + 4 * kEG);
constexpr int kDStride = 16 * kNI;    // accumulator buffer: 16 columns per issuer
constexpr int kColA = kND * kDStride;  // weight-scale atoms of the ring slots
constexpr int kColB = kColA + 4 * kNS;  // activation-scale atoms
constexpr uint32_t kTmemCols = 512;
static_assert(kColB + 4 * kNXS <= (int)kTmemCols, "tensor-memory columns");
constexpr int kEpiStore = B200KV_CHAIN_STORE, kEpiSwiglu = B200KV_CHAIN_SWIGLU;
constexpr unsigned long long kSpinLimitNs = 200ull * 1000 * 1000;

// shared memory: weight boxes, weight atoms, activation boxes, activation
// atoms, the SwiGLU row exchange
constexpr size_t kOffAtoms = (size_t)kNS * kBox;
constexpr size_t kOffXb = (kOffAtoms + (size_t)kNS * kAtom + 1023) / 1024 * 1024;
constexpr size_t kOffXa = kOffXb + (size_t)kNXS * kBBox;
constexpr size_t kOffEx = kOffXa + (size_t)kNXS * kAtom;
constexpr size_t kSmem = kOffEx + (size_t)kEG * kTile * kMaxM * 4 + 1024;
static_assert(kOffXb % 1024 == 0, "activation boxes must be 1024-aligned");

struct ChainOpDev {
  const uint8_t* Sp;          // packed scale atoms [tiles][K/128][512]
  const __nv_bfloat16* X;     // [M, K] rows x_ld apart
  __nv_bfloat16* Out;         // [M, N] (N/2 for SwiGLU) rows out_ld apart
  uint32_t* cnt;              // [tiles] arrival counters
  uint32_t* ready;            // [tiles] ready flags
  float* part;                // [tiles][maxseg][M][128] segment partials
  int64_t x_ld, out_ld;
  int N, K, nsteps, ntiles;
  int dep;                    // op whose output is x, or -1
  int dep_rows;               // output rows per tile of that op (128, 64 for SwiGLU)
  int epi, maxseg;
};

struct ChainArgs {
  ChainOpDev op[kMaxOps];
  uint32_t* gen;              // [G] per-CTA launch generation
  int nops, M, G;
};

struct ChainMaps {
  CUtensorMap m[kMaxOps];
};

__device__ __forceinline__ int range_start(int c, int T, int G) { return c * T / G; }
// CTA whose range holds box b
__device__ __host__ __forceinline__ int cta_of(int b, int T, int G) { return ((b + 1) * G - 1) / T; }

// segments of tile `tile` (boxes [ts, te)): CTAs with a non-empty part of it;
// returns the count and this CTA's ordinal among them
__device__ __host__ inline int tile_segments(int T, int G, int nsteps, int tile, int c, int* ord) {
  const int ts = tile * nsteps, te = ts + nsteps;
  const int f = cta_of(ts, T, G), l = cta_of(te - 1, T, G);
  int n = 0, o = -1;
  for (int cc = f; cc <= l; ++cc) {
    const int a0 = cc * T / G, a1 = (cc + 1) * T / G;
    if ((a0 > ts ? a0 : ts) < (a1 < te ? a1 : te)) {
      if (cc == c) o = n;
      ++n;
    }
  }
  if (ord) *ord = o;
  return n;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded spin until *flag reaches `want` (wrap-safe); on timeout records the
// device status and raises the CTA's abort flag.
__device__ bool wait_flag(const uint32_t* flag, uint32_t want, volatile int* abort) {
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    if ((int32_t)(ld_acquire(flag) - want) >= 0) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kSpinLimitNs) {
      atomicExch(&g_device_status, kDevChainTimeout);
      *abort = 1;
      return false;
    }
    __nanosleep(32);
  }
}

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Visits the CTA's segments in order: fn(j, tile, k0, n, s, sigma) with s the
// CTA-wide sequence number of the segment's first box; stops when fn returns false.
template <typename F>
__device__ __forceinline__ void for_each_segment(const ChainArgs& a, int c, F&& fn) {
  int s = 0, sigma = 0;
  for (int j = 0; j < a.nops; ++j) {
    const ChainOpDev& op = a.op[j];
    const int T = op.ntiles * op.nsteps;
    int b = range_start(c, T, a.G);
    const int b1 = range_start(c + 1, T, a.G);
    while (b < b1) {
      const int tile = b / op.nsteps;
      const int tend = (tile + 1) * op.nsteps;
      const int e = b1 < tend ? b1 : tend;
      const int k0 = b - tile * op.nsteps, n = e - b;
      if (!fn(j, tile, k0, n, s, sigma)) return;
      s += n;
      ++sigma;
      b = e;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    mxfp4_chain_kernel(const __grid_constant__ ChainMaps maps, const __grid_constant__ ChainArgs args) {
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kNST], empty_bar[kNST], xfull_bar[kNXS], xempty_bar[kNXS];
  __shared__ uint64_t d_full[kND], d_free[kND];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int s_abort;
  __shared__ int s_last[kEG];

  // The argument block goes to shared memory first: every role indexes its ops
  // at run time, and run-time indexing of kernel parameters makes a per-thread
  // local copy of them.
  __shared__ __align__(16) ChainArgs a_sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  static_assert(sizeof(ChainArgs) % 8 == 0, "argument block copy");
  for (int i = tid; i < (int)(sizeof(ChainArgs) / 8); i += blockDim.x)
    reinterpret_cast<uint64_t*>(&a_sm)[i] = reinterpret_cast<const uint64_t*>(&args)[i];
  __syncthreads();
  const ChainArgs& a = a_sm;
  const uint32_t gen = *reinterpret_cast<volatile uint32_t*>(&a.gen[c]);
  uint8_t* ring = dsm;
  uint8_t* ratoms = dsm + kOffAtoms;
  uint8_t* xb = dsm + kOffXb;
  uint8_t* xa = dsm + kOffXa;
  float* ex = reinterpret_cast<float*>(dsm + kOffEx);

  if (tid == 0) {
    for (int i = 0; i < kNST; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kSB);  // one commit per box
    }
    for (int i = 0; i < kNXS; ++i) {
      mbar_init(&xfull_bar[i], 4 * a.M);
      mbar_init(&xempty_bar[i], 1);
    }
    for (int b = 0; b < kND; ++b) {
      mbar_init(&d_full[b], kNI);
      mbar_init(&d_free[b], 4);
    }
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_slot;
  if (tid == 0) griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- producer: every weight box of the CTA's list ----------------------
    if (lane == 0) {
      for (int j = 0; j < a.nops; ++j) tma_prefetch_desc(&maps.m[j]);
      int total = 0;
      for_each_segment(a, c, [&](int, int, int, int n, int s, int) {
        total = s + n;
        return true;
      });
      int issued = 0;  // stages
      for_each_segment(a, c, [&](int j, int tile, int k0, int n, int s, int) {
        const ChainOpDev& op = a.op[j];
        for (int q = 0; q < n; ++q) {
          const int box = s + q, sb = box / kSB, st = sb % kNST;
          if (box % kSB == 0) {  // a new stage: its slot free, its bytes expected
            if (sb >= kNST && !mbar_wait_bounded(&empty_bar[st], ((sb / kNST) - 1) & 1)) {
              s_abort = 1;
              return false;
            }
            if (s_abort) return false;
            const int nb = total - box < kSB ? total - box : kSB;
            mbar_arrive_expect_tx(&full_bar[st], (uint32_t)(nb * (kBoxTx + kAtom)));
            issued = sb + 1;
          }
          const int slot = box % kNS;
          tma_load_2d(ring + (size_t)slot * kBox, &maps.m[j], (k0 + q) * kStep, tile * kTile, &full_bar[st]);
          bulk_g2s(ratoms + (size_t)slot * kAtom, op.Sp + ((size_t)tile * op.nsteps + k0 + q) * kAtom, kAtom,
                   &full_bar[st]);
        }
        return true;
      });
      // drain: every copy issued has landed before the CTA may exit
      for (int t = issued > kNST ? issued - kNST : 0; t < issued; ++t)
        mbar_wait_bounded(&full_bar[t % kNST], (t / kNST) & 1);
    }
  } else if (warp <= kNI) {
    // ---------------- MMA issuers: issuer ii takes boxes s with s % 4 == ii ----------------
    const int ii = warp - 1;
    if (lane == 0) {
      const uint32_t a_ring = smem_u32(ring), a_ratoms = smem_u32(ratoms);
      const uint32_t a_xb = smem_u32(xb), a_xa = smem_u32(xa);
      for_each_segment(a, c, [&](int, int, int, int n, int s, int sigma) {
        const int bsel = sigma % kND;
        if (sigma >= kND && !mbar_wait_bounded(&d_free[bsel], ((sigma / kND) - 1) & 1)) {
          s_abort = 1;
          return false;
        }
        tc::fence_after_sync();
        bool first = true;
        const uint32_t tD = tbase + (uint32_t)(bsel * kDStride + 16 * ii);
        for (int q = (ii - s % kNI + kNI) % kNI; q < n; q += kNI) {
          const int box = s + q, slot = box % kNS, xs = box % kNXS, sb = box / kSB;
          if (!mbar_wait_bounded(&full_bar[sb % kNST], (sb / kNST) & 1) ||
              !mbar_wait_bounded(&xfull_bar[xs], (box / kNXS) & 1) || s_abort) {
            s_abort = 1;
            return false;
          }
          tc::fence_after_sync();
          const uint32_t ta = tbase + kColA + 4 * slot, tb = tbase + kColB + 4 * xs;
          mx::tmem_cp_atom(ta, mx::sdesc_atom(a_ratoms + (uint32_t)slot * kAtom));
          mx::tmem_cp_atom(tb, mx::sdesc_atom(a_xa + (uint32_t)xs * kAtom));
          const uint32_t abox = a_ring + (uint32_t)slot * kBox, bbox = a_xb + (uint32_t)xs * kBBox;
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {
            const uint32_t sf = (uint32_t)kq;
            mx::mma_mxf8f6f4(tD, tc::sdesc_sw128(abox + kq * 32, 16, 1024), tc::sdesc_sw128(bbox + kq * 32, 16, 1024),
                             mx::idesc_mxf8f6f4(kTile, kNB, sf), (first && kq == 0) ? 0u : 1u, ta | (sf << 30),
                             tb | (sf << 30));
          }
          first = false;
          tc::commit(&empty_bar[sb % kNST]);
          tc::commit(&xempty_bar[xs]);
        }
        tc::commit(&d_full[bsel]);
        return true;
      });
    }
  } else if (warp < kEw0) {
    // ---------------- activation split ---------------------------------------------------
    // The CTA's boxes in waves of V = kNXS - kNI boxes; a wave's items (box, row m,
    // 32-element block grp: 4 M per box) are dealt to the 128 threads, each
    // waiting for its slots and input tiles, then loading, then converting.  The
    // four warps meet between waves, so no box starts before every box one ring
    // cycle earlier is filled: with the issuers' stride of kNI boxes that keeps
    // every mbarrier wait on these rings within one phase of its target.
    const int xt = tid - 32 * (1 + kNI);  // 0..127
    const int ipb = 4 * a.M;              // items per box
    constexpr int V = kNXS - kNI;
    constexpr int kItems = 4;             // items per thread and wave (V * 32 / 128 at most)
    int total = 0;
    for_each_segment(a, c, [&](int, int, int, int n, int s, int) {
      total = s + n;
      return true;
    });
    griddep_wait();  // inputs of the call are the previous kernel's outputs
    for (int B = 0; B < total; B += V) {
      int nit = 0, box[kItems], jj[kItems], kk[kItems], rr[kItems];
      {  // this thread's items of boxes [B, B + V)
        int idx = xt;
        const int lim = min(V, total - B) * ipb;
        for_each_segment(a, c, [&](int j, int, int k0, int n, int s, int) {
          while (nit < kItems && idx < lim) {
            const int b = B + idx / ipb;
            if (b >= s + n) return true;  // in a later segment
            box[nit] = b;
            jj[nit] = j;
            kk[nit] = k0 + (b - s);
            rr[nit] = idx % ipb;
            ++nit;
            idx += 128;
          }
          return false;
        });
      }
      // Items in runs of one op: a run's waits, then its loads (in flight
      // together), then its conversions.  A thread never waits on a ready flag
      // while it holds an unfilled box of an earlier op, which that flag's tile
      // may need (boxes of an op precede those of later ops in the list).
      bool ok = !s_abort;
      uint4 raw[kItems][4];
      for (int u0 = 0; u0 < nit && ok;) {
        int u1 = u0;
        while (u1 < nit && jj[u1] == jj[u0]) ++u1;
        const ChainOpDev& op = a.op[jj[u0]];
        for (int u = u0; u < u1 && ok; ++u) {
          const int xs = box[u] % kNXS;
          ok = box[u] < kNXS || mbar_wait_bounded(&xempty_bar[xs], ((box[u] / kNXS) - 1) & 1);
          if (ok && op.dep >= 0) {  // the tiles of op dep that produce x[:, 128 k .. 128 k + 127]
            const ChainOpDev& d = a.op[op.dep];
            for (int t = (kk[u] * kStep) / op.dep_rows; ok && t <= (kk[u] * kStep + kStep - 1) / op.dep_rows; ++t)
              ok = wait_flag(d.ready + t, gen + 1, &s_abort);
          }
        }
        if (!ok) break;
        for (int u = u0; u < u1; ++u) {
          const uint4* src = reinterpret_cast<const uint4*>(op.X + (size_t)(rr[u] >> 2) * op.x_ld +
                                                            (size_t)kk[u] * kStep + 32 * (rr[u] & 3));
#pragma unroll
          for (int q = 0; q < 4; ++q) raw[u][q] = __ldcg(src + q);
        }
        for (int u = u0; u < u1; ++u) {
          const int xs = box[u] % kNXS, m = rr[u] >> 2, grp = rr[u] & 3;
          float v[32];
#pragma unroll
          for (int q = 0; q < 4; ++q) mx::bf16x8_to_f32(raw[u][q], v + 8 * q);
          uint8_t* bx = xb + (size_t)xs * kBBox;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            float mxv = 0.f;
#pragma unroll
            for (int e = 0; e < 32; ++e) mxv = fmaxf(mxv, fabsf(v[e]));
            const int sb = mx::term_scale(mxv);
            uint32_t w[8];
            mx::term_codes<32>(v, sb, w);
            const int nrow = 8 * t + m;
            uint8_t* row = bx + nrow * 128;
            *reinterpret_cast<uint4*>(row + (((2 * grp) ^ (nrow & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(row + (((2 * grp + 1) ^ (nrow & 7)) << 4)) =
                make_uint4(w[4], w[5], w[6], w[7]);
            xa[(size_t)xs * kAtom + 16 * nrow + grp] = (uint8_t)sb;
          }
          tc::fence_proxy_async_smem();
          mbar_arrive(&xfull_bar[xs]);  // the box is complete after its 4 M items
        }
        u0 = u1;
      }
      if (!named_bar_and(2, 128, ok)) {  // one decision for the four warps
        s_abort = 1;
        break;
      }
    }
  } else {
    // ---------------- epilogue: two warpgroups take alternate segments ---------------------
    const int eg = (warp - kEw0) >> 2;       // warpgroup
    const int et = tid - 32 * (kEw0 + 4 * eg);  // 0..127 within it
    const int bar = 3 + eg;                  // its named barrier
    const int row = 32 * (warp & 3) + lane;  // tensor-memory lane = row of the tile
    const int M = a.M;
    float* exg = ex + (size_t)eg * kTile * kMaxM;
    for_each_segment(a, c, [&](int j, int tile, int, int n, int s, int sigma) {
      if (sigma % kEG != eg) return true;
      const ChainOpDev& op = a.op[j];
      const int bsel = sigma % kND;
      const bool ok = mbar_wait_bounded(&d_full[bsel], (sigma / kND) & 1);
      tc::fence_after_sync();
      float v[kMaxM];
#pragma unroll
      for (int mm = 0; mm < kMaxM; ++mm) v[mm] = 0.f;
      const uint32_t tl = tbase + (uint32_t)(bsel * kDStride) + ((uint32_t)(32 * (warp & 3)) << 16);
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // issuers 2h, 2h + 1
        float d[32];
        tc::ld32_wait(tl + 32 * h, d);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ii = 2 * h + u;
          const bool active = n >= kNI || ((ii - s % kNI + kNI) % kNI) < n;
          if (active)
#pragma unroll
            for (int mm = 0; mm < kMaxM; ++mm) v[mm] += d[16 * u + mm] + d[16 * u + 8 + mm];
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_free[bsel]);
      // one decision for the group's four warps: they meet at named barriers below
      if (!named_bar_and(bar, 128, ok && !s_abort)) {
        s_abort = 1;
        return false;
      }
      const int T = op.ntiles * op.nsteps;
      int ord = 0;
      const int nseg = tile_segments(T, a.G, op.nsteps, tile, c, &ord);
      if (nseg > 1) {
        // partial out; one thread publishes the arrival with an acquire-release
        // atomic (its release covers the group's stores, ordered before it by
        // the barrier; its acquire, the other segments' partials read below) and
        // learns whether this segment is the tile's last
        float* p = op.part + ((size_t)tile * op.maxseg + ord) * M * kTile;
#pragma unroll
        for (int mm = 0; mm < kMaxM; ++mm)
          if (mm < M) __stcg(p + mm * kTile + row, v[mm]);
        named_bar_sync(bar, 128);
        if (et == 0) s_last[eg] = ((atom_add_acq_rel(op.cnt + tile, 1u) + 1u) % (uint32_t)nseg) == 0u;
        named_bar_sync(bar, 128);
        if (!s_last[eg]) return true;
#pragma unroll
        for (int mm = 0; mm < kMaxM; ++mm) v[mm] = 0.f;
        for (int o = 0; o < nseg; ++o) {  // fixed order: the tile's segments by K
          const float* q = op.part + ((size_t)tile * op.maxseg + o) * M * kTile;
#pragma unroll
          for (int mm = 0; mm < kMaxM; ++mm)
            if (mm < M) v[mm] += __ldcg(q + mm * kTile + row);
        }
      }
      // the finished tile: bf16 rows (or SwiGLU of the gate/up row pairs)
      if (op.epi == kEpiSwiglu) {
#pragma unroll
        for (int mm = 0; mm < kMaxM; ++mm) exg[row * kMaxM + mm] = v[mm];
        named_bar_sync(bar, 128);
        if (row < 64) {
          for (int mm = 0; mm < M; ++mm) {
            const float gv = round_bf(v[mm]), uv = round_bf(exg[(row + 64) * kMaxM + mm]);
            const float sv = silu_bf16(gv);
            op.Out[(size_t)mm * op.out_ld + tile * 64 + row] = __float2bfloat16_rn(sv * uv);
          }
        }
      } else {
        const int nn = tile * kTile + row;
        if (nn < op.N)
          for (int mm = 0; mm < M; ++mm) op.Out[(size_t)mm * op.out_ld + nn] = __float2bfloat16_rn(v[mm]);
      }
      named_bar_sync(bar, 128);
      if (et == 0) st_release_u32(op.ready + tile, gen + 1);
      return true;
    });
  }

  griddep_wait();  // every thread waits before exit
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, kTmemCols);
  if (tid == 0) *reinterpret_cast<volatile uint32_t*>(&a.gen[c]) = gen + 1;
}

struct Layout {
  size_t cnt[kMaxOps], ready[kMaxOps], part[kMaxOps], gen, total;
  int maxseg[kMaxOps];
};

// workspace: per op the tile counters, the ready flags and the segment
// partials; then one generation word per CTA
bool plan_layout(const b200kv_chain_op* ops, int nops, int M, int G, Layout* L) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  for (int j = 0; j < nops; ++j) {
    const int ntiles = cdiv(ops[j].N, kTile), nsteps = ops[j].K / kStep;
    const int T = ntiles * nsteps;
    int mx = 1;
    for (int t = 0; t < ntiles; ++t) mx = std::max(mx, tile_segments(T, G, nsteps, t, -1, nullptr));
    L->maxseg[j] = mx;
    L->cnt[j] = take((size_t)ntiles * 4);
    L->ready[j] = take((size_t)ntiles * 4);
    L->part[j] = mx > 1 ? take((size_t)ntiles * mx * M * kTile * 4) : 0;
  }
  L->gen = take((size_t)G * 4);
  L->total = off;
  return true;
}

int validate(const b200kv_chain_op* ops, int nops, int M) {
  if (!ops || nops < 1 || nops > kMaxOps || M < 1 || M > kMaxM) return B200KV_ERR_INVALID_ARG;
  for (int j = 0; j < nops; ++j) {
    const b200kv_chain_op& o = ops[j];
    if (!o.weight || !o.packed_scales || !o.out || o.N <= 0 || o.K <= 0) return B200KV_ERR_INVALID_ARG;
    if (o.x_from >= j || o.x_from < -1) return B200KV_ERR_INVALID_ARG;
    if (o.epilogue != kEpiStore && o.epilogue != kEpiSwiglu) return B200KV_ERR_INVALID_ARG;
    if (o.K % kStep) return B200KV_ERR_UNSUPPORTED;
    // the work split computes (box index + 1) x CTAs in 32 bits
    if ((int64_t)cdiv(o.N, kTile) * (o.K / kStep) * 1024 >= ((int64_t)1 << 31)) return B200KV_ERR_UNSUPPORTED;
    if (o.epilogue == kEpiSwiglu && o.N % kTile) return B200KV_ERR_UNSUPPORTED;
    const int width = o.epilogue == kEpiSwiglu ? o.N / 2 : o.N;
    if (o.out_stride < width) return B200KV_ERR_INVALID_ARG;
    if (o.x_from >= 0) {
      const b200kv_chain_op& d = ops[o.x_from];
      if ((d.epilogue == kEpiSwiglu ? d.N / 2 : d.N) != o.K) return B200KV_ERR_INVALID_ARG;
      if (d.out_stride & 7 || reinterpret_cast<uintptr_t>(d.out) & 15) return B200KV_ERR_MISALIGNED;
    } else {
      if (!o.x || o.x_stride < o.K) return B200KV_ERR_INVALID_ARG;
      if (o.x_stride & 7 || reinterpret_cast<uintptr_t>(o.x) & 15) return B200KV_ERR_MISALIGNED;
    }
    if ((reinterpret_cast<uintptr_t>(o.weight) | reinterpret_cast<uintptr_t>(o.packed_scales)) & 15)
      return B200KV_ERR_MISALIGNED;
  }
  return B200KV_OK;
}

cudaError_t raise_smem_limit() {
  static std::once_flag once;
  static cudaError_t e = cudaSuccess;
  std::call_once(once, [] {
    e = cudaFuncSetAttribute(mxfp4_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  });
  return e;
}

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

// CTAs of the persistent grid: one per SM (B200KV_CHAIN_CTAS overrides, for tests)
int grid_ctas() {
  const int sms = num_sms_current_device();
  const int force = env_int("B200KV_CHAIN_CTAS", 0);
  return force > 0 ? std::min(force, sms) : sms;
}

}  // namespace

size_t mxfp4_chain_workspace_bytes(const b200kv_chain_op* ops, int nops, int M) {
  if (validate(ops, nops, M) != B200KV_OK) return 0;
  const int G = grid_ctas();
  if (G <= 0) return 0;
  Layout L;
  plan_layout(ops, nops, M, G, &L);
  return L.total;
}

int mxfp4_chain_launch(const b200kv_chain_op* ops, int nops, int M, void* ws, size_t ws_bytes, void* stream) {
  const int v = validate(ops, nops, M);
  if (v != B200KV_OK) return v;
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255)) return B200KV_ERR_WORKSPACE;
  const int G = grid_ctas();
  if (G <= 0 || sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  Layout L;
  plan_layout(ops, nops, M, G, &L);
  if (ws_bytes < L.total) return B200KV_ERR_WORKSPACE;

  ChainMaps maps;
  ChainArgs a = {};
  uint8_t* base = static_cast<uint8_t*>(ws);
  for (int j = 0; j < nops; ++j) {
    const b200kv_chain_op& o = ops[j];
    ChainOpDev& d = a.op[j];
    if (!encode_e2m1_unpacked_2d(&maps.m[j], o.weight, (uint64_t)o.K, (uint64_t)o.N, (uint64_t)(o.K / 2), kTile))
      return B200KV_ERR_UNSUPPORTED;
    d.Sp = static_cast<const uint8_t*>(o.packed_scales);
    d.dep = o.x_from;
    if (o.x_from >= 0) {
      d.X = static_cast<const __nv_bfloat16*>(ops[o.x_from].out);
      d.x_ld = ops[o.x_from].out_stride;
      d.dep_rows = ops[o.x_from].epilogue == kEpiSwiglu ? 64 : kTile;
    } else {
      d.X = static_cast<const __nv_bfloat16*>(o.x);
      d.x_ld = o.x_stride;
      d.dep_rows = kTile;
    }
    d.Out = static_cast<__nv_bfloat16*>(o.out);
    d.out_ld = o.out_stride;
    d.N = o.N;
    d.K = o.K;
    d.nsteps = o.K / kStep;
    d.ntiles = cdiv(o.N, kTile);
    d.epi = o.epilogue;
    d.maxseg = L.maxseg[j];
    d.cnt = reinterpret_cast<uint32_t*>(base + L.cnt[j]);
    d.ready = reinterpret_cast<uint32_t*>(base + L.ready[j]);
    d.part = L.maxseg[j] > 1 ? reinterpret_cast<float*>(base + L.part[j]) : nullptr;
  }
  a.gen = reinterpret_cast<uint32_t*>(base + L.gen);
  a.nops = nops;
  a.M = M;
  a.G = G;

  cudaError_t e = raise_smem_limit();
  if (e != cudaSuccess) return B200KV_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on each other's tiles
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() && env_int("B200KV_CHAIN_PDL", 1) ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, mxfp4_chain_kernel, maps, a);
  if (env_int("B200KV_CHAIN_PLAN", 0))
    fprintf(stderr, "[b200kv] mxfp4_chain ops=%d M=%d ctas=%d smem=%zu workspace=%zu launch=%s\n", nops, M, G,
            (size_t)kSmem, L.total, cudaGetErrorString(e));
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
