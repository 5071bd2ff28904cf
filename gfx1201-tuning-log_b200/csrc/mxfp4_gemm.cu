// MXFP4 (e2m1 + e8m0) W4A16 GEMM for wide batches (M >= 16: prefill chunks,
// batched decode) on block-scaled tcgen05 MMAs, sm_100a.
//
// Same product as mxfp4_gemv.cu / mxfp4_mma.cu (the reference kernel
// h4mv/h4mv.cu:43-104, and at M > 8 the reference's dequant + matmul,
// h4mv/fp8kv_hipw4.py:62-94):
//   out[m, n] = bf16_rn( sum_g 2^(S[n,g]-127) * sum_{j<32} e2m1(W[n,32g+j]) * x[m,32g+j] )
// computed by tcgen05.mma.kind::mxf8f6f4.block_scale.block32 with
//  * A = a 128-row weight tile in e2m1, brought in by TMA from the packed
//    checkpoint layout and unpacked on the way (16 codes per 16-byte chunk, the
//    tensor core's 4-bit operand layout of this kind), with the weight scales
//    from the same 512-byte scale atoms the M <= 8 kernel uses
//    (b200kv_mxfp4_pack_scales);
//  * B = the activations written, by a pre-pass, as two e4m3 terms with their
//    own e8m0 scale per 32-element block: x = t0 * 2^(s0-127) + t1 * 2^(s1-127).
//    The first term takes the top four significant bits of every element (the
//    block maximum scaled into [128, 256)), the second the remainder, which
//    for a bf16 element (eight significant bits) has at most four: both terms
//    are exact for every element within 2^-13 of its block maximum, and an
//    element below that loses at most 2^-21 of the block maximum.  The two
//    terms sit in the N dimension (B row 64 t + j of a 64-token tile), one MMA
//    computes both products and the epilogue adds them.
// So every product is the exact dequantised product and the accumulation is
// fp32, as the reference's dequant + fp32 matmul.  Against the six-term e2m1
// split of mxfp4_mma.cu this is a third of the tensor work (two 8-bit terms at
// half the 4-bit rate) and exact.
//
// Work split: a CTA computes MT weight tiles x NT token tiles over one K-slice;
// a thread-block cluster of ks CTAs splits K, and each CTA finishes a band of
// ceil(128 MT / ks) weight rows: the other ranks push their partials of that
// band (st.async into its shared memory), it adds the ks partials in rank
// order and stores bf16.  Warp 0 streams the stages (A box, B box, their scale
// atoms) through an mbarrier ring, warp 1 issues the MMAs from one thread,
// warps 2-5 drain the accumulators.  Weights stream before the kernel waits on
// the pre-pass (programmatic dependent launch).

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <map>
#include <mutex>
#include <tuple>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "mxfp4_tc.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200kv {
namespace {

constexpr int kRows = 128;            // weight rows per MMA tile (MMA M)
constexpr int kTok = 64;              // activation rows per token tile
constexpr int kBRows = 2 * kTok;      // B rows of a token tile: term t of token j is row 64 t + j (MMA N)
constexpr int kKStep = 128;           // K per step: one A box, one B box and one scale atom each
constexpr int kABox = kRows * 128;    // A box in shared memory (e2m1 codes, 16 per 16-byte chunk)
constexpr int kABoxTx = kRows * 64;   // bytes the TMA signals for it (the packed size)
constexpr int kBBox = kBRows * 128;   // B box: e4m3 codes, 128 B rows, 128-byte swizzle
constexpr int kAtom = mx::kAtom;      // scale atom: 128 rows x 4 groups
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kTmemCols = 512;
constexpr int kSfCol = 256;           // first tensor-memory column of the scale-atom ring
constexpr int kSmemMax = 227 * 1024;

using mx::e4m3x2;
using mx::e4m3x2_val;
using mx::idesc_mxf8f6f4;
using mx::mma_mxf8f6f4;
using mx::sdesc_atom;
using mx::term_scale;
using mx::tmem_cp_atom;

// x [M, K] (row stride x_ld) -> the B operand of every 64-token tile tt,
// Xq[tt][128][K] (row 64 t + j = term t of token 64 tt + j, e4m3), and its
// scale atoms Xs[tt][K/128][512] (byte 16 (row % 32) + 4 (row / 32) + group).
// One thread per (token, 32-element block); tokens past M get zero codes.
__global__ void __launch_bounds__(256) xsplit_e4m3_kernel(const __nv_bfloat16* __restrict__ X, int64_t x_ld,
                                                          uint8_t* __restrict__ Xq, uint8_t* __restrict__ Xs,
                                                          int M, int K, int ttiles) {
  griddep_launch_dependents();
  // x is the previous kernel's output, and the previous GEMM may still read
  // Xq / Xs: wait for it before reading or writing anything
  griddep_wait();
  const int ngroups = K >> 5, nsteps = K / kKStep;
  const int64_t total = (int64_t)ttiles * kTok * ngroups;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / ngroups), g = (int)(i % ngroups);
    float r[32];
    if (m < M) {
      const uint4* src = reinterpret_cast<const uint4*>(X + (size_t)m * x_ld + 32 * (size_t)g);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 v = __ldg(src + q);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          r[8 * q + 2 * e] = __uint_as_float(u[e] << 16);
          r[8 * q + 2 * e + 1] = __uint_as_float(u[e] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) r[e] = 0.f;
    }
    const int tt = m / kTok, tl = m % kTok;
    uint8_t* atom = Xs + ((size_t)tt * nsteps + (g >> 2)) * kAtom;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      float mx = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) mx = fmaxf(mx, fabsf(r[e]));
      const int sb = term_scale(mx);
      const float inv = __uint_as_float((uint32_t)(254 - sb) << 23);  // 2^-(sb-127)
      const float scl = sb ? __uint_as_float((uint32_t)sb << 23) : 0x1p-127f;  // 2^(sb-127)
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t c0 = e4m3x2(r[4 * k] * inv, r[4 * k + 1] * inv);
        const uint32_t c1 = e4m3x2(r[4 * k + 2] * inv, r[4 * k + 3] * inv);
        const float2 v0 = e4m3x2_val(c0), v1 = e4m3x2_val(c1);
        r[4 * k] = fmaf(-v0.x, scl, r[4 * k]);
        r[4 * k + 1] = fmaf(-v0.y, scl, r[4 * k + 1]);
        r[4 * k + 2] = fmaf(-v1.x, scl, r[4 * k + 2]);
        r[4 * k + 3] = fmaf(-v1.y, scl, r[4 * k + 3]);
        w[k] = c0 | (c1 << 16);
      }
      const int row = kTok * t + tl;
      uint4* dst = reinterpret_cast<uint4*>(Xq + ((size_t)tt * kBRows + row) * K + 32 * (size_t)g);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      atom[16 * (row & 31) + 4 * (row >> 5) + (g & 3)] = (uint8_t)sb;
    }
  }
}

struct GemmArgs {
  const uint8_t* Sp;   // packed weight scale atoms [ceil(N/128)][K/128][512]
  const uint8_t* Xs;   // activation-term scale atoms [ttiles][K/128][512]
  __nv_bfloat16* Out;  // [M, N]
  int N, K, M;
  int nsteps;          // K / 128
  int sps;             // steps per K-slice
  int kb;              // steps per stage (1 or 2)
  int nstages;         // ring depth
  int wtiles;          // ceil(N / 128)
  int ttiles;          // ceil(M / 64)
  int vec_out;         // Out 16-byte aligned and N % 8 == 0: 16-byte output stores
  int n256;            // NT = 2: both token tiles in one N = 256 MMA (B200KV_GEMM_N256=0: two of 128)
  int swiglu;          // Out [M, N / 2] = SwiGLU of row-interleaved gate_up weights (K unsplit, vec_out)
};


// Dynamic shared memory: the stage ring, then (ks > 1) the receive area of the
// K-slice reduction, recv[src rank][band row][tokens] in fp32, whose 16-byte
// chunks are rotated by (band row & 7) so the finishing reads of 32
// consecutive rows hit distinct banks.  A stage holds kb steps: the A boxes
// (step q, weight tile mt), the B boxes (q, token tile nt), then the scale
// atoms, each operand's kb atoms contiguous (one bulk copy each, as they lie
// in memory).  Every mbarrier round trip of the ring costs a few hundred ns
// on the single-thread producer and issuer, so a stage must carry enough
// weight bytes to cover it.
template <int MT, int NT>
struct GemmLayout {
  int nstages, ks, kb;
  __host__ __device__ int stage() const {
    return (kb * (MT * kABox + NT * kBBox + (MT + NT) * kAtom) + 1023) / 1024 * 1024;
  }
  __host__ __device__ int a_off(int mt, int q) const { return (q * MT + mt) * kABox; }
  __host__ __device__ int b_off(int nt, int q) const { return kb * MT * kABox + (q * NT + nt) * kBBox; }
  __host__ __device__ int sfa_off(int mt, int q) const {
    return kb * (MT * kABox + NT * kBBox) + (mt * kb + q) * kAtom;
  }
  __host__ __device__ int sfb_off(int nt, int q) const {
    return kb * (MT * kABox + NT * kBBox) + ((MT + nt) * kb + q) * kAtom;
  }
  __host__ __device__ int band() const { return (MT * kRows + ks - 1) / ks; }
  __host__ __device__ size_t recv() const { return (size_t)nstages * stage(); }
  __host__ __device__ size_t bytes() const {
    return recv() + (ks > 1 ? (size_t)ks * band() * NT * kTok * 4 : 0) + 1024;
  }
};

template <int MT, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    mxfp4_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const GemmArgs a) {
  using L = GemmLayout<MT, NT>;
  constexpr int kT = NT * kTok;  // tokens of the CTA tile
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages];
  __shared__ uint64_t d_full, recv_bar;
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x, ksz = gridDim.x;  // K-slice = rank in the cluster (ks, 1, 1)
  const int wt0 = blockIdx.y * MT, tt0 = blockIdx.z * NT;
  const int s_begin = rank * a.sps;
  const int ns = max(0, min(a.nsteps, s_begin + a.sps) - s_begin);  // 128-k steps of this slice
  const int kb = a.kb;
  const int nstg = (ns + kb - 1) / kb;  // stages of this slice
  const int mt_n = min(MT, a.wtiles - wt0), nt_n = min(NT, a.ttiles - tt0);
  const int nst = a.nstages;
  const L lay{nst, ksz, kb};
  const int stage_bytes = lay.stage();
  const int band = lay.band();
  const int my_rows = max(0, min(band, MT * kRows - rank * band));
  float* recv = reinterpret_cast<float*>(dsm + lay.recv());
  const uint32_t recv_bytes = ksz > 1 ? (uint32_t)((ksz - 1) * my_rows * kT * 4) : 0u;

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    mbar_init(&d_full, 1);
    mbar_init(&recv_bar, 1);
    fence_mbar_init();
    if (recv_bytes) mbar_arrive_expect_tx(&recv_bar, recv_bytes);  // peers' pushes complete it
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_slot;
  if (ksz > 1) cluster_arrive_relaxed();  // recv_bar is initialised (peers wait before pushing)
  if (tid == 0) griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ---------------------------------------------------
    if (lane == 0 && ns > 0) {
      tma_prefetch_desc(&wmap);
      tma_prefetch_desc(&xmap);
      auto steps_of = [&](int s) { return min(kb, ns - s * kb); };
      auto tx_of = [&](int s) {
        return (uint32_t)(steps_of(s) * (mt_n * (kABoxTx + kAtom) + nt_n * (kBBox + kAtom)));
      };
      auto issue_w = [&](int s) {
        uint8_t* st = dsm + (size_t)(s % nst) * stage_bytes;
        uint64_t* bar = &full_bar[s % nst];
        const int k = s_begin + s * kb, nq = steps_of(s);
        for (int mt = 0; mt < mt_n; ++mt) {
          for (int q = 0; q < nq; ++q)
            tma_load_2d(st + lay.a_off(mt, q), &wmap, (k + q) * kKStep, (wt0 + mt) * kRows, bar);
          bulk_g2s(st + lay.sfa_off(mt, 0), a.Sp + ((size_t)(wt0 + mt) * a.nsteps + k) * kAtom,
                   (uint32_t)(nq * kAtom), bar);
        }
      };
      auto issue_x = [&](int s) {
        uint8_t* st = dsm + (size_t)(s % nst) * stage_bytes;
        uint64_t* bar = &full_bar[s % nst];
        const int k = s_begin + s * kb, nq = steps_of(s);
        for (int nt = 0; nt < nt_n; ++nt) {
          for (int q = 0; q < nq; ++q)
            tma_load_2d(st + lay.b_off(nt, q), &xmap, (k + q) * kKStep, (tt0 + nt) * kBRows, bar);
          bulk_g2s(st + lay.sfb_off(nt, 0), a.Xs + ((size_t)(tt0 + nt) * a.nsteps + k) * kAtom,
                   (uint32_t)(nq * kAtom), bar);
        }
      };
      // weights and their scales are load-time data: the first ring's worth
      // streams before this grid waits on the pre-pass that writes the terms
      const int pre = min(nstg, nst);
      for (int s = 0; s < pre; ++s) {
        mbar_arrive_expect_tx(&full_bar[s], tx_of(s));
        issue_w(s);
      }
      griddep_wait();
      for (int s = 0; s < pre; ++s) issue_x(s);
      int issued = pre;
      for (int s = pre; s < nstg; ++s) {
        const int slot = s % nst;
        if (!mbar_wait_bounded(&empty_bar[slot], ((s / nst) - 1) & 1)) break;  // stop issuing
        mbar_arrive_expect_tx(&full_bar[slot], tx_of(s));
        issue_w(s);
        issue_x(s);
        issued = s + 1;
      }
      // drain: every copy issued has landed before the CTA may exit
      for (int t = max(0, issued - nst); t < issued; ++t) mbar_wait_bounded(&full_bar[t % nst], (t / nst) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ---------------------------------------------------
    if (lane == 0 && ns > 0) {
      const uint32_t ring = smem_u32(dsm);
      bool failed = false;
      for (int s = 0; s < nstg; ++s) {
        const int slot = s % nst;
        if (!mbar_wait_bounded(&full_bar[slot], (s / nst) & 1)) {
          failed = true;  // issue nothing more
          break;
        }
        tc::fence_after_sync();
        const int nq = min(kb, ns - s * kb);
        const uint32_t st = ring + (uint32_t)slot * (uint32_t)stage_bytes;
        // scale atoms of this slot: A (mt, q) at column 4 (mt kb + q), B (nt, q) at
        // 4 (MT kb + q NT + nt): the atoms of a step's token tiles side by side,
        // rows 128 nt + r of an N = 256 B operand at column r / 32 + 4 nt
        const uint32_t tsf = tbase + kSfCol + 4 * (MT + NT) * kb * slot;
        auto sfa_col = [&](int mt, int q) { return tsf + 4 * (mt * kb + q); };
        auto sfb_col = [&](int nt, int q) { return tsf + 4 * (MT * kb + q * NT + nt); };
        for (int q = 0; q < nq; ++q) {
          for (int mt = 0; mt < mt_n; ++mt) tmem_cp_atom(sfa_col(mt, q), sdesc_atom(st + lay.sfa_off(mt, q)));
          for (int nt = 0; nt < nt_n; ++nt) tmem_cp_atom(sfb_col(nt, q), sdesc_atom(st + lay.sfb_off(nt, q)));
        }
        // two token tiles: their B boxes are adjacent (256 K-major rows), so one
        // N = 256 MMA takes both -- half the MMAs to issue from this thread
        const bool n256 = NT == 2 && nt_n == 2 && a.n256;
        for (int q = 0; q < nq; ++q) {
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {  // K = 32 each, scale byte kq of the atoms
            const uint32_t sf = (uint32_t)kq;
            const uint32_t acc = (s > 0 || q > 0 || kq > 0) ? 1u : 0u;
            for (int mt = 0; mt < mt_n; ++mt) {
              const uint64_t adesc = tc::sdesc_sw128(st + lay.a_off(mt, q) + 32 * kq, 16, 1024);
              if (n256) {
                mma_mxf8f6f4(tbase + (uint32_t)(mt * NT) * kBRows, adesc,
                             tc::sdesc_sw128(st + lay.b_off(0, q) + 32 * kq, 16, 1024),
                             idesc_mxf8f6f4(kRows, 2 * kBRows, sf), acc, sfa_col(mt, q) | (sf << 30),
                             sfb_col(0, q) | (sf << 30));
              } else {
                for (int nt = 0; nt < nt_n; ++nt)
                  mma_mxf8f6f4(tbase + (uint32_t)(mt * NT + nt) * kBRows, adesc,
                               tc::sdesc_sw128(st + lay.b_off(nt, q) + 32 * kq, 16, 1024),
                               idesc_mxf8f6f4(kRows, kBRows, sf), acc, sfa_col(mt, q) | (sf << 30),
                               sfb_col(nt, q) | (sf << 30));
              }
            }
          }
        }
        tc::commit(&empty_bar[slot]);
      }
      if (!failed) tc::commit(&d_full);
    }
  } else {
    // ---------------- warps 2-5: epilogue ------------------------------------------
    const int et = tid - 64;                 // 0..127
    const int lrow = 32 * (warp & 3) + lane;  // tensor-memory lane of this thread
    bool ok = ns == 0 || mbar_wait_bounded(&d_full, 0);
    ok = __all_sync(0xffffffffu, ok);
    tc::fence_after_sync();
    if (ksz > 1) cluster_wait();  // every peer's recv_bar is initialised
    griddep_wait();               // before any output store
    const uint32_t rbar_local = smem_u32(&recv_bar);
    for (int mt = 0; mt < MT; ++mt) {
      const int r = mt * kRows + lrow;  // row of the CTA tile
      const int n = wt0 * kRows + r;
      const int owner = ksz > 1 ? r / band : 0;
      const int br = r - owner * band;  // row within the owner's band
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {  // tokens 32 h .. 32 h + 31 of token tile nt
          float v[32];
          if (ok && ns > 0 && mt < mt_n && nt < nt_n) {
            float d0[32], d1[32];
            const uint32_t tl = tbase + (uint32_t)(mt * NT + nt) * kBRows + ((uint32_t)(32 * (warp & 3)) << 16);
            tc::ld32_wait(tl + 32 * h, d0);        // term 0
            tc::ld32_wait(tl + kTok + 32 * h, d1);  // term 1
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = d0[j] + d1[j];
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          const int tok0 = nt * kTok + 32 * h;  // first token (within the CTA tile) of v
          if (ksz == 1 && a.vec_out) {
            // into the (drained) ring as a [token][row] bf16 tile, stored below in 16-byte chunks
            __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(dsm);
#pragma unroll
            for (int j = 0; j < 32; ++j) tile[(size_t)(tok0 + j) * (MT * kRows) + r] = __float2bfloat16_rn(v[j]);
          } else if (ksz == 1) {
            const int m0 = tt0 * kTok + tok0;
            if (n < a.N)
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (m0 + j < a.M) a.Out[(size_t)(m0 + j) * a.N + n] = __float2bfloat16_rn(v[j]);
          } else {
            float* rowp = recv + ((size_t)rank * band + br) * kT;
            if (owner == rank) {
#pragma unroll
              for (int c = 0; c < 8; ++c)
                reinterpret_cast<float4*>(rowp)[((tok0 >> 2) + c) ^ (br & 7)] =
                    make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            } else {
              const uint32_t raddr = map_to_rank(smem_u32(rowp), owner);
              const uint32_t rbar = map_to_rank(rbar_local, owner);
#pragma unroll
              for (int c = 0; c < 8; ++c)
                st_async_v4_f32(raddr + 16u * (uint32_t)(((tok0 >> 2) + c) ^ (br & 7)),
                                make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]), rbar);
            }
          }
        }
      }
    }
    tc::fence_before_sync();
    if (ksz == 1 && a.vec_out && a.swiglu) {
      // weight tile w holds gate rows 64 w .. 64 w + 63, then the same up rows:
      // 8 gate and the 8 matching up values of a token give one 16-byte chunk
      // of act[m, 64 w + c] = bf16(bf16(silu(g)) * u), g and u the bf16 products
      named_bar_sync(1, 128);
      const uint4* tile = reinterpret_cast<const uint4*>(dsm);
      constexpr int kCh = MT * kRows / 8;  // 16-byte chunks per token row of the tile
      constexpr int kChS = kCh / 2;        // output chunks per token row
      const int half = a.N / 2;
      for (int idx = et; idx < kT * kChS; idx += 128) {
        const int tok = idx / kChS, c = idx % kChS;
        const int mt = c / 8, j = c % 8;
        const int m = tt0 * kTok + tok, wt = wt0 + mt;
        if (m < a.M && wt * kRows < a.N) {  // N % 128 == 0: a weight tile lies wholly inside or outside
          const uint4 g4 = tile[(size_t)tok * kCh + mt * 16 + j], u4 = tile[(size_t)tok * kCh + mt * 16 + 8 + j];
          const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&g4);
          const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&u4);
          uint4 o4;
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&o4);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float gv = __bfloat162float(g[e]);
            const float sv = silu_bf16(gv);
            o[e] = __float2bfloat16_rn(sv * __bfloat162float(u[e]));
          }
          *reinterpret_cast<uint4*>(a.Out + (size_t)m * half + (size_t)wt * 64 + 8 * j) = o4;
        }
      }
    } else if (ksz == 1 && a.vec_out) {
      // the tile's token rows are contiguous runs of output: coalesced 16-byte stores
      named_bar_sync(1, 128);
      const uint4* tile = reinterpret_cast<const uint4*>(dsm);
      constexpr int kCh = MT * kRows / 8;  // 16-byte chunks per token row of the tile
      for (int idx = et; idx < kT * kCh; idx += 128) {
        const int tok = idx / kCh, c = idx % kCh;
        const int m = tt0 * kTok + tok, n0 = wt0 * kRows + 8 * c;
        if (m < a.M && n0 < a.N)  // N % 8 == 0: a chunk lies wholly inside or outside
          *reinterpret_cast<uint4*>(a.Out + (size_t)m * a.N + n0) = tile[idx];
      }
    }
    if (ksz > 1) {
      // finish this rank's band: fixed-order sum over the ranks' partials
      named_bar_sync(1, 128);  // the local partial is in place
      if (my_rows > 0 && (recv_bytes == 0 || mbar_wait_bounded(&recv_bar, 0))) {
        for (int it = et; it < my_rows * (kT / 4); it += 128) {
          const int br = it % my_rows, c = it / my_rows;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q = 0; q < ksz; ++q) {
            const float4 x = reinterpret_cast<const float4*>(recv + ((size_t)q * band + br) * kT)[c ^ (br & 7)];
            acc.x += x.x;
            acc.y += x.y;
            acc.z += x.z;
            acc.w += x.w;
          }
          const int n = wt0 * kRows + rank * band + br;
          const int m0 = tt0 * kTok + 4 * c;
          if (n < a.N && n < (wt0 + mt_n) * kRows) {
            const float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (m0 + e < a.M) a.Out[(size_t)(m0 + e) * a.N + n] = __float2bfloat16_rn(o[e]);
          }
        }
      }
    }
  }

  griddep_wait();  // every thread waits before exit
  tc::fence_before_sync();
  __syncthreads();  // all tensor-memory reads are done
  if (warp == 0) tc::tmem_dealloc(tbase, kTmemCols);
}

template <int MT, int NT>
cudaError_t raise_smem_limit(size_t smem) {
  static std::mutex mu;
  static size_t limit = 0;
  std::lock_guard<std::mutex> g(mu);
  if (smem <= limit) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(mxfp4_gemm_kernel<MT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) limit = smem;
  return e;
}

// clusters of ks CTAs with `smem` bytes each that the device holds at once
template <int MT, int NT>
int max_active_clusters(int ks, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, ks, smem);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (raise_smem_limit<MT, NT>(smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, mxfp4_gemm_kernel<MT, NT>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

struct Plan {
  int mt = 0, nt = 0, ks = 0, nst = 0, kb = 1;
  size_t smem = 0;
};

template <int MT, int NT>
void consider(Plan& best, double& best_cost, const GemmArgs& a, int sms, int force_ks, int force_st,
              int force_kb) {
  const int tiles = cdiv(a.wtiles, MT) * cdiv(a.ttiles, NT);
  for (int ks = 1; ks <= 8 && ks <= a.nsteps; ++ks)
  for (int kb = 1; kb <= 2; ++kb) {
    if (force_ks && ks != force_ks) continue;
    if (force_kb && kb != force_kb) continue;
    const int sps = cdiv(a.nsteps, ks);
    const int stages = cdiv(sps, kb);
    const GemmLayout<MT, NT> l0{0, ks, kb};
    const size_t fixed = l0.bytes();
    const int fit = (int)((kSmemMax - (long)fixed) / l0.stage());
    int nst = min(kMaxStages, min(stages, fit));
    if (force_st) nst = min(nst, force_st);
    if (nst < 1) continue;
    const size_t smem = GemmLayout<MT, NT>{nst, ks, kb}.bytes();
    const int resident = max_active_clusters<MT, NT>(ks, smem);
    if (resident <= 0) continue;
    const int waves = cdiv(tiles, resident);
    const int active = min(tiles, resident) * ks;
    // per stage: weight bytes at this CTA's share of the HBM bandwidth
    // (about 360 cycles per 8 KB when every SM streams), or the MMAs
    // (4 x 64 cycles per 128 x 128 x 128 block), whichever is longer
    // or the single issuing thread: about 70 cycles per MMA, 53 per scale-atom
    // copy and 250 per mbarrier wait (two token tiles go in one N = 256 MMA).
    // With one token tile (M <= 64) a flat 700 cycles fits the measurements better.
    const double fill = min(1.0, (double)active / sms);
    const int mmas = kb * 4 * MT * ((NT == 2 && a.n256) ? 1 : NT);
    const double issue = a.ttiles > 1 ? mmas * 70.0 + kb * (MT + NT) * 53.0 + 250.0 : 700.0;
    double stage_cost = fmax(fmax(kb * MT * 360.0 * fill, kb * MT * NT * 256.0), issue);
    if (nst < 2 && stages > 1) stage_cost *= 2.0;  // a one-stage ring does not overlap loads and MMAs
    const double cost = waves * (stages * stage_cost + 800.0) + (ks > 1 ? 150.0 * ks * MT * NT : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best.mt = MT;
      best.nt = NT;
      best.ks = ks;
      best.nst = nst;
      best.kb = kb;
      best.smem = smem;
    }
  }
}

template <int MT, int NT>
cudaError_t launch_gemm(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& a, const Plan& p,
                        cudaStream_t st) {
  const cudaError_t e = raise_smem_limit<MT, NT>(p.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ks, cdiv(a.wtiles, MT), cdiv(a.ttiles, NT));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = p.ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, mxfp4_gemm_kernel<MT, NT>, wm, xm, a);
}

cudaError_t launch_split(const __nv_bfloat16* X, int64_t x_ld, uint8_t* Xq, uint8_t* Xs, int M, int K,
                         int ttiles, int sms, cudaStream_t st) {
  const int64_t total = (int64_t)ttiles * kTok * (K >> 5);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, xsplit_e4m3_kernel, X, x_ld, Xq, Xs, M, K, ttiles);
}

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

}  // namespace

size_t mxfp4_gemm_wide_workspace_bytes(int M, int K) {
  if (M <= 0 || K <= 0 || K % kKStep) return 0;
  const size_t tt = (size_t)cdiv(M, kTok);
  return tt * kBRows * (size_t)K + tt * (size_t)(K / kKStep) * kAtom;
}

int mxfp4_gemm_wide_launch(const void* W, const void* Sp, const void* X, int64_t x_ld, void* ws,
                           size_t ws_bytes, void* Out, int N, int K, int M, int epilogue, void* stream) {
  if (!W || !Sp || !X || !Out) return B200KV_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || M <= 0 || x_ld < K) return B200KV_ERR_INVALID_ARG;
  if (epilogue != 0 && epilogue != 1) return B200KV_ERR_INVALID_ARG;
  if (K % kKStep || (epilogue == 1 && N % kRows)) return B200KV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(Sp) & 15) ||
      (reinterpret_cast<uintptr_t>(X) & 15) || (x_ld & 7) || (reinterpret_cast<uintptr_t>(ws) & 127) ||
      (epilogue == 1 && (reinterpret_cast<uintptr_t>(Out) & 15)))
    return B200KV_ERR_MISALIGNED;
  const size_t need = mxfp4_gemm_wide_workspace_bytes(M, K);
  if (!ws || ws_bytes < need) return B200KV_ERR_WORKSPACE;
  const int sms = num_sms_current_device();
  if (sms <= 0 || sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;

  GemmArgs a;
  a.N = N;
  a.K = K;
  a.M = M;
  a.nsteps = K / kKStep;
  a.wtiles = cdiv(N, kRows);
  a.ttiles = cdiv(M, kTok);
  uint8_t* Xq = static_cast<uint8_t*>(ws);
  uint8_t* Xs = Xq + (size_t)a.ttiles * kBRows * K;
  a.Sp = static_cast<const uint8_t*>(Sp);
  a.Xs = Xs;
  a.Out = static_cast<__nv_bfloat16*>(Out);
  a.n256 = env_int("B200KV_GEMM_N256", 1) != 0;
  a.vec_out = (reinterpret_cast<uintptr_t>(Out) & 15) == 0 && N % 8 == 0;
  a.swiglu = epilogue;

  // plan: tile shape (MT weight tiles x NT token tiles), K-split, ring depth;
  // the SwiGLU epilogue pairs rows of one CTA tile, so it takes K unsplit
  const int force_mt = env_int("B200KV_GEMM_MT", 0), force_nt = env_int("B200KV_GEMM_NT", 0);
  const int force_ks = epilogue == 1 ? 1 : env_int("B200KV_GEMM_KSPLIT", 0);
  const int force_st = env_int("B200KV_GEMM_STAGES", 0);
  const int force_kb = env_int("B200KV_GEMM_KB", 0);
  Plan p;
  double cost = 1e30;
  auto want = [&](int mt, int nt) {
    return (!force_mt || force_mt == mt) && (!force_nt || force_nt == nt);
  };
  if (want(1, 1)) consider<1, 1>(p, cost, a, sms, force_ks, force_st, force_kb);
  if ((a.wtiles > 1 || force_mt == 2) && want(2, 1)) consider<2, 1>(p, cost, a, sms, force_ks, force_st, force_kb);
  if ((a.ttiles > 1 || force_nt == 2) && want(1, 2)) consider<1, 2>(p, cost, a, sms, force_ks, force_st, force_kb);
  if (p.ks == 0) return B200KV_ERR_UNSUPPORTED;
  a.sps = cdiv(a.nsteps, p.ks);
  a.nstages = p.nst;
  a.kb = p.kb;
  if (env_int("B200KV_GEMM_PLAN", 0))
    fprintf(stderr, "[b200kv] mxfp4_gemm_wide N=%d K=%d M=%d: MT=%d NT=%d ks=%d kb=%d stages=%d smem=%zu\n", N,
            K, M, p.mt, p.nt, p.ks, p.kb, p.nst, p.smem);

  CUtensorMap wm, xm;
  if (!encode_e2m1_unpacked_2d(&wm, W, (uint64_t)K, (uint64_t)N, (uint64_t)(K / 2), kRows) ||
      !encode_u8_2d(&xm, Xq, (uint64_t)K, (uint64_t)a.ttiles * kBRows, (uint64_t)K, 128, kBRows, true))
    return B200KV_ERR_UNSUPPORTED;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_split(static_cast<const __nv_bfloat16*>(X), x_ld, Xq, Xs, M, K, a.ttiles, sms, st);
  if (e == cudaSuccess) {
    if (p.mt == 1 && p.nt == 1)
      e = launch_gemm<1, 1>(wm, xm, a, p, st);
    else if (p.mt == 2)
      e = launch_gemm<2, 1>(wm, xm, a, p, st);
    else
      e = launch_gemm<1, 2>(wm, xm, a, p, st);
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

// ---- allocation-free variant ------------------------------------------------------
// Callers that cannot allocate device memory (an engine that has already handed
// all free HBM to its KV-cache pool, or a host that binds this C ABI with no
// device allocator of its own) get the same GEMM with its activation-term
// scratch in a fixed array of this library: up to kNoAllocMaxM activation rows
// of K <= kNoAllocMaxK (4.3 MB, held on every GPU that loads the library).
constexpr int kNoAllocMaxM = 2 * kTok;
constexpr int kNoAllocMaxK = 16384;
constexpr size_t kNoAllocBytes =
    (size_t)(kNoAllocMaxM / kTok) * kBRows * kNoAllocMaxK + (size_t)(kNoAllocMaxM / kTok) * (kNoAllocMaxK / kKStep) * kAtom;
static __device__ __align__(256) uint8_t g_wide_scratch[kNoAllocBytes];

namespace {
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
// device address of g_wide_scratch per device ordinal, and the context it was
// looked up in: a device reset (or a primary context torn down and made again)
// reloads the module, so the address is looked up again when the context changes
void* g_scratch_ptr[kMaxScratchDevices];
CUcontext g_scratch_ctx[kMaxScratchDevices];

CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    else
      cudaGetLastError();
  });
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}
}  // namespace

int mxfp4_gemm_wide_noalloc_launch(const void* W, const void* Sp, const void* X, int64_t x_ld, void* Out, int N,
                                   int K, int M, void* stream) {
  // argument errors first, in the workspace entry point's order, then the scratch limit
  if (!W || !Sp || !X || !Out) return B200KV_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || M <= 0 || x_ld < K) return B200KV_ERR_INVALID_ARG;
  if (K % kKStep) return B200KV_ERR_UNSUPPORTED;
  if (M > kNoAllocMaxM || K > kNoAllocMaxK) return B200KV_ERR_WORKSPACE;
  if (mxfp4_gemm_wide_workspace_bytes(M, K) > kNoAllocBytes) return B200KV_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxScratchDevices) {
    cudaGetLastError();
    return B200KV_ERR_NO_DEVICE;
  }
  void* ptr = nullptr;
  {
    // set-up, once per device (and context), with that device current: the
    // array's device address
    std::lock_guard<std::mutex> g(g_scratch_mu);
    const CUcontext ctx = current_context();
    if (!g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_wide_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return B200KV_ERR_NO_DEVICE;
      }
      g_scratch_ptr[dev] = p;
      g_scratch_ctx[dev] = ctx;
    }
    ptr = g_scratch_ptr[dev];
  }
  // the pre-pass rewrites every byte the GEMM reads: nothing needs clearing
  return mxfp4_gemm_wide_launch(W, Sp, X, x_ld, ptr, kNoAllocBytes, Out, N, K, M, 0, stream);
}

}  // namespace b200kv
