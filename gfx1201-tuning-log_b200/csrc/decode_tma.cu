// fp8-e4m3 paged-KV split-K decode attention with TMA page loads (sm_100a).
//
// Same contract as decode_attn.cu (the reference's split-KV flash decode,
// vllm-fp8kv/fp8kv_v3.py:4-113, and its single-pass predecessor
// vllm-fp8kv/fp8kv_kernel.py:4-72); this is the path for fp8 caches whose
// pages can be described by a tensor map (block_size 16/32/64/128, 16-byte
// strides, the pool's block count known).
//
// Why a second kernel.  The row-per-thread cp.async gather of decode_attn.cu
// makes every warp instruction touch 32 different cache lines, and its V
// operand goes through a separate fp8 -> f16 pass in shared memory; at batch 1
// those two steps were over half of a launch (timed per phase with
// %globaltimer).  Here:
//  * one producer warp issues one TMA load per (page, K or V): a page of one kv
//    head (block_size rows of 128 bytes) lands as a 128-byte-swizzled tile, so
//    the fragment reads below are bank-conflict free without padding;
//  * before waiting on the previous kernel (programmatic dependent launch) the
//    producer reads the block table and prefetches the first pages into L2;
//  * the V^T operand of O^T += V^T P^T is built in registers: ldmatrix.trans
//    over the fp8 rows viewed as 16-bit pairs gives each thread two tokens x
//    two dims, one byte permute and two exact fp8x2 -> f16x2 converts turn that
//    into the A fragments of two MMAs (dims 2g and 2g+1 of a 16-dim group sit
//    in MMA rows g and g+8; the output mapping follows);
//  * S^T = q K^T, the per-warp online softmax in the log2 domain, the cluster
//    merge through distributed shared memory and the numerics (q pre-scaled to
//    f16 by an exact power of two per head, P rounded to f16, fp32
//    accumulation) are those of decode_attn.cu.
// One CTA = CW compute warps (ST / CW tokens of each stage apiece) + the
// producer warp; 3 stages of (K, V) pages of ST tokens each.  Ring shapes:
// ST = 128 with 4 or 8 compute warps (96 KB in flight per CTA) and ST = 64
// with 4 (48 KB), whose CTA fits in the shared memory an MXFP4 GEMV CTA
// leaves free, so that under programmatic dependent launch it becomes
// resident while the GEMV that produces q still runs: its block-table reads
// and the L2 prefetch of its pages then overlap that GEMV, and the next
// GEMV's CTAs fit beside it in turn.  The launcher picks the shape from the
// grid and the share of each CTA.

#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "tma.cuh"
#include "warp_mma.cuh"

namespace cg = cooperative_groups;

namespace b200kv {

namespace {

constexpr int kHD = 128;           // head_dim (bytes per fp8 row)
constexpr int kMaxStages = 4;
constexpr int kMaxCWarps = 8;      // compute warps: 4 or 8 (+ the producer warp)
constexpr int kMaxCS = 16;         // cluster size bound
constexpr float kLog2eT = 1.4426950408889634f;

// ring of NS stages of ST tokens (K and V pages of one kv head), CW compute warps
template <int ST, int NS, int CW>
struct Ring {
  static_assert(ST == 64 || ST == 128, "stage tokens");
  static_assert(NS >= 2 && NS <= kMaxStages, "stages");
  static_assert((CW == 4 || CW == 8) && ST / CW >= 16, "compute warps");
  static constexpr int kThreads = (CW + 1) * 32;
  static constexpr int kStageTok = ST;
  static constexpr int kStages = NS;
  static constexpr int kTPW = ST / CW;             // tokens of a stage per compute warp
  static constexpr int kHalfStage = ST * kHD;      // K (or V) bytes of one stage
  static constexpr int kStageBytes = 2 * kHalfStage;
  static constexpr int kDynSmem = NS * kStageBytes + 1024;  // + alignment slack
};

struct TmaDecodeParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  const int32_t* qsl;
  const int32_t* seq_lens;
  const int32_t* bt;
  int64_t bt_stride;
  const float* k_scale;
  const float* v_scale;
  float sm_scale;
  int bs_shift;  // log2(block_size), block_size in {16, 32, 64, 128}
  int out_by_qsl;  // bit 0: output row qsl[s] (else s); bit 1: one-token sequences only
};

template <int GQA>
struct TmaShared {
  alignas(16) float part_o[GQA][kHD];  // this CTA's unnormalised o (read by peers)
  float wm[kMaxCWarps][8], wl[kMaxCWarps][8];
  float part_m[8], part_l[8];
  alignas(16) float inbox_o[GQA * kHD];     // [source rank][the elements this rank finishes]
  float inbox_ml[kMaxCS][2][8];             // every rank's (m, l) per head
  float rw[kMaxCS][8];                      // every rank's weight in the output
  uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], inbox_bar;
};

// byte offset of (row, byte b) in a 128-byte-swizzled tile (1024-byte aligned)
__device__ __forceinline__ uint32_t swz(int row, int b) {
  return (uint32_t)(row * 128 + ((((b >> 4) ^ row) & 7) << 4) + (b & 15));
}

template <int GQA, int ST, int NS, int CW>
__global__ void __launch_bounds__((CW + 1) * 32)
    decode_tma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const TmaDecodeParams p) {
  using RG = Ring<ST, NS, CW>;
  constexpr int kCWarps = CW, kThreadsT = RG::kThreads;
  constexpr int kStageTok = RG::kStageTok, kStages = RG::kStages, kTPW = RG::kTPW;
  constexpr int kHalfStage = RG::kHalfStage, kStageBytes = RG::kStageBytes;
  constexpr int kNT8 = kTPW / 8;    // 8-token MMA tiles of S^T per warp and stage
  constexpr int kNJ = kTPW / 16;    // 16-token slices of P^T per warp and stage
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ TmaShared<GQA> S;

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int kh = blockIdx.y;
  const int seq = blockIdx.z;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int g = lane >> 2;
  const int c = lane & 3;

  // Mixed batches: a sequence with more than one query token is the varlen
  // prefill kernel's (every CTA of the cluster serves this sequence, so the
  // whole cluster leaves, before any barrier or cluster arrival).
  if ((p.out_by_qsl & 2) && p.qsl[seq + 1] - p.qsl[seq] != 1) {
    griddep_wait();
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.full_bar[s], 1);
      mbar_init(&S.empty_bar[s], kCWarps);
    }
    mbar_init(&S.inbox_bar, 1);
    fence_mbar_init();
    if (csize > 1)  // the peers' pushes: their o elements of this rank plus their (m, l)
      mbar_arrive_expect_tx(&S.inbox_bar, (uint32_t)((csize - 1) * (GQA * kHD / csize + 2 * GQA) * 4));
    // The next kernel may launch now.  Sequence metadata and block-table rows
    // are read, and pages prefetched into L2, before this grid waits on the
    // previous one; q, the shared-memory loads of K and V and the output come
    // after griddep_wait().
    griddep_launch_dependents();
  }
  const int seqlen = max(p.seq_lens[seq], 0);
  const int q_tok = p.qsl[seq];
  const int out_row = (p.out_by_qsl & 1) ? q_tok : seq;
  const int bs = 1 << p.bs_shift;
  const int unit = max(bs, 16);  // shares start on a page boundary
  const int per = ((seqlen + csize - 1) / csize + unit - 1) / unit * unit;
  const int lo = min(seqlen, rank * per);
  const int hi = min(seqlen, lo + per);
  const int nchunks = (hi - lo + kStageTok - 1) / kStageTok;
  __syncthreads();  // barrier init visible
  if (csize > 1) cluster_arrive_relaxed();  // the inbox barrier is initialised

  float m_run = -INFINITY, l_run = 0.f;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;

  if (warp == kCWarps) {
    // ---------------- producer: one TMA load per (page, K or V) ----------------
    const int32_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;
    const int ppc = kStageTok >> p.bs_shift;           // pages per stage (divides 32)
    const int p0 = lo >> p.bs_shift;                   // first page of this share
    const int npages = (hi - lo + bs - 1) >> p.bs_shift;
    auto entry = [&](int q) { return q < npages ? bt_row[p0 + q] : 0; };
    int win = 0;  // lanes hold the entries of pages 32*win + lane (and the next window)
    int e_cur = entry(lane), e_nxt = entry(32 + lane);
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    if (lane < npages) {  // every page of the first window (all of a short share)
      tma_prefetch_l2_4d(&kmap, 0, kh, 0, e_cur);
      tma_prefetch_l2_4d(&vmap, 0, kh, 0, e_cur);
    }
    griddep_wait();
    int ch = 0;
    for (; ch < nchunks; ++ch) {
      const int s = ch % kStages;
      int ok = 1;
      if (lane == 0 && ch >= kStages) ok = mbar_wait_bounded(&S.empty_bar[s], ((ch / kStages) - 1) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;  // stop issuing; drain below
      const int q0 = ch * ppc;
      if ((q0 >> 5) != win) {  // a stage never straddles two windows
        ++win;
        e_cur = e_nxt;
        e_nxt = entry(32 * (win + 1) + lane);
      }
      const int npc = min(ppc, npages - q0);
      if (lane == 0) mbar_arrive_expect_tx(&S.full_bar[s], (uint32_t)(npc * bs * kHD * 2));
      __syncwarp();
      const int j = lane - (q0 & 31);
      if (j >= 0 && j < npc) {
        uint8_t* kd = smem + (size_t)s * kStageBytes + (size_t)j * bs * kHD;
        tma_load_4d(kd, &kmap, 0, kh, 0, e_cur, &S.full_bar[s]);
        tma_load_4d(kd + kHalfStage, &vmap, 0, kh, 0, e_cur, &S.full_bar[s]);
      }
    }
    // every load issued has landed before the stages are reused or the CTA exits
    if (lane == 0)
      for (int t = max(0, ch - kStages); t < ch; ++t)
        mbar_wait_bounded(&S.full_bar[t % kStages], (t / kStages) & 1);
    __syncwarp();
  } else {
    // ---------------- compute warps -------------------------------------------------
    griddep_wait();  // q is the previous kernel's output
    uint32_t qa[8][2];
    float score_scale;
    {
      const int h = g < GQA ? g : 0;
      const __nv_bfloat16* qb = p.q + (int64_t)q_tok * p.q_st + (int64_t)(kh * GQA + h) * p.q_sh;
      float qv[8][4];
#pragma unroll
      for (int ds = 0; ds < 8; ++ds) {
        const uint2 raw = *reinterpret_cast<const uint2*>(qb + 16 * ds + 4 * c);
        qv[ds][0] = __uint_as_float(raw.x << 16);
        qv[ds][1] = __uint_as_float(raw.x & 0xFFFF0000u);
        qv[ds][2] = __uint_as_float(raw.y << 16);
        qv[ds][3] = __uint_as_float(raw.y & 0xFFFF0000u);
      }
      float mx = 0.f;
#pragma unroll
      for (int ds = 0; ds < 8; ++ds)
#pragma unroll
        for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fabsf(qv[ds][e]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);
      int sh = (E == 0xFF || mx == 0.f) ? 0 : 131 - E;  // head max * 2^sh in [2^4, 2^5)
      sh = max(-126, min(127, sh));
      const float up = __uint_as_float((uint32_t)(sh + 127) << 23);
      score_scale = p.sm_scale * __ldg(p.k_scale) * kLog2eT * __uint_as_float((uint32_t)(127 - sh) << 23);
#pragma unroll
      for (int ds = 0; ds < 8; ++ds) {
        qa[ds][0] = g < GQA ? pack_f16x2(qv[ds][0] * up, qv[ds][1] * up) : 0u;
        qa[ds][1] = g < GQA ? pack_f16x2(qv[ds][2] * up, qv[ds][3] * up) : 0u;
      }
    }

    for (int ch = 0; ch < nchunks; ++ch) {
      const int s = ch % kStages;
      if (!mbar_wait_bounded(&S.full_bar[s], (ch / kStages) & 1)) break;
      uint8_t* kst = smem + (size_t)s * kStageBytes;
      uint8_t* vst = kst + kHalfStage;
      const int nt = min(kStageTok, hi - (lo + ch * kStageTok));
      const int w0 = warp * kTPW;
      const int ntw = max(0, min(kTPW, nt - w0));
      if (ntw > 0) {
        if (ntw < kTPW) {
          // rows past the share hold other tokens or stale bytes (possibly NaN
          // codes): zero this warp's V rows there so that 0 * V stays 0
          for (int i = lane; i < (kTPW - ntw) * 8; i += 32)
            *reinterpret_cast<uint4*>(vst + (w0 + ntw + (i >> 3)) * kHD + (i & 7) * 16) = make_uint4(0, 0, 0, 0);
          __syncwarp();
        }
        // ---- S^T = q K^T over the warp's token tiles of 8 --------------------------
        float sfr[kNT8][4];
#pragma unroll
        for (int t = 0; t < kNT8; ++t) {
#pragma unroll
          for (int e = 0; e < 4; ++e) sfr[t][e] = 0.f;
          const int row = w0 + 8 * t + g;
#pragma unroll
          for (int ds = 0; ds < 8; ++ds) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(kst + swz(row, 16 * ds + 4 * c));
            mma16816<true>(sfr[t], qa[ds][0], 0u, qa[ds][1], 0u, e4m3x2_to_f16x2(w & 0xFFFFu),
                           e4m3x2_to_f16x2(w >> 16));
          }
        }
        // ---- online softmax for head g over this warp's tokens --------------------
        float mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < kNT8; ++t)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tok = 8 * t + 2 * c + e;
            const float v = tok < ntw ? sfr[t][e] * score_scale : -INFINITY;
            sfr[t][e] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);  // finite: ntw >= 1
        const float alpha = exp2f(m_run - m_new);
        m_run = m_new;
        float psum = 0.f;
        uint32_t pb[kNT8];
#pragma unroll
        for (int t = 0; t < kNT8; ++t) {
          const float p0 = exp2f(sfr[t][0] - m_new);
          const float p1 = exp2f(sfr[t][1] - m_new);
          psum += p0 + p1;
          pb[t] = pack_f16x2(p0, p1);
        }
        l_run = l_run * alpha + psum;
        const float a0 = __shfl_sync(0xffffffffu, alpha, (2 * c) * 4);
        const float a1 = __shfl_sync(0xffffffffu, alpha, (2 * c + 1) * 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i][0] *= a0; o[i][1] *= a1; o[i][2] *= a0; o[i][3] *= a1;
        }
        // ---- O^T += V^T P^T: token slices of 16 x 4 dim groups of 32 --------------
        // ldmatrix.trans over rows viewed as 16-bit pairs: matrix m (lanes 8m..8m+7
        // give its rows) = tokens 8*(m&1).., dims 16*(m>>1).. of the group; thread
        // (g, c) gets bytes {V[2c][2g], V[2c][2g+1], V[2c+1][2g], V[2c+1][2g+1]}.
#pragma unroll
        for (int j = 0; j < kNJ; ++j) {
          const int vrow = w0 + 16 * j + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            uint32_t m[4];
            ldsm_x4_trans(m, vst + swz(vrow, 32 * i2 + (lane >> 4) * 16));
            uint32_t f[8];  // (dim 2g, dim 2g+1) token pairs of matrices 0..3
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t x = __byte_perm(m[q], 0u, 0x3120);  // [V0d, V1d | V0d', V1d']
              f[2 * q] = e4m3x2_to_f16x2(x & 0xFFFFu);
              f[2 * q + 1] = e4m3x2_to_f16x2(x >> 16);
            }
            // MMA rows g / g+8 = dims 2g / 2g+1 of the 16-dim group
            mma16816<true>(o[2 * i2], f[0], f[1], f[2], f[3], pb[2 * j], pb[2 * j + 1]);
            mma16816<true>(o[2 * i2 + 1], f[4], f[5], f[6], f[7], pb[2 * j], pb[2 * j + 1]);
          }
        }
      }
      __syncwarp();
      if (ntw > 0 && ntw < kTPW)  // generic writes before any later TMA write of the stage
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (lane == 0) mbar_arrive(&S.empty_bar[s]);
    }
  }

  // ---- merge the 4 compute warps: per-warp state -> this CTA's partial ------------
  if (warp < kCWarps) {
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (c == 0) {
      S.wm[warp][g] = m_run;
      S.wl[warp][g] = l_run;
    }
  }
  __syncthreads();  // the stages are free from here on (all loads have landed)
  float (*wo)[GQA][kHD] = reinterpret_cast<float (*)[GQA][kHD]>(smem);
  if (warp < kCWarps) {
    float wgt[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int h = (2 * c + e) & 7;
      float mc = -INFINITY;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) mc = fmaxf(mc, S.wm[w][h]);
      const float mw = S.wm[warp][h];
      wgt[e] = (mw == -INFINITY) ? 0.f : exp2f(mw - mc);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int h = 2 * c + e;
        if (h < GQA) {
          wo[warp][h][16 * i + 2 * g] = o[i][e] * wgt[e];
          wo[warp][h][16 * i + 2 * g + 1] = o[i][2 + e] * wgt[e];
        }
      }
  }
  __syncthreads();
  for (int e = tid; e < GQA * kHD; e += kThreadsT) {
    const int h = e / kHD, d = e % kHD;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kCWarps; ++w) s += wo[w][h][d];
    S.part_o[h][d] = s;
  }
  if (tid < GQA) {
    float mc = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCWarps; ++w) mc = fmaxf(mc, S.wm[w][tid]);
    float lc = 0.f;
    if (mc != -INFINITY)
#pragma unroll
      for (int w = 0; w < kCWarps; ++w)
        if (S.wm[w][tid] != -INFINITY) lc += S.wl[w][tid] * exp2f(S.wm[w][tid] - mc);
    S.part_m[tid] = mc;
    S.part_l[tid] = lc;
  }
  // ---- merge the cluster's partials: push, then reduce locally ----------------------
  // Rank r finishes elements [r per_cta, (r + 1) per_cta) of the (head, dim)
  // block.  Every rank pushes its (m, l) of every head and its o of those
  // elements into rank r's inbox (st.async, counted on r's inbox barrier), so the
  // merge costs one one-way trip and no rank waits on a cluster barrier.
  constexpr int E = GQA * kHD;
  const int per_cta = E / csize, e0 = rank * per_cta;
  __syncthreads();  // part_o, part_m, part_l complete
  if (csize > 1) cluster_wait();
  const uint32_t bar_local = smem_u32(&S.inbox_bar);
  for (int it = tid; it < E + csize * 2 * GQA; it += kThreadsT) {
    int r;
    float v;
    float* dst;
    if (it < E) {
      r = it / per_cta;
      v = (&S.part_o[0][0])[it];
      dst = &S.inbox_o[rank * per_cta + (it - r * per_cta)];
    } else {
      const int j = it - E, k = j % (2 * GQA);
      r = j / (2 * GQA);
      v = k < GQA ? S.part_m[k] : S.part_l[k - GQA];
      dst = &S.inbox_ml[rank][k / GQA][k % GQA];
    }
    if (r == rank)
      *dst = v;
    else
      st_async_f32(map_to_rank(smem_u32(dst), r), v, map_to_rank(bar_local, r));
  }
  if (csize > 1) mbar_wait_bounded(&S.inbox_bar, 0);
  __syncthreads();  // this rank's own inbox entries are visible too

  griddep_wait();  // every thread, before the output store (and before exit)
  const float vsc = __ldg(p.v_scale);
  __nv_bfloat16* out_base = p.out + (int64_t)out_row * p.o_st + (int64_t)(kh * GQA) * p.o_sh;
  if (tid < GQA) {
    float mg = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxCS; ++r)
      if (r < csize) mg = fmaxf(mg, S.inbox_ml[r][0][tid]);
    float wr[kMaxCS];
    float lg = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxCS; ++r) {
      const float mr = r < csize ? S.inbox_ml[r][0][tid] : -INFINITY;
      wr[r] = (mr == -INFINITY) ? 0.f : exp2f(mr - mg);
      if (r < csize) lg += wr[r] * S.inbox_ml[r][1][tid];
    }
    const float inv = lg > 0.f ? vsc / lg : 0.f;
#pragma unroll
    for (int r = 0; r < kMaxCS; ++r)
      if (r < csize) S.rw[r][tid] = wr[r] * inv;
  }
  __syncthreads();
  for (int i = tid; i < per_cta; i += kThreadsT) {
    const int e = e0 + i, h = e / kHD, d = e % kHD;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxCS; ++r)  // the products rounded before the sum, as the gather path
      if (r < csize) acc = __fadd_rn(acc, __fmul_rn(S.rw[r][h], S.inbox_o[r * per_cta + i]));
    out_base[(int64_t)h * p.o_sh + d] = __float2bfloat16_rn(acc);
  }
}

template <int GQA, int ST, int NS, int CW>
cudaError_t launch_tma(const CUtensorMap& km, const CUtensorMap& vm, const TmaDecodeParams& p,
                       int csize, int hkv, int num_seqs, cudaStream_t stream) {
  using RG = Ring<ST, NS, CW>;
  static_assert(NS * RG::kStageBytes >= CW * GQA * kHD * 4, "stages must hold the merge");
  auto kern = decode_tma_kernel<GQA, ST, NS, CW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, RG::kDynSmem);
  if (e != cudaSuccess) return e;
  if (csize > 8) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(csize, hkv, num_seqs);
  lc.blockDim = dim3(RG::kThreads, 1, 1);
  lc.dynamicSmemBytes = RG::kDynSmem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&lc, kern, km, vm, p);
}

// Ring shapes (tokens per stage, compute warps): 0 = (128, 4), 1 = (128, 8), 2 = (64, 4).
template <int GQA>
cudaError_t launch_ring(int ring, const CUtensorMap& km, const CUtensorMap& vm, const TmaDecodeParams& p,
                        int csize, int hkv, int num_seqs, cudaStream_t stream) {
  if (ring == 2) return launch_tma<GQA, 64, 3, 4>(km, vm, p, csize, hkv, num_seqs, stream);
  if (ring == 1) return launch_tma<GQA, 128, 3, 8>(km, vm, p, csize, hkv, num_seqs, stream);
  return launch_tma<GQA, 128, 3, 4>(km, vm, p, csize, hkv, num_seqs, stream);
}

}  // namespace

// Returns B200KV_ERR_UNSUPPORTED (nothing launched) when the cache cannot be
// described by tensor maps; the caller then takes the cp.async kernel.
int decode_tma_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                      const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                      int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                      const int32_t* qsl, const int32_t* seq_lens, const int32_t* bt,
                      int64_t bt_stride, const float* k_scale, const float* v_scale,
                      float sm_scale, int num_seqs, int hkv, int gqa, int block_size,
                      int num_blocks, int out_by_qsl, int csize, int ctx_bound, void* stream) {
  if (block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128)
    return B200KV_ERR_UNSUPPORTED;
  if (num_blocks <= 0 || csize < 1 || csize > kMaxCS) return B200KV_ERR_UNSUPPORTED;
  const char* env = getenv("B200KV_DECODE_TMA");
  if (env && env[0] == '0') return B200KV_ERR_UNSUPPORTED;
  CUtensorMap km, vm;
  if (!encode_paged_kv(&km, k_cache, kHD, (uint32_t)hkv, (uint32_t)block_size, (uint64_t)num_blocks,
                       (uint64_t)sk2, (uint64_t)sk1, (uint64_t)sk0) ||
      !encode_paged_kv(&vm, v_cache, kHD, (uint32_t)hkv, (uint32_t)block_size, (uint64_t)num_blocks,
                       (uint64_t)sv2, (uint64_t)sv1, (uint64_t)sv0))
    return B200KV_ERR_UNSUPPORTED;
  TmaDecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_st;
  p.q_sh = q_sh;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_st = o_st;
  p.o_sh = o_sh;
  p.qsl = qsl;
  p.seq_lens = seq_lens;
  p.bt = bt;
  p.bt_stride = bt_stride;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.sm_scale = sm_scale;
  p.bs_shift = __builtin_ctz((unsigned)block_size);
  p.out_by_qsl = out_by_qsl;
  // Ring shape, from the grid G = CTAs of the launch and a CTA's share of the
  // context bound (measured on B200 in 32-layer decode steps of the 7B model
  // at context 4096, where these kernels alternate with MXFP4 GEMVs):
  //  * G above the SM count and shares of at most four 128-token stages:
  //    64-token stages.  Two or more CTAs per SM then fit beside a GEMV CTA
  //    and start early (batch 2: 2516 -> 2328 us a step; batch 4: 2295 -> 2142),
  //    where longer shares want the deeper ring (batch 8: 2688 vs 2915);
  //  * G at most half the SM count: 128-token stages and eight compute warps
  //    (tensor-parallel shards at batch 1: TP2 1224 -> 1181 us, TP8 810 -> 795);
  //  * otherwise 128-token stages and four compute warps (batch 1, one GPU).
  // Pages of 128 tokens need the 128-token stage.  B200KV_DECODE_RING =
  // 128 | 128w8 | 64 forces one.
  const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
  const int64_t grid = (int64_t)csize * hkv * num_seqs;
  const int share = cdiv(ctx_bound, csize);
  int ring = 0;
  if (grid > sms && share <= 4 * 128 && block_size <= 64)
    ring = 2;
  else if (2 * grid <= sms)
    ring = 1;
  const char* renv = getenv("B200KV_DECODE_RING");
  if (renv && renv[0]) {
    ring = 0;
    if (!strcmp(renv, "128w8")) ring = 1;
    else if (!strcmp(renv, "64") && block_size <= 64) ring = 2;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (gqa) {
    case 1: e = launch_ring<1>(ring, km, vm, p, csize, hkv, num_seqs, st); break;
    case 2: e = launch_ring<2>(ring, km, vm, p, csize, hkv, num_seqs, st); break;
    case 4: e = launch_ring<4>(ring, km, vm, p, csize, hkv, num_seqs, st); break;
    case 8: e = launch_ring<8>(ring, km, vm, p, csize, hkv, num_seqs, st); break;
    default: return B200KV_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
