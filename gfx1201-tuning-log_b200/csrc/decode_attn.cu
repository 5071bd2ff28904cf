// fp8-e4m3 (or bf16) paged-KV split-K decode attention for sm_100a.
//
// Same contract as the reference's split-KV flash decode
// (vllm-fp8kv/fp8kv_v3.py:4-113) and its single-pass predecessor
// (vllm-fp8kv/fp8kv_kernel.py:4-72): per (sequence, kv head), the GQA query
// heads of the sequence's query token attend over its paged K/V; k_scale is
// folded into the score scale and v_scale is applied to the output.
//
// B200 design.  The work is 4 multiply-adds per KV byte at GQA 4, and on CUDA
// cores the fp8 -> fp32 converts, packed FMAs and cross-lane reductions cost
// ~11 instructions per HBM byte (measured with ncu on the first version of
// this kernel, 47% issue utilisation at 1.3 TB/s), far more than an HBM-bound
// kernel can afford.  So the dot products run on the tensor pipe (mma.sync,
// fp32 accumulation), the way the reference's own kernel used tl.dot
// (fp8kv_v3.py:67,73), and the kernel stays HBM-bound:
//  * One thread-block CLUSTER of CS CTAs (CS <= 16) per (sequence, kv head);
//    CTA r of the cluster owns an equal share of the context.  The shares'
//    (m, l, o) partials are merged through distributed shared memory at the
//    end, so there is no global scratch, no atomic and no second launch.
//  * A CTA (4 warps) streams its share in 128-token chunks: one thread per K
//    and V row issues 16-byte asynchronous copies (cp.async) into a
//    double-buffered stage, so the next chunk is in flight while this one is
//    computed.  The block-table gather is one cached int load per row.
//  * Each warp owns 32 tokens of a chunk.  S^T = q K^T with the GQA heads as
//    the 16 rows of the A operand (q, pre-scaled to f16 by an exact power of
//    two per head) and 8 tokens as the B operand, read straight from the fp8
//    rows with one 32-bit load and two fp8x2 -> f16x2 hardware converts
//    (exact).  The S^T accumulator fragments ARE the B-operand fragments of
//    O^T += V^T P^T, so P never leaves registers; V^T comes from ldmatrix.trans
//    over the rows converted to f16 (exact).  P is rounded to f16 for the MMA
//    (the reference rounds it to bf16, fp8kv_v3.py:73).
//  * Online softmax per warp in the log2 domain; warps and cluster peers merge
//    with the log-sum-exp weights of the reference's reduce (fp8kv_v3.py:97-113).
//  * bf16 caches (fp8kv_kernel.py's K_FP8=False) run the same schedule with
//    bf16 operands and no converts.

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "warp_mma.cuh"

namespace cg = cooperative_groups;

namespace b200kv {

constexpr int kHeadDim = 128;
constexpr int kChunk = 128;          // tokens staged per pipeline stage
constexpr int kWarps = 4;            // each warp owns 32 tokens of a chunk
constexpr int kThreads = kWarps * 32;
constexpr int kMaxCluster = 16;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  const uint8_t* k;  // byte pointers; strides below are in bytes
  const uint8_t* v;
  int64_t sk0, sk1, sk2, sv0, sv1, sv2;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  const int32_t* qsl;
  const int32_t* seq_lens;
  const int32_t* bt;
  int64_t bt_stride;
  const float* k_scale;
  const float* v_scale;
  float sm_scale;
  int block_size, bs_shift;  // bs_shift = log2(block_size) or -1
  int out_by_qsl;  // bit 0: output row qsl[s] (else s); bit 1: one-token sequences only
};

namespace {

// Shared-memory layout of one CTA.  K rows are padded so the 8 tokens x 4
// lanes of a B-fragment load hit distinct banks; V rows that ldmatrix reads are
// padded to 272 bytes so its 8 row addresses hit distinct 16-byte groups.
template <bool FP8>
struct Layout {
  static constexpr int KP = FP8 ? 144 : 288;        // K row pitch (bytes)
  static constexpr int VP = FP8 ? 128 : 272;        // V row pitch as staged
  static constexpr int CP = 272;                    // f16 V row pitch after convert
  static constexpr int STAGE = kChunk * (KP + VP);
  static constexpr int VCONV = FP8 ? kWarps * 32 * CP : 0;
  static constexpr int BYTES = 2 * STAGE + VCONV;
};

template <int GQA>
struct DecodeShared {
  alignas(16) float part_o[GQA][kHeadDim];  // this CTA's unnormalised o (read by peers)
  float wm[kWarps][8], wl[kWarps][8];       // per-warp softmax state at the end
  float part_m[8], part_l[8];               // this CTA's max / sum (read by peers)
  float rm[kMaxCluster][8], rl[kMaxCluster][8];  // every rank's (m, l)
  float rw[kMaxCluster][8];                 // every rank's weight in the output
};

// One CTA = 4 warps = one share of a (sequence, kv head)'s context; cluster
// peers hold the other shares.  Per 128-token chunk each warp owns 32 tokens:
//   S^T = q (A: 16 rows = the GQA heads, zero-padded) x K^T (B: 8 tokens)
//   O^T += V^T (A: 16 dims x 16 tokens, ldmatrix.trans) x P^T (B: the S^T
//          accumulator fragments rounded to f16 -- same register layout)
// with an online softmax per warp; warps and cluster peers merge at the end.
template <int GQA, bool FP8>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const DecodeParams p) {
  using L = Layout<FP8>;
  constexpr int RB = FP8 ? kHeadDim : 2 * kHeadDim;  // bytes per cached row
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ DecodeShared<GQA> S;

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int kh = blockIdx.y;
  const int seq = blockIdx.z;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int g = lane >> 2;   // fragment row group: head (S^T) / token (K^T)
  const int c = lane & 3;

  // mixed batches: sequences with more than one query token belong to the
  // varlen prefill kernel (cluster-uniform: the cluster serves one sequence)
  if ((p.out_by_qsl & 2) && p.qsl[seq + 1] - p.qsl[seq] != 1) {
    griddep_wait();
    return;
  }

  // The next kernel may launch now.  Sequence metadata and block-table rows
  // are read before this grid waits on the previous one (no kernel that
  // triggers early writes them); q, K and V are read, and the output written,
  // only after griddep_wait().
  if (tid == 0) griddep_launch_dependents();
  const int seqlen = max(p.seq_lens[seq], 0);
  const int q_tok = p.qsl[seq];
  const int out_row = (p.out_by_qsl & 1) ? q_tok : seq;
  const int per = ((seqlen + csize - 1) / csize + 15) & ~15;
  const int lo = min(seqlen, rank * per);
  const int hi = min(seqlen, lo + per);
  const int nchunks = (hi - lo + kChunk - 1) / kChunk;
  const int32_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;

  // ---- chunk loader: one thread per row (kChunk == kThreads), 16-byte pieces --
  auto row_block = [&](int ch) -> int64_t {  // block of this thread's row, or -1
    const int tok = lo + ch * kChunk + tid;
    if (ch >= nchunks || tok >= hi) return -1;
    const int bi = p.bs_shift >= 0 ? tok >> p.bs_shift : tok / p.block_size;
    return bt_row[bi];
  };
  auto issue_chunk = [&](int ch, int64_t blk) {
    uint8_t* ks = smem + (ch & 1) * L::STAGE;
    uint8_t* vs = ks + kChunk * L::KP;
    const int tok = lo + ch * kChunk + tid;
    if (blk >= 0) {
      const int64_t slot = p.bs_shift >= 0 ? tok & (p.block_size - 1) : tok % p.block_size;
      const uint8_t* kg = p.k + blk * p.sk0 + slot * p.sk1 + kh * p.sk2;
      const uint8_t* vg = p.v + blk * p.sv0 + slot * p.sv1 + kh * p.sv2;
#pragma unroll
      for (int j = 0; j < RB / 16; ++j) {
        cp_async16(ks + tid * L::KP + j * 16, kg + j * 16);
        cp_async16(vs + tid * L::VP + j * 16, vg + j * 16);
      }
    }
    cp_async_commit();
  };
  // both stages' block-table entries before the wait, then both stages in flight
  const int64_t blk0 = row_block(0), blk1 = row_block(1);
  griddep_wait();
  issue_chunk(0, blk0);
  issue_chunk(1, blk1);

  // ---- q as the A operand: rows = heads (g < GQA), per-head exact prescale --
  // A fragment of 16 dims: a0 = (head g, dims 4c, 4c+1), a2 = (head g, dims
  // 4c+2, 4c+3); rows 8..15 (a1, a3) are zero.  The same dim order is used for
  // the K^T B fragments, so the permutation inside a 16-dim slice cancels.
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
    float base = p.sm_scale * (FP8 ? __ldg(p.k_scale) : 1.f) * kLog2e;
    if constexpr (FP8) {
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
      base *= __uint_as_float((uint32_t)(127 - sh) << 23);
#pragma unroll
      for (int ds = 0; ds < 8; ++ds) {
        qa[ds][0] = pack_f16x2(qv[ds][0] * up, qv[ds][1] * up);
        qa[ds][1] = pack_f16x2(qv[ds][2] * up, qv[ds][3] * up);
      }
    } else {
#pragma unroll
      for (int ds = 0; ds < 8; ++ds) {
        qa[ds][0] = pack_bf16x2(qv[ds][0], qv[ds][1]);
        qa[ds][1] = pack_bf16x2(qv[ds][2], qv[ds][3]);
      }
    }
    if (g >= GQA) {
#pragma unroll
      for (int ds = 0; ds < 8; ++ds) qa[ds][0] = qa[ds][1] = 0u;
    }
    score_scale = base;
  }

  // ---- per-warp online softmax state (thread (g, c) tracks head g) ---------
  float m_run = -INFINITY, l_run = 0.f;
  float o[8][4];  // O^T fragments: dims 16i + {g, g+8}, heads {2c, 2c+1}
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;

  for (int ch = 0; ch < nchunks; ++ch) {
    // chunks ch and ch+1 are in flight (an empty group stands in past the end)
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t* ks = smem + (ch & 1) * L::STAGE;
    const uint8_t* vs = ks + kChunk * L::KP;
    const int nt = min(kChunk, hi - (lo + ch * kChunk));
    const int w0 = warp * 32;                 // this warp's first token in the chunk
    const int ntw = max(0, min(32, nt - w0));  // its valid tokens
    if (ntw > 0) {  // this warp's tokens of the chunk

      // V rows of this warp as f16 (fp8 path), zero past the valid tokens
      const uint8_t* vrows;
      int vpitch;
      if constexpr (FP8) {
        uint8_t* vc = smem + 2 * L::STAGE + warp * 32 * L::CP;
        for (int i = lane; i < 32 * 16; i += 32) {
          const int r = i >> 4, j = i & 15;  // row, 8-byte piece
          uint4 h = make_uint4(0, 0, 0, 0);
          if (r < ntw) {
            const uint2 raw = *reinterpret_cast<const uint2*>(vs + (w0 + r) * L::VP + j * 8);
            h.x = e4m3x2_to_f16x2(raw.x & 0xFFFFu);
            h.y = e4m3x2_to_f16x2(raw.x >> 16);
            h.z = e4m3x2_to_f16x2(raw.y & 0xFFFFu);
            h.w = e4m3x2_to_f16x2(raw.y >> 16);
          }
          *reinterpret_cast<uint4*>(vc + r * L::CP + j * 16) = h;
        }
        __syncwarp();
        vrows = vc;
        vpitch = L::CP;
      } else {
        // rows past the valid tokens hold stale bytes: zero them so 0 * V stays 0
        uint8_t* vw = const_cast<uint8_t*>(vs) + w0 * L::VP;
        for (int i = ntw * 16 + lane; i < 32 * 16; i += 32)
          *reinterpret_cast<uint4*>(vw + (i >> 4) * L::VP + (i & 15) * 16) = make_uint4(0, 0, 0, 0);
        __syncwarp();
        vrows = vw;
        vpitch = L::VP;
      }

      // ---- S^T = q K^T over 4 token tiles of 8 --------------------------------
      float sfr[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sfr[t][e] = 0.f;
        const uint8_t* krow = ks + (w0 + 8 * t + g) * L::KP;
#pragma unroll
        for (int ds = 0; ds < 8; ++ds) {
          uint32_t b0, b1;
          if constexpr (FP8) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(krow + 16 * ds + 4 * c);
            b0 = e4m3x2_to_f16x2(w & 0xFFFFu);
            b1 = e4m3x2_to_f16x2(w >> 16);
          } else {
            const uint2 w = *reinterpret_cast<const uint2*>(krow + 32 * ds + 8 * c);
            b0 = w.x;
            b1 = w.y;
          }
          mma16816<FP8>(sfr[t], qa[ds][0], 0u, qa[ds][1], 0u, b0, b1);
        }
      }

      // ---- online softmax for head g over this warp's tokens ------------------
      float mx = -INFINITY;
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tok = 8 * t + 2 * c + e;
          const float v = tok < ntw ? sfr[t][e] * score_scale : -INFINITY;
          sfr[t][e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);          // finite: ntw >= 1
      const float alpha = exp2f(m_run - m_new);      // 0 on the first chunk
      m_run = m_new;
      float psum = 0.f;
      uint32_t pb[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float p0 = exp2f(sfr[t][0] - m_new);
        const float p1 = exp2f(sfr[t][1] - m_new);
        psum += p0 + p1;
        pb[t] = FP8 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
      }
      l_run = l_run * alpha + psum;
      // rescale O^T: this thread holds heads 2c and 2c+1, whose alpha lives in
      // the lanes with g == 2c / 2c+1
      const float a0 = __shfl_sync(0xffffffffu, alpha, (2 * c) * 4);
      const float a1 = __shfl_sync(0xffffffffu, alpha, (2 * c + 1) * 4);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= a0; o[i][1] *= a1; o[i][2] *= a0; o[i][3] *= a1;
      }

      // ---- O^T += V^T P^T over 2 token slices of 16 ---------------------------
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int vtok = 16 * j + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t a[4];
          ldsm_x4_trans(a, vrows + vtok * vpitch + (16 * i + ((lane >> 3) & 1) * 8) * 2);
          mma16816<FP8>(o[i], a[0], a[1], a[2], a[3], pb[2 * j], pb[2 * j + 1]);
        }
      }
    }
    __syncthreads();  // stage ch&1 is free: chunk ch+2 goes there
    issue_chunk(ch + 2, row_block(ch + 2));
  }
  cp_async_wait<0>();  // only empty groups remain; the stages are reused below

  // ---- merge the 4 warps: per-warp state -> this CTA's partial --------------
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (c == 0 && g < 8) {
    S.wm[warp][g] = m_run;
    S.wl[warp][g] = l_run;
  }
  __syncthreads();  // staging buffers are free from here on
  float (*wo)[GQA][kHeadDim] = reinterpret_cast<float (*)[GQA][kHeadDim]>(smem);
  {
    // per-warp weight of head h relative to the CTA max
    float wgt[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int h = 2 * c + e;
      float mc = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) mc = fmaxf(mc, S.wm[w][h & 7]);
      const float mw = S.wm[warp][h & 7];
      wgt[e] = (mw == -INFINITY) ? 0.f : exp2f(mw - mc);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int h = 2 * c + e;
        if (h < GQA) {
          wo[warp][h][16 * i + g] = o[i][e] * wgt[e];
          wo[warp][h][16 * i + g + 8] = o[i][2 + e] * wgt[e];
        }
      }
  }
  __syncthreads();
  for (int e = tid; e < GQA * kHeadDim; e += kThreads) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += wo[w][h][d];
    S.part_o[h][d] = s;
  }
  if (tid < GQA) {
    float mc = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mc = fmaxf(mc, S.wm[w][tid]);
    float lc = 0.f;
    if (mc != -INFINITY)
#pragma unroll
      for (int w = 0; w < kWarps; ++w)
        if (S.wm[w][tid] != -INFINITY) lc += S.wl[w][tid] * exp2f(S.wm[w][tid] - mc);
    S.part_m[tid] = mc;
    S.part_l[tid] = lc;
  }
  const float vsc = FP8 ? __ldg(p.v_scale) : 1.f;
  __nv_bfloat16* out_base = p.out + (int64_t)out_row * p.o_st + (int64_t)(kh * GQA) * p.o_sh;

  // ---- merge the cluster's partials through distributed shared memory -----
  // Every remote read is issued independently of the others: one round of
  // (m, l) loads, then one float4 of one rank's o per work item, so the merge
  // costs two distributed-shared-memory round trips whatever the cluster size.
  cluster.sync();
  if (tid < csize * GQA) {
    const int r = tid / GQA, h = tid % GQA;
    S.rm[r][h] = cluster.map_shared_rank(&S.part_m[0], r)[h];
    S.rl[r][h] = cluster.map_shared_rank(&S.part_l[0], r)[h];
  }
  __syncthreads();
  if (tid < GQA) {
    float mg = -INFINITY;
    for (int r = 0; r < csize; ++r) mg = fmaxf(mg, S.rm[r][tid]);
    float lg = 0.f;
    if (mg != -INFINITY)
      for (int r = 0; r < csize; ++r)
        if (S.rm[r][tid] != -INFINITY) lg += exp2f(S.rm[r][tid] - mg) * S.rl[r][tid];
    const float inv = lg > 0.f ? vsc / lg : 0.f;
    for (int r = 0; r < csize; ++r)
      S.rw[r][tid] = (mg != -INFINITY && S.rm[r][tid] != -INFINITY) ? exp2f(S.rm[r][tid] - mg) * inv : 0.f;
  }
  __syncthreads();
  // this CTA writes elements [e0, e0 + per_cta) of the (head, dim) block;
  // contribution of rank r to element i lands in contrib[r * per_cta + i]
  constexpr int E = GQA * kHeadDim;
  const int per_cta = E / csize, nv = per_cta / 4, e0 = rank * per_cta;
  float* contrib = reinterpret_cast<float*>(smem);  // the stages are free
  for (int it = tid; it < csize * nv; it += kThreads) {
    const int r = it / nv, v = it - r * nv;
    const int e = e0 + 4 * v;
    const float w = S.rw[r][e / kHeadDim];
    float4 ov = make_float4(0.f, 0.f, 0.f, 0.f);
    if (w != 0.f) ov = *reinterpret_cast<const float4*>(cluster.map_shared_rank(&S.part_o[0][0], r) + e);
    *reinterpret_cast<float4*>(contrib + r * per_cta + 4 * v) =
        make_float4(w * ov.x, w * ov.y, w * ov.z, w * ov.w);
  }
  __syncthreads();
  for (int i = tid; i < per_cta; i += kThreads) {
    float acc = 0.f;
    for (int r = 0; r < csize; ++r) acc += contrib[r * per_cta + i];
    const int e = e0 + i, h = e / kHeadDim, d = e % kHeadDim;
    out_base[(int64_t)h * p.o_sh + d] = __float2bfloat16_rn(acc);
  }
  cluster.sync();  // peers' shared memory stays alive until every rank is done
}

template <int GQA, bool FP8>
cudaError_t launch_decode(const DecodeParams& p, int csize, int hkv, int num_seqs,
                          cudaStream_t stream) {
  const size_t smem = Layout<FP8>::BYTES;
  static_assert(Layout<FP8>::BYTES >= kWarps * GQA * kHeadDim * 4, "stages must hold the merge");
  cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<GQA, FP8>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (csize > 8) {
    e = cudaFuncSetAttribute(decode_attn_kernel<GQA, FP8>,
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(csize, hkv, num_seqs);
  lc.blockDim = dim3(kThreads, 1, 1);
  lc.dynamicSmemBytes = smem;
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
  return cudaLaunchKernelEx(&lc, decode_attn_kernel<GQA, FP8>, p);
}

}  // namespace

int decode_tma_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                      const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                      int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                      const int32_t* qsl, const int32_t* seq_lens, const int32_t* bt,
                      int64_t bt_stride, const float* k_scale, const float* v_scale,
                      float sm_scale, int num_seqs, int hkv, int gqa, int block_size,
                      int num_blocks, int out_by_qsl, int csize, int ctx_bound, void* stream);

// Cluster size (CTAs per (sequence, kv head)): the largest power of two <= 16
// that keeps the grid within two CTAs per SM, but at least one CTA per 4096
// tokens of the context bound, and at least 64 tokens per CTA.
int decode_cluster_size(int num_seqs, int hkv, int ctx_bound, int requested) {
  int want;
  if (requested > 0) {
    want = requested;
  } else {
    const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
    const int pairs = num_seqs * hkv;
    want = 1;
    while (want * 2 <= kMaxCluster && pairs * want * 2 <= 2 * sms) want *= 2;
    const int need = cdiv(ctx_bound, 4096);
    if (want < need) want = need;
    const int cap = cdiv(ctx_bound, 64);
    if (want > cap) want = cap;
  }
  int cs = 1;
  while (cs < want && cs < kMaxCluster) cs *= 2;
  return cs;
}

int decode_attn_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                       const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                       int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                       const int32_t* qsl, const int32_t* seq_lens, const int32_t* bt,
                       int64_t bt_stride, const float* k_scale, const float* v_scale,
                       float sm_scale, int num_seqs, int hq, int hkv, int head_dim,
                       int block_size, int num_blocks, int max_blocks, int hint, int kv_dtype,
                       int out_by_qsl, int num_splits, void* stream) {
  if (!q || !k_cache || !v_cache || !out || !qsl || !seq_lens || !bt) return B200KV_ERR_INVALID_ARG;
  if (num_seqs <= 0 || hq <= 0 || hkv <= 0 || block_size <= 0 || max_blocks <= 0)
    return B200KV_ERR_INVALID_ARG;
  if (hq % hkv) return B200KV_ERR_INVALID_ARG;
  if (head_dim != kHeadDim) return B200KV_ERR_UNSUPPORTED;
  if (kv_dtype != B200KV_KV_FP8_E4M3 && kv_dtype != B200KV_KV_BF16) return B200KV_ERR_UNSUPPORTED;
  const bool fp8 = kv_dtype == B200KV_KV_FP8_E4M3;
  if (fp8 && (!k_scale || !v_scale)) return B200KV_ERR_INVALID_ARG;
  const int gqa = hq / hkv;
  if (gqa != 1 && gqa != 2 && gqa != 4 && gqa != 8) return B200KV_ERR_UNSUPPORTED;
  if (num_splits < 0 || num_splits > kMaxCluster) return B200KV_ERR_UNSUPPORTED;
  const int esz = fp8 ? 1 : 2;
  const int64_t strides[6] = {sk0, sk1, sk2, sv0, sv1, sv2};
  for (int i = 0; i < 6; ++i)
    if ((strides[i] * esz) % 16) return B200KV_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(q) & 15) || ((q_st % 8) != 0) || ((q_sh % 8) != 0))
    return B200KV_ERR_MISALIGNED;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;

  const int ctx = hint > 0 ? hint : max_blocks * block_size;
  const int cs = decode_cluster_size(num_seqs, hkv, ctx, num_splits);
  if (fp8) {  // pages by TMA when the cache can be described by tensor maps
    const int r = decode_tma_launch(q, q_st, q_sh, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2,
                                    out, o_st, o_sh, qsl, seq_lens, bt, bt_stride, k_scale, v_scale,
                                    sm_scale, num_seqs, hkv, gqa, block_size, num_blocks, out_by_qsl,
                                    cs, ctx, stream);
    if (r != B200KV_ERR_UNSUPPORTED) return r;
  }

  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_st;
  p.q_sh = q_sh;
  p.k = static_cast<const uint8_t*>(k_cache);
  p.v = static_cast<const uint8_t*>(v_cache);
  p.sk0 = sk0 * esz; p.sk1 = sk1 * esz; p.sk2 = sk2 * esz;
  p.sv0 = sv0 * esz; p.sv1 = sv1 * esz; p.sv2 = sv2 * esz;
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
  p.block_size = block_size;
  p.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz((unsigned)block_size) : -1;
  p.out_by_qsl = out_by_qsl;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (gqa * 2 + (fp8 ? 1 : 0)) {
    case 3: e = launch_decode<1, true>(p, cs, hkv, num_seqs, st); break;
    case 2: e = launch_decode<1, false>(p, cs, hkv, num_seqs, st); break;
    case 5: e = launch_decode<2, true>(p, cs, hkv, num_seqs, st); break;
    case 4: e = launch_decode<2, false>(p, cs, hkv, num_seqs, st); break;
    case 9: e = launch_decode<4, true>(p, cs, hkv, num_seqs, st); break;
    case 8: e = launch_decode<4, false>(p, cs, hkv, num_seqs, st); break;
    case 17: e = launch_decode<8, true>(p, cs, hkv, num_seqs, st); break;
    case 16: e = launch_decode<8, false>(p, cs, hkv, num_seqs, st); break;
    default: return B200KV_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
