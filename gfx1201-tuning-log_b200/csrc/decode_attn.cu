// fp8-e4m3 (or bf16) paged-KV split-K decode attention for sm_100a.
//
// Same contract as the reference's split-KV flash decode
// (vllm-fp8kv/fp8kv_v3.py:4-113) and its single-pass predecessor
// (vllm-fp8kv/fp8kv_kernel.py:4-72): per (sequence, kv head), the GQA query
// heads of the sequence's query token attend over its paged K/V; k_scale is
// folded into the score scale and v_scale is applied to the output.
//
// B200 design (CUDA cores, no tensor cores -- the work is 4 multiply-adds per
// KV byte at GQA 4 and the kernel is HBM-bound):
//  * One thread-block CLUSTER of CS CTAs (CS <= 16) per (sequence, kv head);
//    CTA r of the cluster owns an equal share of the context.  The shares'
//    (m, l, o) partials are merged through distributed shared memory at the
//    end, so there is no global scratch, no atomic and no second launch.
//  * A CTA (16 warps; 8 for GQA 8) streams its share in 128-token chunks with 16-byte
//    asynchronous copies (cp.async) of every K and V row into a double-buffered
//    shared-memory stage: the next chunk is in flight while the current one is
//    computed.  The block-table gather is one cached int load per row.
//  * Pass 1 (QK): 16 lanes per token, 8 dims per lane, fp8x2 -> f16x2 hardware
//    converts, packed fp32 FMA (FFMA2) against the pre-scaled query held in
//    registers, and a 16-lane reduce-scatter so each lane ends with one
//    (token, head) score.  Scores go to shared memory in the log2 domain.
//  * The softmax is exact inside a chunk (max, exp2, sum per head); chunks are
//    merged online (running max and sum, one rescale of the fp32 accumulators
//    per chunk).  Pass 2 (PV) accumulates p * V with FFMA2 and a shared-memory
//    reduction folds the token groups.
//  * The log-sum-exp merge of the cluster's partials is the one the reference
//    does in its reduce kernel (fp8kv_v3.py:97-113).

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace cg = cooperative_groups;

namespace b200kv {

constexpr int kHeadDim = 128;
constexpr int kChunk = 128;          // tokens staged per pipeline stage
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
  int block_size, out_by_qsl;
};

namespace {

// 8 KV elements (one lane's 8 dims) -> 8 fp32.
template <bool FP8>
struct KvConvert;

template <>
struct KvConvert<true> {
  static constexpr int kRowBytes = kHeadDim;
  __device__ __forceinline__ static void load8(const uint8_t* p, float2 (&f)[4]) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const uint32_t w[2] = {raw.x, raw.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const __half2_raw lo =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xFFFFu), __NV_E4M3);
      const __half2_raw hi =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
      f[2 * i] = __half22float2(*reinterpret_cast<const __half2*>(&lo));
      f[2 * i + 1] = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    }
  }
};

template <>
struct KvConvert<false> {
  static constexpr int kRowBytes = kHeadDim * 2;
  __device__ __forceinline__ static void load8(const uint8_t* p, float2 (&f)[4]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      f[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
  }
};

// 16-lane reduce-scatter: on entry v[0..15] are this lane's partials; on exit
// v[0] holds the sum over the 16 lanes of entry v[sub] (sub = lane % 16).
__device__ __forceinline__ void reduce_scatter16(float (&v)[16], int sub) {
#pragma unroll
  for (int half = 8; half >= 1; half >>= 1) {
    const bool upper = (sub & half) != 0;
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float keep = upper ? v[j + half] : v[j];
      const float send = upper ? v[j] : v[j + half];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, half);
    }
  }
}

template <int GQA>
struct DecodeSmem {
  float sc[GQA][kChunk];      // scores of the chunk (log2 domain)
  float pt[kChunk][GQA];      // probabilities, token-major for pass 2
  float part_o[GQA][kHeadDim];  // this CTA's unnormalised o (read by cluster peers)
  float part_m[8], part_l[8];   // this CTA's running max / sum (read by peers)
  float alpha[8];               // per-chunk rescale of the running o
  float run_m[8], run_l[8];
  float comb_m[8], comb_l[8];
};

// Threads per CTA: 512 (32 token groups of 16 lanes) keeps 16 warps per SM busy
// even when a (sequence, kv head) gets only one CTA per SM; GQA 8 needs twice
// the query/accumulator registers per lane, so it runs 256 threads.
template <int GQA>
constexpr int decode_threads() { return GQA <= 4 ? 512 : 256; }

template <int GQA, bool FP8>
__global__ void __launch_bounds__(decode_threads<GQA>())
    decode_attn_kernel(const DecodeParams p) {
  using Cvt = KvConvert<FP8>;
  constexpr int NTHR = decode_threads<GQA>();
  constexpr int NWARP = NTHR / 32;
  constexpr int NG = NTHR / 16;       // 16-lane token groups
  constexpr int RB = Cvt::kRowBytes;
  constexpr int CPR = RB / 16;        // 16-byte chunks per row
  constexpr int TQ = 16 / GQA;        // tokens per 16-lane group step in pass 1
  constexpr int STAGE = 2 * kChunk * RB;
  static_assert(2 * STAGE >= NWARP * GQA * kHeadDim * 4, "stages must hold the warp reduction");

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;                                         // [2][K|V][kChunk][RB]
  DecodeSmem<GQA>& S = *reinterpret_cast<DecodeSmem<GQA>*>(smem + 2 * STAGE);

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int kh = blockIdx.y;
  const int seq = blockIdx.z;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int sub = lane & 15;
  const int grp = tid >> 4;  // 0..NG-1

  const int seqlen = max(p.seq_lens[seq], 0);
  const int q_tok = p.qsl[seq];
  const int out_row = p.out_by_qsl ? q_tok : seq;
  // this CTA's token range: an equal share, rounded to 16 tokens
  const int per = ((seqlen + csize - 1) / csize + 15) & ~15;
  const int lo = min(seqlen, rank * per);
  const int hi = min(seqlen, lo + per);
  const int nchunks = (hi - lo + kChunk - 1) / kChunk;
  const int32_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;

  auto issue_chunk = [&](int c) {
    uint8_t* ks = stages + (c & 1) * STAGE;
    uint8_t* vs = ks + kChunk * RB;
    const int t0 = lo + c * kChunk;
    const int nt = min(kChunk, hi - t0);
    for (int i = tid; i < nt * CPR; i += NTHR) {
      const int r = i / CPR, ch = i % CPR;
      const int tok = t0 + r;
      const int64_t blk = bt_row[tok / p.block_size];
      const int64_t slot = tok % p.block_size;
      cp_async16(ks + r * RB + ch * 16, p.k + blk * p.sk0 + slot * p.sk1 + kh * p.sk2 + ch * 16);
      cp_async16(vs + r * RB + ch * 16, p.v + blk * p.sv0 + slot * p.sv1 + kh * p.sv2 + ch * 16);
    }
    cp_async_commit();
  };
  if (nchunks > 0) issue_chunk(0);

  // ---- query: this lane's 8 dims of every GQA head, pre-scaled ------------
  const float qscale = p.sm_scale * (FP8 ? __ldg(p.k_scale) : 1.f) * kLog2e;
  float2 qf[GQA][4];
  {
    const __nv_bfloat16* qb = p.q + (int64_t)q_tok * p.q_st + (int64_t)(kh * GQA) * p.q_sh;
#pragma unroll
    for (int h = 0; h < GQA; ++h) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qb + (int64_t)h * p.q_sh + 8 * sub);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qf[h][i] = make_float2(__uint_as_float(w[i] << 16) * qscale,
                               __uint_as_float(w[i] & 0xFFFF0000u) * qscale);
    }
  }
  if (tid < 8) {
    S.run_m[tid] = -INFINITY;
    S.run_l[tid] = 0.f;
  }
  float2 of[GQA][4];
#pragma unroll
  for (int h = 0; h < GQA; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) of[h][e] = make_float2(0.f, 0.f);

  for (int c = 0; c < nchunks; ++c) {
    __syncthreads();  // stage (c+1)&1 and the score buffers are free again
    if (c + 1 < nchunks) {
      issue_chunk(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint8_t* ks = stages + (c & 1) * STAGE;
    const uint8_t* vs = ks + kChunk * RB;
    const int nt = min(kChunk, hi - (lo + c * kChunk));

    // ---- pass 1: scores (both 16-lane groups of a warp run the same trips) --
    for (int wbase = warp * 2 * TQ; wbase < nt; wbase += NG * TQ) {
      const int base = wbase + (grp & 1) * TQ;
      float v[16];
#pragma unroll
      for (int i = 0; i < TQ; ++i) {
        const int tok = base + i;
        float2 kf[4];
        if (tok < nt) {
          Cvt::load8(ks + tok * RB + 8 * sub * (RB / kHeadDim), kf);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) kf[e] = make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int h = 0; h < GQA; ++h) {
          float2 a = __fmul2_rn(qf[h][0], kf[0]);
#pragma unroll
          for (int e = 1; e < 4; ++e) a = __ffma2_rn(qf[h][e], kf[e], a);
          v[i * GQA + h] = a.x + a.y;
        }
      }
      reduce_scatter16(v, sub);
      const int tok = base + sub / GQA;
      if (tok < nt) S.sc[sub % GQA][tok] = v[0];
    }
    __syncthreads();

    // ---- chunk statistics and online merge into the running state ---------
    for (int h = warp; h < GQA; h += NWARP) {
      float m = -INFINITY;
      for (int t = lane; t < nt; t += 32) m = fmaxf(m, S.sc[h][t]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float m_old = S.run_m[h];
      const float m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int t = lane; t < nt; t += 32) {
        const float e = exp2f(S.sc[h][t] - m_new);
        S.pt[t][h] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) {
        const float a = exp2f(m_old - m_new);  // 0 on the first chunk
        S.alpha[h] = a;
        S.run_l[h] = S.run_l[h] * a + l;
        S.run_m[h] = m_new;
      }
    }
    __syncthreads();

    // ---- pass 2: o = o * alpha + sum_t p[t] * V[t] --------------------------
#pragma unroll
    for (int h = 0; h < GQA; ++h) {
      const float2 a2 = make_float2(S.alpha[h], S.alpha[h]);
#pragma unroll
      for (int e = 0; e < 4; ++e) of[h][e] = __fmul2_rn(of[h][e], a2);
    }
    for (int tok = grp; tok < nt; tok += NG) {
      float2 vf[4];
      Cvt::load8(vs + tok * RB + 8 * sub * (RB / kHeadDim), vf);
      float pw[GQA];
      if constexpr (GQA == 4) {
        const float4 p4 = *reinterpret_cast<const float4*>(&S.pt[tok][0]);
        pw[0] = p4.x; pw[1] = p4.y; pw[2] = p4.z; pw[3] = p4.w;
      } else {
#pragma unroll
        for (int h = 0; h < GQA; ++h) pw[h] = S.pt[tok][h];
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) {
        const float2 pp = make_float2(pw[h], pw[h]);
#pragma unroll
        for (int e = 0; e < 4; ++e) of[h][e] = __ffma2_rn(pp, vf[e], of[h][e]);
      }
    }
  }

  // ---- fold the token groups: this CTA's unnormalised partial ---------------
  // (the two groups of a warp through a shuffle, the warps through the staging
  // buffers, which are free now)
#pragma unroll
  for (int h = 0; h < GQA; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      of[h][e].x += __shfl_xor_sync(0xffffffffu, of[h][e].x, 16);
      of[h][e].y += __shfl_xor_sync(0xffffffffu, of[h][e].y, 16);
    }
  __syncthreads();
  float (*red)[GQA][kHeadDim] = reinterpret_cast<float (*)[GQA][kHeadDim]>(stages);
  if (lane < 16) {
#pragma unroll
    for (int h = 0; h < GQA; ++h) {
      float4* dst = reinterpret_cast<float4*>(&red[warp][h][8 * sub]);
      dst[0] = make_float4(of[h][0].x, of[h][0].y, of[h][1].x, of[h][1].y);
      dst[1] = make_float4(of[h][2].x, of[h][2].y, of[h][3].x, of[h][3].y);
    }
  }
  __syncthreads();
  for (int e = tid; e < GQA * kHeadDim; e += NTHR) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) s += red[w][h][d];
    S.part_o[h][d] = s;
  }
  if (tid < GQA) {
    S.part_m[tid] = S.run_m[tid];
    S.part_l[tid] = S.run_l[tid];
  }
  const float vsc = FP8 ? __ldg(p.v_scale) : 1.f;
  __nv_bfloat16* out_base = p.out + (int64_t)out_row * p.o_st + (int64_t)(kh * GQA) * p.o_sh;

  // ---- merge the cluster's partials through distributed shared memory -----
  cluster.sync();
  if (tid < GQA) {
    float mg = -INFINITY;
    for (int r = 0; r < csize; ++r) mg = fmaxf(mg, cluster.map_shared_rank(&S.part_m[0], r)[tid]);
    float lg = 0.f;
    if (mg != -INFINITY)
      for (int r = 0; r < csize; ++r)
        lg += exp2f(cluster.map_shared_rank(&S.part_m[0], r)[tid] - mg) *
              cluster.map_shared_rank(&S.part_l[0], r)[tid];
    S.comb_m[tid] = mg;
    S.comb_l[tid] = lg;
  }
  __syncthreads();
  // rank r writes elements [r*E/csize, (r+1)*E/csize) of the GQA x 128 output
  constexpr int E = GQA * kHeadDim;
  const int e0 = rank * E / csize, e1 = (rank + 1) * E / csize;
  for (int e = e0 + tid; e < e1; e += NTHR) {
    const int h = e / kHeadDim, d = e % kHeadDim;
    const float mg = S.comb_m[h];
    float acc = 0.f;
    if (mg != -INFINITY)
      for (int r = 0; r < csize; ++r)
        acc += exp2f(cluster.map_shared_rank(&S.part_m[0], r)[h] - mg) *
               cluster.map_shared_rank(&S.part_o[0][0], r)[h * kHeadDim + d];
    const float lg = S.comb_l[h];
    out_base[(int64_t)h * p.o_sh + d] = __float2bfloat16_rn(lg > 0.f ? acc * vsc / lg : 0.f);
  }
  cluster.sync();  // peers' shared memory stays alive until every rank is done
}

template <int GQA, bool FP8>
size_t decode_smem_bytes() {
  const size_t rb = FP8 ? kHeadDim : 2 * kHeadDim;
  return 2 * 2 * kChunk * rb + sizeof(DecodeSmem<GQA>);
}

template <int GQA, bool FP8>
cudaError_t launch_decode(const DecodeParams& p, int csize, int hkv, int num_seqs,
                          cudaStream_t stream) {
  const size_t smem = decode_smem_bytes<GQA, FP8>();
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
  lc.blockDim = dim3(decode_threads<GQA>(), 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, decode_attn_kernel<GQA, FP8>, p);
}

}  // namespace

// Cluster size (CTAs per (sequence, kv head)): the largest power of two <= 16
// that keeps the grid within one CTA per SM, but at least one CTA per 4096
// tokens of the context bound, and at least 64 tokens per CTA.
int decode_cluster_size(int num_seqs, int hkv, int ctx_bound, int requested) {
  int want;
  if (requested > 0) {
    want = requested;
  } else {
    const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
    const int pairs = num_seqs * hkv;
    want = 1;
    while (want * 2 <= kMaxCluster && pairs * want * 2 <= sms) want *= 2;
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
                       int block_size, int max_blocks, int hint, int kv_dtype, int out_by_qsl,
                       int num_splits, void* stream) {
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
  p.out_by_qsl = out_by_qsl;

  const int ctx = hint > 0 ? hint : max_blocks * block_size;
  const int cs = decode_cluster_size(num_seqs, hkv, ctx, num_splits);
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
