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
//  * One CTA (4 warps) per (split, kv head, sequence).  A split is a span of at
//    most 256 tokens.  At entry the CTA hands every 128-byte K row and V row of
//    its span to the TMA engine as one-dimensional bulk copies into shared
//    memory (two mbarriers: K lands first), so the whole span is in flight at
//    once -- the memory-level parallelism the HBM needs -- and the block table
//    gather costs one cached int load per row.
//  * Pass 1 (QK): 16 lanes per token, 8 dims per lane, fp8x2 -> f16x2 hardware
//    converts, packed fp32 FMA (FFMA2) against the pre-scaled query held in
//    registers, and a 16-lane reduce-scatter so each lane ends with one
//    (token, head) score.  Scores go to shared memory in the log2 domain.
//  * Because the span is resident, the softmax is exact per span (no online
//    rescaling): max, exp2, sum per head, then Pass 2 (PV) accumulates
//    p * V in fp32 registers and a shared-memory reduction folds the 8 token
//    groups.
//  * Splits write (m, l, o) partials; the last CTA of a (sequence, kv head) --
//    found with one atomic on a self-resetting counter -- merges them with the
//    log-sum-exp weights of fp8kv_v3.py:97-113 and writes bf16.  One launch.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace b200kv {

constexpr int kHeadDim = 128;
constexpr int kSpanMax = 256;
constexpr int kDecodeThreads = 128;
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
  int num_seqs, hkv, block_size, span, max_splits, out_by_qsl;
  int* counters;   // [num_seqs * hkv]
  float* part_ml;  // [num_seqs][hkv][max_splits][GQA][2]
  float* part_o;   // [num_seqs][hkv][max_splits][GQA][128]
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

// K+V staging region; after pass 2 it holds the [8 groups][GQA][128] fp32
// reduction, so it is at least that large.
__host__ __device__ constexpr int kv_region_bytes(int span, int rb, int gqa) {
  return (2 * span * rb > 8 * gqa * kHeadDim * 4) ? 2 * span * rb : 8 * gqa * kHeadDim * 4;
}

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

template <int GQA, bool FP8>
__global__ void __launch_bounds__(kDecodeThreads)
    decode_attn_kernel(const DecodeParams p) {
  using Cvt = KvConvert<FP8>;
  constexpr int RB = Cvt::kRowBytes;
  constexpr int TQ = 16 / GQA;  // tokens per 16-lane group step in pass 1

  extern __shared__ __align__(128) uint8_t smem[];
  // layout (span = p.span): [K rows | V rows] (at least 8*GQA*128 floats, reused
  // for the token-group reduction), scores [GQA][span], p [span][GQA], stats, barriers
  const int span = p.span;
  const int kv_bytes = kv_region_bytes(span, RB, GQA);
  uint8_t* ks = smem;
  uint8_t* vs = smem + span * RB;
  float* sc = reinterpret_cast<float*>(smem + kv_bytes);  // [GQA][span]
  float* pt = sc + GQA * span;                              // [span][GQA]
  float* stat_m = pt + GQA * span;                          // [8]
  float* stat_l = stat_m + 8;                               // [8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(stat_l + 8); // [2]
  int* flag = reinterpret_cast<int*>(bars + 2);

  const int sp = blockIdx.x;
  const int kh = blockIdx.y;
  const int seq = blockIdx.z;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int sub = lane & 15;
  const int grp = tid >> 4;  // 0..7

  const int seqlen = p.seq_lens[seq];
  const int q_tok = p.qsl[seq];
  const int out_row = p.out_by_qsl ? q_tok : seq;
  const int lo = sp * p.span;
  __nv_bfloat16* out_base = p.out + (int64_t)out_row * p.o_st + (int64_t)(kh * GQA) * p.o_sh;

  if (seqlen <= 0) {
    if (sp == 0)
      for (int i = tid; i < GQA * kHeadDim; i += kDecodeThreads)
        out_base[(int64_t)(i / kHeadDim) * p.o_sh + (i % kHeadDim)] = __float2bfloat16_rn(0.f);
    return;
  }
  int nsplit = (seqlen + p.span - 1) / p.span;
  if (nsplit > p.max_splits) {
    if (sp == 0 && kh == 0 && tid == 0) atomicExch(&g_device_status, kDevSplitOverflow);
    nsplit = p.max_splits;
  }
  if (lo >= seqlen || sp >= nsplit) return;
  const int hi = min(seqlen, lo + p.span);
  const int nt = hi - lo;

  // ---- stage K and V rows of the span through the TMA engine ---------------
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], (uint32_t)(nt * RB));
    mbar_arrive_expect_tx(&bars[1], (uint32_t)(nt * RB));
  }
  __syncthreads();
  const int32_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;
  for (int i = tid; i < nt; i += kDecodeThreads) {
    const int tok = lo + i;
    const int64_t blk = bt_row[tok / p.block_size];
    const int64_t slot = tok % p.block_size;
    bulk_g2s(ks + i * RB, p.k + blk * p.sk0 + slot * p.sk1 + kh * p.sk2, RB, &bars[0]);
  }
  for (int i = tid; i < nt; i += kDecodeThreads) {
    const int tok = lo + i;
    const int64_t blk = bt_row[tok / p.block_size];
    const int64_t slot = tok % p.block_size;
    bulk_g2s(vs + i * RB, p.v + blk * p.sv0 + slot * p.sv1 + kh * p.sv2, RB, &bars[1]);
  }

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

  // ---- pass 1: scores ---------------------------------------------------------
  if (__syncthreads_or(!mbar_wait_bounded(&bars[0], 0))) return;
  // both 16-lane groups of a warp run the same trip count (full-warp shuffles)
  for (int wbase = (tid >> 5) * 2 * TQ; wbase < nt; wbase += 8 * TQ) {
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
    if (tok < nt) sc[(sub % GQA) * span + tok] = v[0];
  }
  __syncthreads();

  // ---- exact softmax statistics of the span, per head -----------------------
  const int warp = tid >> 5;
  for (int h = warp; h < GQA; h += kDecodeThreads / 32) {
    float m = -INFINITY;
    for (int t = lane; t < nt; t += 32) m = fmaxf(m, sc[h * span + t]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float e = exp2f(sc[h * span + t] - m);
      pt[t * GQA + h] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      stat_m[h] = m;
      stat_l[h] = l;
    }
  }
  __syncthreads();

  // ---- pass 2: o = sum_t p[t] * V[t] ---------------------------------------
  if (__syncthreads_or(!mbar_wait_bounded(&bars[1], 0))) return;
  float2 of[GQA][4];
#pragma unroll
  for (int h = 0; h < GQA; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) of[h][e] = make_float2(0.f, 0.f);
  for (int tok = grp; tok < nt; tok += 8) {
    float2 vf[4];
    Cvt::load8(vs + tok * RB + 8 * sub * (RB / kHeadDim), vf);
    float pw[GQA];
    if constexpr (GQA == 4) {
      const float4 p4 = *reinterpret_cast<const float4*>(pt + tok * 4);
      pw[0] = p4.x; pw[1] = p4.y; pw[2] = p4.z; pw[3] = p4.w;
    } else {
#pragma unroll
      for (int h = 0; h < GQA; ++h) pw[h] = pt[tok * GQA + h];
    }
#pragma unroll
    for (int h = 0; h < GQA; ++h) {
      const float2 pp = make_float2(pw[h], pw[h]);
#pragma unroll
      for (int e = 0; e < 4; ++e) of[h][e] = __ffma2_rn(pp, vf[e], of[h][e]);
    }
  }
  __syncthreads();  // K region is free now: reuse it for the group reduction
  float* red = reinterpret_cast<float*>(ks);  // [8 groups][GQA][128]
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
    float4* dst = reinterpret_cast<float4*>(red + (grp * GQA + h) * kHeadDim + 8 * sub);
    dst[0] = make_float4(of[h][0].x, of[h][0].y, of[h][1].x, of[h][1].y);
    dst[1] = make_float4(of[h][2].x, of[h][2].y, of[h][3].x, of[h][3].y);
  }
  __syncthreads();

  const int d = tid;  // kDecodeThreads == kHeadDim
  float o_acc[GQA];
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
    float s = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) s += red[(g * GQA + h) * kHeadDim + d];
    o_acc[h] = s;
  }
  const float vsc = FP8 ? __ldg(p.v_scale) : 1.f;

  if (nsplit == 1) {
#pragma unroll
    for (int h = 0; h < GQA; ++h)
      out_base[(int64_t)h * p.o_sh + d] = __float2bfloat16_rn(o_acc[h] * vsc / stat_l[h]);
    return;
  }

  // ---- split partials + last-arriver combine ---------------------------------
  const int64_t pair = (int64_t)seq * p.hkv + kh;
  const int64_t pbase = (pair * p.max_splits + sp) * GQA;
#pragma unroll
  for (int h = 0; h < GQA; ++h) p.part_o[(pbase + h) * kHeadDim + d] = o_acc[h];
  if (tid < GQA) {
    p.part_ml[(pbase + tid) * 2 + 0] = stat_m[tid];
    p.part_ml[(pbase + tid) * 2 + 1] = stat_l[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&p.counters[pair], 1);
    *flag = (old == nsplit - 1);
  }
  __syncthreads();
  if (!*flag) return;
  __threadfence();

  const int64_t pb0 = pair * p.max_splits * GQA;
  for (int h = warp; h < GQA; h += kDecodeThreads / 32) {
    float mg = -INFINITY;
    for (int s = lane; s < nsplit; s += 32) mg = fmaxf(mg, __ldcg(&p.part_ml[(pb0 + s * GQA + h) * 2]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, o));
    float lg = 0.f;
    for (int s = lane; s < nsplit; s += 32)
      lg += exp2f(__ldcg(&p.part_ml[(pb0 + s * GQA + h) * 2]) - mg) *
            __ldcg(&p.part_ml[(pb0 + s * GQA + h) * 2 + 1]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lg += __shfl_xor_sync(0xffffffffu, lg, o);
    if (lane == 0) {
      stat_m[h] = mg;
      stat_l[h] = lg;
    }
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
    const float mg = stat_m[h];
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s)
      acc += exp2f(__ldcg(&p.part_ml[(pb0 + s * GQA + h) * 2]) - mg) *
             __ldcg(&p.part_o[(pb0 + s * GQA + h) * kHeadDim + d]);
    out_base[(int64_t)h * p.o_sh + d] = __float2bfloat16_rn(acc * vsc / stat_l[h]);
  }
  if (tid == 0) p.counters[pair] = 0;  // ready for the next call
}

size_t decode_smem_bytes(int span, bool fp8, int gqa) {
  const int rb = fp8 ? kHeadDim : 2 * kHeadDim;
  return (size_t)kv_region_bytes(span, rb, gqa) + 2 * (size_t)gqa * span * sizeof(float) +
         16 * sizeof(float) + 2 * sizeof(uint64_t) + 16;
}

template <int GQA, bool FP8>
cudaError_t launch_decode(const DecodeParams& p, dim3 grid, cudaStream_t stream) {
  const size_t smem = decode_smem_bytes(p.span, FP8, GQA);
  cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<GQA, FP8>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  decode_attn_kernel<GQA, FP8><<<grid, kDecodeThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

// Split geometry shared by the workspace-size query and the launch.
struct DecodePlan {
  int span, max_splits;
  size_t off_counters, off_ml, off_o, total;
};

static int decode_plan(int num_seqs, int hq, int hkv, int block_size, int max_blocks, int hint,
                       int num_splits, DecodePlan* plan) {
  if (num_seqs <= 0 || hq <= 0 || hkv <= 0 || block_size <= 0 || max_blocks <= 0)
    return B200KV_ERR_INVALID_ARG;
  if (hq % hkv) return B200KV_ERR_INVALID_ARG;
  const int ctx = hint > 0 ? hint : max_blocks * block_size;
  int span;
  if (num_splits > 0) {
    span = cdiv(ctx, num_splits);
  } else {
    const int sms = num_sms_current_device() > 0 ? num_sms_current_device() : 148;
    const int pairs = num_seqs * hkv;
    const int splits = cdiv(4 * sms, pairs);
    span = cdiv(ctx, splits);
    if (span < 64) span = 64;
  }
  span = (span + 15) & ~15;
  if (span > kSpanMax) span = kSpanMax;
  if (span < 16) span = 16;
  plan->span = span;
  plan->max_splits = cdiv(ctx, span);
  const int gqa = hq / hkv;
  const size_t pairs = (size_t)num_seqs * hkv;
  plan->off_counters = 0;
  plan->off_ml = align_up(pairs * sizeof(int), 256);
  plan->off_o = plan->off_ml + align_up(pairs * plan->max_splits * gqa * 2 * sizeof(float), 256);
  plan->total = plan->off_o + align_up(pairs * plan->max_splits * gqa * kHeadDim * sizeof(float), 256);
  return B200KV_OK;
}

int decode_attn_workspace_size(int num_seqs, int hq, int hkv, int head_dim, int block_size,
                               int max_blocks, int hint, int num_splits, size_t* bytes) {
  if (!bytes) return B200KV_ERR_INVALID_ARG;
  if (head_dim != kHeadDim) return B200KV_ERR_UNSUPPORTED;
  DecodePlan plan;
  const int rc = decode_plan(num_seqs, hq, hkv, block_size, max_blocks, hint, num_splits, &plan);
  if (rc) return rc;
  *bytes = plan.total;
  return B200KV_OK;
}

int decode_attn_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                       const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                       int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                       const int32_t* qsl, const int32_t* seq_lens, const int32_t* bt,
                       int64_t bt_stride, const float* k_scale, const float* v_scale,
                       float sm_scale, int num_seqs, int hq, int hkv, int head_dim,
                       int block_size, int max_blocks, int hint, int kv_dtype, int out_by_qsl,
                       int num_splits, void* ws, size_t ws_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !out || !qsl || !seq_lens || !bt) return B200KV_ERR_INVALID_ARG;
  if (head_dim != kHeadDim) return B200KV_ERR_UNSUPPORTED;
  if (kv_dtype != B200KV_KV_FP8_E4M3 && kv_dtype != B200KV_KV_BF16) return B200KV_ERR_UNSUPPORTED;
  const bool fp8 = kv_dtype == B200KV_KV_FP8_E4M3;
  if (fp8 && (!k_scale || !v_scale)) return B200KV_ERR_INVALID_ARG;
  DecodePlan plan;
  int rc = decode_plan(num_seqs, hq, hkv, block_size, max_blocks, hint, num_splits, &plan);
  if (rc) return rc;
  const int gqa = hq / hkv;
  if (gqa != 1 && gqa != 2 && gqa != 4 && gqa != 8) return B200KV_ERR_UNSUPPORTED;
  if (!ws || ws_bytes < plan.total) return B200KV_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) & 255) return B200KV_ERR_MISALIGNED;
  const int esz = fp8 ? 1 : 2;
  // bulk copies need 16-byte aligned rows
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
  p.num_seqs = num_seqs;
  p.hkv = hkv;
  p.block_size = block_size;
  p.span = plan.span;
  p.max_splits = plan.max_splits;
  p.out_by_qsl = out_by_qsl;
  uint8_t* w = static_cast<uint8_t*>(ws);
  p.counters = reinterpret_cast<int*>(w + plan.off_counters);
  p.part_ml = reinterpret_cast<float*>(w + plan.off_ml);
  p.part_o = reinterpret_cast<float*>(w + plan.off_o);

  const dim3 grid(plan.max_splits, hkv, num_seqs);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (gqa * 2 + (fp8 ? 1 : 0)) {
    case 3: e = launch_decode<1, true>(p, grid, st); break;
    case 2: e = launch_decode<1, false>(p, grid, st); break;
    case 5: e = launch_decode<2, true>(p, grid, st); break;
    case 4: e = launch_decode<2, false>(p, grid, st); break;
    case 9: e = launch_decode<4, true>(p, grid, st); break;
    case 8: e = launch_decode<4, false>(p, grid, st); break;
    case 17: e = launch_decode<8, true>(p, grid, st); break;
    case 16: e = launch_decode<8, false>(p, grid, st); break;
    default: return B200KV_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
