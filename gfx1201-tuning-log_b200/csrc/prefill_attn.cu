// fp8-KV (or bf16) paged causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory), sm_100a.
//
// Contract of the reference kernel vllm-fp8kv/fp8kv_prefill.py:32-121
// (_prefill_attn), generalised from one sequence to varlen batches:
//   * rows of a tile pack (128 / GQA) tokens x GQA query heads of one kv head
//     (fp8kv_prefill.py:46-50), so a K/V tile feeds all GQA heads at once;
//   * query position q0 + i attends keys 0 .. q0 + i (causal, continuation
//     chunks start at q0 = seq_len - qlen, fp8kv_prefill.py:179);
//   * k_scale is folded into the score scale in the log2 domain (exp2 softmax,
//     fp8kv_prefill.py:57-60) and v_scale is applied to the output (:117-118).
//
// B200 design:
//  * One CTA (4 warps) per (128-row query tile, kv head, sequence).  Q, K, V
//    and P live in shared memory as f16 in the tensor core's canonical
//    K-major / MN-major 128-byte-swizzled layouts; fp8 K/V rows are converted
//    to f16 exactly (hardware cvt) on the way in.  Q is converted from bf16 to
//    f16 with an exact per-row power-of-two prescale (undone in the score
//    scale), so no query value loses precision or overflows.
//  * S = Q K^T (M=128 rows, N=128 keys, K=128 dims) and O += P V (N=128 dims)
//    are tcgen05.mma kind::f16 instructions issued by one thread, with both
//    accumulators in tensor memory (256 of the SM's 512 columns); completion
//    is signalled through tcgen05.commit on an mbarrier.
//  * Softmax: thread t owns TMEM lane t (= query row t); it reads its score row
//    with tcgen05.ld, applies the causal mask, keeps the running max / sum,
//    writes P (f16, <= 1) back to shared memory for the P V MMA, and rescales
//    its O row in tensor memory only when its running max moved.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "tcgen05.cuh"

namespace b200kv {
namespace {

constexpr int kD = 128;        // head dim
constexpr int kRows = 128;     // query rows per CTA (tokens x GQA heads)
constexpr int kBN = 128;       // keys per KV tile
constexpr int kThreads = 128;
constexpr int kTile = kRows * kD * 2;  // one f16 128x128 operand: 32 KB
constexpr float kLog2e = 1.4426950408889634f;

struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  const uint8_t* k;
  const uint8_t* v;
  int64_t sk0, sk1, sk2, sv0, sv1, sv2;  // bytes
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  const int32_t* cu_q;      // [NS+1] or null (single sequence)
  const int32_t* seq_lens;  // [NS] or null
  const int32_t* bt;
  int64_t bt_stride;
  const float* k_scale;
  const float* v_scale;
  float sm_scale;
  int block_size, bs_shift;
  int q0_single, qlen_single;
  int only_multi;  // skip one-token sequences (the decode kernel's, in a mixed batch)
  int head_fast;   // grid (kv heads, query tiles, sequences), else (query tiles, kv heads, sequences)
};

// Byte offset of the 16-byte chunk `c16` (0..15) of row `r` of a 128 x 128 f16
// operand stored as two 64-column blocks [block][row][128 B], 128B-swizzled.
__device__ __forceinline__ uint32_t sw128_off(int r, int c16) {
  const int blk = c16 >> 3, ch = c16 & 7;
  return (uint32_t)(blk * (kRows * 128) + r * 128 + ((ch ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(r) : "r"(two_bytes));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}

// One cached K or V row (128 dims) -> f16 row r of a swizzled operand.
template <bool FP8>
__device__ __forceinline__ void stage_row(uint8_t* dst, int r, const uint8_t* src, bool ok) {
  if constexpr (FP8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // 16 fp8 -> 2 chunks of 8 f16
      uint4 raw = ok ? *reinterpret_cast<const uint4*>(src + 16 * i) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      uint4 lo, hi;
      lo.x = e4m3x2_to_f16x2(w[0] & 0xFFFFu);
      lo.y = e4m3x2_to_f16x2(w[0] >> 16);
      lo.z = e4m3x2_to_f16x2(w[1] & 0xFFFFu);
      lo.w = e4m3x2_to_f16x2(w[1] >> 16);
      hi.x = e4m3x2_to_f16x2(w[2] & 0xFFFFu);
      hi.y = e4m3x2_to_f16x2(w[2] >> 16);
      hi.z = e4m3x2_to_f16x2(w[3] & 0xFFFFu);
      hi.w = e4m3x2_to_f16x2(w[3] >> 16);
      *reinterpret_cast<uint4*>(dst + sw128_off(r, 2 * i)) = lo;
      *reinterpret_cast<uint4*>(dst + sw128_off(r, 2 * i + 1)) = hi;
    }
  } else {
    // bf16 caches: convert bf16 -> f16 (exact for |x| in f16's normal range;
    // bf16 KV caches are a debug mode of the reference, fp8kv_kernel.py K_FP8)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint4 raw = ok ? *reinterpret_cast<const uint4*>(src + 16 * i) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      uint4 o;
      uint32_t* op = &o.x;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        op[e] = pack_f16x2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xFFFF0000u));
      *reinterpret_cast<uint4*>(dst + sw128_off(r, i)) = o;
    }
  }
}

template <int GQA, bool FP8>
__global__ void __launch_bounds__(kThreads, 1) prefill_attn_kernel(const PrefillParams p) {
  constexpr int TPT = kRows / GQA;  // tokens per query tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTile;
  uint8_t* sV = smem + 2 * kTile;
  uint8_t* sP = smem + 3 * kTile;
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_slot;
  __shared__ int fail_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  // The kv head is the fastest grid index and query tiles go longest causal
  // rows first, so the longest tiles of every head start in the first waves
  // (at most 65535 query tiles, the grid's y limit; else the tile is fastest).
  const int seq = blockIdx.z;
  const int kh = p.head_fast ? blockIdx.x : blockIdx.y;
  const int qt = p.head_fast ? (int)(gridDim.y - 1 - blockIdx.y) : blockIdx.x;

  const int qstart = p.cu_q ? p.cu_q[seq] : 0;
  const int qlen = p.cu_q ? p.cu_q[seq + 1] - qstart : p.qlen_single;
  const int kvlen = p.seq_lens ? p.seq_lens[seq] : p.q0_single + p.qlen_single;
  const int q0 = kvlen - qlen;
  const int t0 = qt * TPT;
  if (t0 >= qlen || qlen <= 0 || (p.only_multi && qlen == 1)) return;  // CTA-uniform
  const int last_tok = min(qlen, t0 + TPT) - 1;
  const int kv_hi = q0 + last_tok + 1;  // keys [0, kv_hi) are visible to this tile
  const int ntiles = (kv_hi + kBN - 1) / kBN;

  // this thread's query row: token t0 + r / GQA, head kh*GQA + r % GQA
  const int tl = tid / GQA, g = tid % GQA;
  const int tok = t0 + tl;
  const bool valid = tok < qlen;
  const int qpos = valid ? q0 + tok : 0x7FFFFFFF;  // padding rows see every key (finite)

  if (tid == 0) {
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    fence_mbar_init();
    fail_flag = 0;
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, 256);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_slot;
  const uint32_t tS = tbase, tO = tbase + 128;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  // ---- Q row -> f16 with an exact per-row power-of-two prescale ------------
  float score_scale;
  {
    const __nv_bfloat16* qr = p.q + (int64_t)(qstart + (valid ? tok : 0)) * p.q_st +
                              (int64_t)(kh * GQA + g) * p.q_sh;
    uint4 raw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) raw[i] = valid ? *reinterpret_cast<const uint4*>(qr + 8 * i) : make_uint4(0, 0, 0, 0);
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(w[e] << 16)), fabsf(__uint_as_float(w[e] & 0xFFFF0000u))));
    }
    const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);
    int sh = (E == 0xFF || mx == 0.f) ? 0 : 131 - E;  // row max * 2^sh in [2^4, 2^5)
    sh = max(-126, min(127, sh));
    const float up = __uint_as_float((uint32_t)(sh + 127) << 23);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
      uint4 o;
      uint32_t* op = &o.x;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        op[e] = pack_f16x2(__uint_as_float(w[e] << 16) * up, __uint_as_float(w[e] & 0xFFFF0000u) * up);
      *reinterpret_cast<uint4*>(sQ + sw128_off(tid, i)) = o;
    }
    score_scale = p.sm_scale * (FP8 ? __ldg(p.k_scale) : 1.f) * kLog2e *
                  __uint_as_float((uint32_t)(127 - sh) << 23);
  }

  constexpr uint32_t kIdescQK = tc::idesc_f16_f32(kRows, kBN, false);
  constexpr uint32_t kIdescPV = tc::idesc_f16_f32(kRows, kD, true);
  const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
  const int32_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;

  float m_run = -INFINITY, l_run = 0.f;
  uint32_t ph_s = 0, ph_o = 0;
  bool failed = false;

  for (int j = 0; j < ntiles; ++j) {
    const int kbase = j * kBN;
    // ---- K, V rows of this tile -> f16 operands (thread = key row) ------------
    {
      const int key = kbase + tid;
      const bool ok = key < kv_hi;
      const uint8_t* ksrc = p.k;
      const uint8_t* vsrc = p.v;
      if (ok) {
        const int bi = p.bs_shift >= 0 ? key >> p.bs_shift : key / p.block_size;
        const int64_t slot = p.bs_shift >= 0 ? key & (p.block_size - 1) : key % p.block_size;
        const int64_t blk = bt_row[bi];
        ksrc = p.k + blk * p.sk0 + slot * p.sk1 + kh * p.sk2;
        vsrc = p.v + blk * p.sv0 + slot * p.sv1 + kh * p.sv2;
      }
      stage_row<FP8>(sK, tid, ksrc, ok);
      stage_row<FP8>(sV, tid, vsrc, ok);
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ---- S = Q K^T ----------------------------------------------------------------
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        const uint32_t off = (ks >> 2) * (kRows * 128) + (ks & 3) * 32;
        tc::mma_f16(tS, tc::sdesc_sw128(aQ + off, 16, 1024), tc::sdesc_sw128(aK + off, 16, 1024),
                    kIdescQK, ks > 0);
      }
      tc::commit(&bar_s);
    }
    if (!failed) failed = !mbar_wait_bounded(&bar_s, ph_s);
    ph_s ^= 1;
    tc::fence_after_sync();

    // ---- online softmax on this thread's row ----------------------------------
    float tmax = -INFINITY;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      float s[32];
      tc::ld32(tS + lane_off + 32 * c4, s);
      tc::wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int kp = kbase + 32 * c4 + i;
        if (kp <= qpos && kp < kv_hi) tmax = fmaxf(tmax, s[i] * score_scale);
      }
    }
    const float m_new = fmaxf(m_run, tmax);  // finite: key 0 is visible to every row
    const float alpha = exp2f(m_run - m_new);
    float psum = 0.f;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      float s[32];
      tc::ld32(tS + lane_off + 32 * c4, s);
      tc::wait_ld();
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float pv[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int i = 8 * q8 + 2 * e + h;
            const int kp = kbase + 32 * c4 + i;
            pv[h] = (kp <= qpos && kp < kv_hi) ? exp2f(s[i] * score_scale - m_new) : 0.f;
            psum += pv[h];
          }
          pk[e] = pack_f16x2(pv[0], pv[1]);
        }
        *reinterpret_cast<uint4*>(sP + sw128_off(tid, 4 * c4 + q8)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    l_run = l_run * alpha + psum;
    m_run = m_new;
    // rescale this row of O when its max moved (warp-collective TMEM access)
    if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        float o[32];
        tc::ld32(tO + lane_off + 32 * c4, o);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= alpha;
        tc::st32(tO + lane_off + 32 * c4, o);
      }
      tc::wait_st();
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ---- O += P V -------------------------------------------------------------------
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < kBN / 16; ++ks) {
        const uint32_t aoff = (ks >> 2) * (kRows * 128) + (ks & 3) * 32;  // P: K-major over keys
        const uint32_t boff = ks * 16 * 128;                               // V: 16 key rows
        tc::mma_f16(tO, tc::sdesc_sw128(aP + aoff, 16, 1024),
                    tc::sdesc_sw128(aV + boff, kRows * 128, 1024), kIdescPV, (j > 0 || ks > 0));
      }
      tc::commit(&bar_o);
    }
    if (!failed) failed = !mbar_wait_bounded(&bar_o, ph_o);
    ph_o ^= 1;
    tc::fence_after_sync();
  }

  // ---- epilogue: O / l * v_scale -> bf16 -------------------------------------------
  const float vsc = FP8 ? __ldg(p.v_scale) : 1.f;
  const float inv = (l_run > 0.f) ? vsc / l_run : 0.f;
  __nv_bfloat16* orow = p.out + (int64_t)(qstart + (valid ? tok : 0)) * p.o_st + (int64_t)(kh * GQA + g) * p.o_sh;
#pragma unroll
  for (int c4 = 0; c4 < 4; ++c4) {
    float o[32];
    tc::ld32(tO + lane_off + 32 * c4, o);
    tc::wait_ld();
    if (valid && !failed) {
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 b = __floats2bfloat162_rn(o[8 * q8 + 2 * e] * inv, o[8 * q8 + 2 * e + 1] * inv);
          w[e] = *reinterpret_cast<const uint32_t*>(&b);
        }
        *reinterpret_cast<uint4*>(orow + 32 * c4 + 8 * q8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

template <int GQA, bool FP8>
cudaError_t launch_prefill(const PrefillParams& p, int qtiles, int hkv, int ns, cudaStream_t st) {
  const size_t smem = 4 * (size_t)kTile + 1024;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<GQA, FP8>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const dim3 grid = p.head_fast ? dim3(hkv, qtiles, ns) : dim3(qtiles, hkv, ns);
  prefill_attn_kernel<GQA, FP8><<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

int prefill_fp8_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                       const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                       int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                       const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                       const int32_t* block_table, int64_t bt_stride, const float* k_scale,
                       const float* v_scale, float sm_scale, int num_seqs, int qmax,
                       int q0_single, int qlen_single, int gqa, int hkv, int block_size,
                       int num_blocks, int only_multi, void* stream, int total_q);

int prefill_attn_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                        const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                        int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                        const int32_t* block_table, int64_t bt_stride, const float* k_scale,
                        const float* v_scale, float sm_scale, int num_seqs, int max_qlen,
                        int q0_single, int qlen_single, int hq, int hkv, int head_dim,
                        int block_size, int num_blocks, int kv_dtype, int only_multi, void* stream,
                        int total_q) {
  if (!q || !k_cache || !v_cache || !out || !block_table) return B200KV_ERR_INVALID_ARG;
  if (num_seqs <= 0 || hq <= 0 || hkv <= 0 || block_size <= 0 || num_blocks < 0 || hq % hkv)
    return B200KV_ERR_INVALID_ARG;
  if ((cu_seqlens_q == nullptr) != (seq_lens == nullptr)) return B200KV_ERR_INVALID_ARG;
  if (!cu_seqlens_q && (num_seqs != 1 || qlen_single < 0 || q0_single < 0)) return B200KV_ERR_INVALID_ARG;
  if (head_dim != kD) return B200KV_ERR_UNSUPPORTED;
  if (kv_dtype != B200KV_KV_FP8_E4M3 && kv_dtype != B200KV_KV_BF16) return B200KV_ERR_UNSUPPORTED;
  const bool fp8 = kv_dtype == B200KV_KV_FP8_E4M3;
  if (fp8 && (!k_scale || !v_scale)) return B200KV_ERR_INVALID_ARG;
  const int gqa = hq / hkv;
  if (gqa != 1 && gqa != 2 && gqa != 4 && gqa != 8) return B200KV_ERR_UNSUPPORTED;
  const int esz = fp8 ? 1 : 2;
  const int64_t cs[6] = {sk0, sk1, sk2, sv0, sv1, sv2};
  for (int i = 0; i < 6; ++i)
    if ((cs[i] * esz) % 16) return B200KV_ERR_MISALIGNED;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
        reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) ||
      (q_st % 8) || (q_sh % 8) || (o_st % 8) || (o_sh % 8))
    return B200KV_ERR_MISALIGNED;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  const int qmax = cu_seqlens_q ? max_qlen : qlen_single;
  if (qmax <= 0) return B200KV_OK;
  if (fp8) {  // 8-bit tensor-core path with TMA page gathers (csrc/prefill_fp8.cu)
    const int r = prefill_fp8_launch(q, q_st, q_sh, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2,
                                     out, o_st, o_sh, cu_seqlens_q, seq_lens, block_table,
                                     bt_stride, k_scale, v_scale, sm_scale, num_seqs, qmax,
                                     q0_single, qlen_single, gqa, hkv, block_size, num_blocks,
                                     only_multi, stream, total_q);
    if (r >= 0) return r;
  }
  PrefillParams p;
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
  p.cu_q = cu_seqlens_q;
  p.seq_lens = seq_lens;
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.sm_scale = sm_scale;
  p.block_size = block_size;
  p.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz((unsigned)block_size) : -1;
  p.q0_single = q0_single;
  p.qlen_single = qlen_single;
  p.only_multi = only_multi;
  const int qtiles = cdiv(qmax, kRows / gqa);
  p.head_fast = qtiles <= 65535;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (gqa * 2 + (fp8 ? 1 : 0)) {
    case 3: e = launch_prefill<1, true>(p, qtiles, hkv, num_seqs, st); break;
    case 2: e = launch_prefill<1, false>(p, qtiles, hkv, num_seqs, st); break;
    case 5: e = launch_prefill<2, true>(p, qtiles, hkv, num_seqs, st); break;
    case 4: e = launch_prefill<2, false>(p, qtiles, hkv, num_seqs, st); break;
    case 9: e = launch_prefill<4, true>(p, qtiles, hkv, num_seqs, st); break;
    case 8: e = launch_prefill<4, false>(p, qtiles, hkv, num_seqs, st); break;
    case 17: e = launch_prefill<8, true>(p, qtiles, hkv, num_seqs, st); break;
    case 16: e = launch_prefill<8, false>(p, qtiles, hkv, num_seqs, st); break;
    default: return B200KV_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
