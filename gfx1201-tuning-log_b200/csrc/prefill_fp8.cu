// fp8-e4m3 paged-KV causal prefill attention on 8-bit tcgen05 MMAs, sm_100a.
//
// Same contract as prefill_attn.cu (the reference kernel
// vllm-fp8kv/fp8kv_prefill.py:32-121 generalised to varlen batches): rows of a
// query tile pack (128 / GQA) tokens x GQA heads of one kv head, query position
// q0 + i sees keys 0 .. q0 + i, k_scale folds into the score scale (log2
// domain), v_scale scales the output.
//
// B200 design:
//  * The K and V pages are gathered by TMA straight from the paged cache: one
//    4-D tensor-map load per (page, kv head) brings that head's fp8 rows into a
//    128-byte-swizzled shared-memory tile, 128 / block_size loads per 128-key
//    tile, with no conversion pass and no copy through registers.
//  * Both products run as kind::f8f6f4 MMAs on e4m3 operands.  The bf16 query
//    is split once into two e4m3 terms, q ~= qh + ql (qh = q rounded to 4
//    significant bits after an exact per-row power-of-two prescale, ql = the
//    rest, which is exact for every element within 2^-9 of the row maximum),
//    and so is every probability tile, p ~= ph + pl; S = qh K^T + ql K^T and
//    O += ph V + pl V accumulate in tensor memory.  Each product so keeps an
//    8-bit significand, the precision of the reference's bf16 operands
//    (fp8kv_prefill.py:88,114), at the tensor cores' 8-bit rate: two 8-bit MMAs
//    take the time of one 16-bit MMA.
//  * A CTA owns TWO 128-row query tiles (A and B) of one (sequence, kv head)
//    and shares every K/V tile between them.  16 softmax warps form four
//    warpgroups, one per (query tile, half of the 128 score columns), one query
//    row per thread; the two halves of a row trade their partial maxima through
//    shared memory and a named barrier.  Warp 16 issues the TMA loads through a
//    2-stage K/V ring and warp 17 issues the MMAs from one thread, in the order
//    PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1), so the tensor core works on one
//    tile while the softmax of the other runs.  Tensor memory: S_A, S_B, O_A,
//    O_B = all 512 columns.
//  * The softmax reads its scores from tensor memory twice, 32 columns at a
//    time (max, then exp2 + split + store).  The exponentials run as f16x2
//    (one MUFU op per key pair) and the e4m3 split works on the f16 pairs with
//    integer and f16x2 ops.  Measured with ncu, the MUFU / conversion pipe is
//    what bounds this kernel (above 100 % of its sustained rate), ahead of the
//    tensor pipe.
//  * Lazy rescaling: a row's running max only moves when a tile's max exceeds
//    it by more than 2^4, so O is rarely read back and rescaled.  p is formed
//    times 2^4 (so p <= 2^8 fits e4m3, and the probabilities down to 2^-10
//    split into normal e4m3 terms); O and l carry the same factor and the same
//    stale max, which cancel in O / l.  Modelled on the CPU, this keeps the
//    error before the output's bf16 rounding at ~7e-3 on the reference's test
//    data (K, V ~ 2 N(0,1) in e4m3), against 5e-2 with p <= 1 unscaled.
//  * Keys past the sequence (the tail of the last page, and pages not loaded)
//    are masked in S and their V rows are zeroed before the P V products, so
//    stale or non-finite cache bytes never reach the output.
//  * Every wait is bounded; a timeout records kDevMbarrierTimeout and the CTA
//    drains its copies before it frees tensor memory and exits.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200kv {
namespace {

constexpr int kD = 128;       // head dim (= 128 fp8 bytes per row)
constexpr int kRows = 128;    // query rows per CTA
constexpr int kBN = 128;      // keys per KV tile
constexpr int kStages = 2;    // K/V ring depth
constexpr int kSoftWarps = 16;  // 4 warpgroups: (query tile A/B) x (column half 0/1)
constexpr int kThreads = (kSoftWarps + 2) * 32;  // + TMA warp + MMA warp
constexpr int kOp = kRows * 128;  // one 128 x 128 fp8 operand: 16 KB
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 4.f;  // rescale only when the max grows by > 2^4
constexpr float kPOff = 4.f;  // p is computed times 2^4 (<= 2^8 with kLazy)

// shared-memory map (offsets from a 1024-byte aligned base)
constexpr int kOffQ = 0;                          // [tile][qh, ql]
constexpr int kOffK = 4 * kOp;                    // K stages
constexpr int kOffV = kOffK + kStages * kOp;      // V stages
constexpr int kOffP = kOffV + kStages * kOp;      // [tile][ph, pl]
constexpr int kSmemBytes = kOffP + 4 * kOp;       // 192 KB

struct Fp8PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  const int32_t* cu_q;      // [NS+1] or null (single sequence)
  const int32_t* seq_lens;  // [NS] or null
  const int32_t* bt;
  int64_t bt_stride;
  const float* k_scale;
  const float* v_scale;
  float sm_scale;
  int pblk_shift;  // log2(block_size), block_size in {16, 32, 64, 128}
  int q0_single, qlen_single;
  int qpairs;      // gridDim.x: pairs of 128-row query tiles
  int only_multi;  // skip one-token sequences (the decode kernel's, in a mixed batch)
  int compact;     // the item index enumerates the (sequence, tile pair) items of the batch (gridDim.z = 1)
  int head_fast;   // grid (kv heads, items, z), else (items, kv heads, z)
  int num_seqs;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// (a, b) -> two e4m3 bytes, a in the low byte.
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// Split x into hi + lo with hi = x rounded to 4 significant bits (half away
// from zero on the magnitude; exact in e4m3 when |x| >= 2^-6) and lo = x - hi
// (exact in fp32, |lo| <= 2^-4 |x|), so hi + e4m3(lo) carries x to 2^-8.
__device__ __forceinline__ void split4(float x, float& hi, float& lo) {
  hi = __uint_as_float((__float_as_uint(x) + 0x00080000u) & 0xFFF00000u);
  lo = x - hi;
}

// 16 floats -> 16 e4m3 bytes of hi and of lo * LO_SCALE (element 0 in the
// lowest byte).
template <int LO_SCALE>
__device__ __forceinline__ void pack16(const float* v, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    float a0, a1, a2, a3, b0, b1, b2, b3;
    split4(v[4 * w + 0], a0, b0);
    split4(v[4 * w + 1], a1, b1);
    split4(v[4 * w + 2], a2, b2);
    split4(v[4 * w + 3], a3, b3);
    constexpr float ls = (float)LO_SCALE;
    h[w] = e4m3x2(a0, a1) | (e4m3x2(a2, a3) << 16);
    l[w] = e4m3x2(b0 * ls, b1 * ls) | (e4m3x2(b2 * ls, b3 * ls) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// (a, b) -> f16x2 with a in the low half
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// f16x2 -> two e4m3 bytes (low half in the low byte), in the low 16 bits
__device__ __forceinline__ uint32_t e4m3x2_h2(uint32_t x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(x));
  return (uint32_t)r;
}
__device__ __forceinline__ float h2_sum_f32(uint32_t x) {
  float a, b;
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.f32.f16 %0, l;\n cvt.f32.f16 %1, h;\n}"
      : "=f"(a), "=f"(b) : "r"(x));
  return a + b;
}

// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled [rows][128 B] tile
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

template <int GQA>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_fp8_kernel(const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const Fp8PrefillParams p) {
  constexpr int TPT = kRows / GQA;  // tokens per query tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ uint64_t kv_full[kStages], kv_empty[kStages];
  __shared__ uint64_t s_full[2], p_full[2], pv_done[2], q_full;
  __shared__ uint32_t tmem_slot;
  __shared__ float xch[2][2][2][128];  // [tile parity][query tile][column half][row]: row max, then l

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // The kv head is the fastest grid index (blockIdx.x), so the CTAs of one
  // (sequence, tile pair) item start together for every head and the longest
  // items run in the first waves; with the item fastest, the longest items of
  // the last heads were dispatched last and set the end of the call.  Beyond
  // 65535 items (the grid's y limit) the item is the fastest index.
  const int kh = p.head_fast ? blockIdx.x : blockIdx.y;
  const int item = p.head_fast ? blockIdx.y : blockIdx.x;
  int seq = blockIdx.z;
  int pair = p.qpairs - 1 - item;  // longest causal rows first
  if (p.compact) {
    // The grid holds about as many CTAs (per kv head) as the batch has tile
    // pairs, not sequences x the longest sequence's pairs: a mixed batch's
    // one-token sequences, and the short ones of a ragged batch, then cost no
    // CTA that only returns (those CTAs, one per SM at a time, had delayed the
    // real ones).  Warp 0 finds the item of this CTA: a scan of the
    // sequences' pair counts, 32 sequences at a time.
    __shared__ int s_item[2];
    if (warp == 0) {
      const int target = item;
      int base = 0, fseq = -1, fpair = 0;
      for (int s0 = 0; s0 < p.num_seqs && fseq < 0; s0 += 32) {
        const int s = s0 + lane;
        int cnt = 0;
        if (s < p.num_seqs) {
          const int ql = p.cu_q[s + 1] - p.cu_q[s];
          cnt = (ql <= 0 || (p.only_multi && ql == 1)) ? 0 : (ql + 2 * TPT - 1) / (2 * TPT);
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        if (target < base + total) {
          const unsigned hit = __ballot_sync(0xffffffffu, target >= base + incl - cnt && target < base + incl);
          const int src = __ffs(hit) - 1;
          const int first = base + __shfl_sync(0xffffffffu, incl - cnt, src);
          const int npairs = __shfl_sync(0xffffffffu, cnt, src);
          fseq = s0 + src;
          fpair = npairs - 1 - (target - first);  // longest causal rows first within a sequence
        }
        base += total;
      }
      if (lane == 0) {
        s_item[0] = fseq;
        s_item[1] = fpair;
      }
    }
    __syncthreads();
    seq = s_item[0];
    pair = s_item[1];
    if (seq < 0) return;  // past the batch's items (CTA-uniform)
  }

  const int qstart = p.cu_q ? p.cu_q[seq] : 0;
  const int qlen = p.cu_q ? p.cu_q[seq + 1] - qstart : p.qlen_single;
  const int kvlen = p.seq_lens ? p.seq_lens[seq] : p.q0_single + p.qlen_single;
  const int q0 = kvlen - qlen;
  const int t0 = pair * 2 * TPT;  // first token of tile A
  if (t0 >= qlen || qlen <= 0 || (p.only_multi && qlen == 1)) return;  // CTA-uniform
  const bool hasB = t0 + TPT < qlen;
  const int kvhiA = q0 + min(qlen, t0 + TPT);  // keys [0, kvhi) are visible to a tile
  const int kvhiB = hasB ? q0 + min(qlen, t0 + 2 * TPT) : kvhiA;
  const int nA = (kvhiA + kBN - 1) / kBN;
  const int nB = hasB ? (kvhiB + kBN - 1) / kBN : 0;
  const int kv_hi = kvhiB;                // of the CTA
  const int nmax = hasB ? nB : nA;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(&q_full, kSoftWarps);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_slot;  // S_A 0, S_B 128, O_A 256, O_B 384

  if (warp == kSoftWarps) {
    // ---------------- TMA producer (the whole warp) -------------------------------
    // Lane l holds the block id of page 32 w + l of the current window w of
    // the CTA's pages: one load per lane, where one dependent load per page
    // had put a global round trip before each page's copies; a tile's pages
    // never straddle two windows (pages per tile divide 32), and lane i of the
    // tile issues page i's two copies.
    const int32_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;
    const int pblk = 1 << p.pblk_shift;
    const int ppt = kBN >> p.pblk_shift;                 // pages per tile
    const int npg = (kv_hi + pblk - 1) >> p.pblk_shift;  // pages of the CTA
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int win = -1, ent = 0;
    int issued = nmax;
    for (int j = 0; j < nmax; ++j) {
      const int st = j % kStages;
      int ok = 1;
      if (lane == 0 && j >= kStages) ok = mbar_wait_bounded(&kv_empty[st], ((j / kStages) - 1) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) {  // stop issuing; drain what is in flight
        issued = j;
        break;
      }
      const int p0 = j * ppt;  // first page of tile j
      if ((p0 >> 5) != win) {
        win = p0 >> 5;
        const int pg = 32 * win + lane;
        ent = pg < npg ? __ldg(bt_row + pg) : 0;
      }
      const int keys = min(kBN, kv_hi - j * kBN);
      const int npages = (keys + pblk - 1) >> p.pblk_shift;
      if (lane == 0) mbar_arrive_expect_tx(&kv_full[st], (uint32_t)(npages * pblk * 128 * 2));
      __syncwarp();
      const int i = lane - (p0 & 31);
      if (i >= 0 && i < npages) {
        tma_load_4d(smem + kOffK + st * kOp + i * pblk * 128, &kmap, 0, kh, 0, ent, &kv_full[st]);
        tma_load_4d(smem + kOffV + st * kOp + i * pblk * 128, &vmap, 0, kh, 0, ent, &kv_full[st]);
      }
    }
    // drain: every load issued has landed before the CTA may exit
    if (lane == 0)
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait_bounded(&kv_full[j % kStages], (j / kStages) & 1);
    __syncwarp();
  } else if (warp == kSoftWarps + 1) {
    // ---------------- MMA issuer ------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t kIdescQK = tc::idesc_f16_f32(kRows, kBN, false);
      constexpr uint32_t kIdescPV = tc::idesc_f16_f32(kRows, kD, true);
      const uint32_t aQ = smem_u32(smem + kOffQ);
      const uint32_t aK = smem_u32(smem + kOffK);
      const uint32_t aV = smem_u32(smem + kOffV);
      const uint32_t aP = smem_u32(smem + kOffP);
      bool failed = !mbar_wait_bounded(&q_full, 0);
      tc::fence_after_sync();
      auto qk = [&](int X, int j) {  // S_X = Q_X K(j)^T
        const int st = j % kStages;
        if (!failed) failed = !mbar_wait_bounded(&kv_full[st], (j / kStages) & 1);
        if (failed) {  // issue nothing more; commit so the softmax warps do not wait
          tc::commit(&s_full[X]);
          return;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_f8(tbase + X * 128,
                       tc::sdesc_sw128(aQ + (2 * X + part) * kOp + ks * 32, 16, 1024),
                       tc::sdesc_sw128(aK + st * kOp + ks * 32, 16, 1024), kIdescQK,
                       (part | ks) != 0);
        tc::commit(&s_full[X]);
      };
      auto pv = [&](int X, int j) {  // O_X += P_X V(j)
        const int st = j % kStages;
        if (!failed) failed = !mbar_wait_bounded(&p_full[X], j & 1);
        if (failed) {
          tc::commit(&pv_done[X]);
          return;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_f8(tbase + 256 + X * 128,
                       tc::sdesc_sw128(aP + (2 * X + part) * kOp + ks * 32, 16, 1024),
                       tc::sdesc_sw128(aV + st * kOp + ks * 32 * 128, kOp, 1024), kIdescPV,
                       (j > 0 || part > 0 || ks > 0));
        tc::commit(&pv_done[X]);
      };
      qk(0, 0);
      if (hasB) qk(1, 0);
      for (int j = 0; j < nmax; ++j) {
        if (j < nA) {
          pv(0, j);
          if (j + 1 < nA) qk(0, j + 1);
        }
        if (j < nB) pv(1, j);
        tc::commit(&kv_empty[j % kStages]);
        if (j + 1 < nB) qk(1, j + 1);
      }
    }
  } else {
    // ---------------- softmax: warpgroup (X, H) owns columns 64H .. 64H+63 of the
    // score / output rows of query tile X; thread = row ----------------------------
    const int X = warp >> 3, H = (warp >> 2) & 1;
    const int row = tid & 127;
    const int bar_id = 1 + X;  // named barrier of the 8 warps of tile X
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tbase + X * 128 + 64 * H, tO = tbase + 256 + X * 128 + 64 * H;
    const int tX0 = t0 + X * TPT;
    const int tok = tX0 + row / GQA, g = row % GQA;
    const bool valid = tok < qlen;
    const int qpos = valid ? q0 + tok : 0x7FFFFFFF;  // padding rows see every key (finite)
    const int kvX = X ? kvhiB : kvhiA;
    const int nX = X ? nB : nA;

    // Q row -> per-row power-of-two prescale (max in [2^7, 2^8)) -> qh, ql; each
    // half loads its own 64 elements and the halves trade their maxima
    float score_c;
    {
      const __nv_bfloat16* qr = p.q + (int64_t)(qstart + (valid ? tok : 0)) * p.q_st +
                                (int64_t)(kh * GQA + g) * p.q_sh + 64 * H;
      uint4 raw[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        raw[i] = valid ? *reinterpret_cast<const uint4*>(qr + 8 * i) : make_uint4(0, 0, 0, 0);
      float mx = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(w[e] << 16)),
                               fabsf(__uint_as_float(w[e] & 0xFFFF0000u))));
      }
      xch[0][X][H][row] = mx;
      named_bar_sync(bar_id, 256);
      mx = fmaxf(mx, xch[0][X][H ^ 1][row]);
      named_bar_sync(bar_id, 256);  // both halves read before the slot is reused
      const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);
      int sh = (E == 0xFF || mx == 0.f) ? 0 : 134 - E;
      sh = max(-126, min(127, sh));
      const float up = __uint_as_float((uint32_t)(sh + 127) << 23);
      uint8_t* sQh = smem + kOffQ + (2 * X) * kOp;
      uint8_t* sQl = sQh + kOp;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {  // 16 elements per 16-byte chunk
        const int c = 4 * H + cc;
        float v[16];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 r4 = raw[2 * cc + h];
          const uint32_t w[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[8 * h + 2 * e] = __uint_as_float(w[e] << 16) * up;
            v[8 * h + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u) * up;
          }
        }
        uint4 hi, lo;
        pack16<1>(v, hi, lo);
        *reinterpret_cast<uint4*>(sQh + swz(row, c)) = hi;
        *reinterpret_cast<uint4*>(sQl + swz(row, c)) = lo;
      }
      score_c = p.sm_scale * __ldg(p.k_scale) * kLog2e * __uint_as_float((uint32_t)(127 - sh) << 23);
    }
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&q_full);

    float m_run = -INFINITY, l_half = 0.f;
    bool failed = false;
    uint8_t* sPh = smem + kOffP + (2 * X) * kOp;
    uint8_t* sPl = sPh + kOp;
    for (int j = 0; j < nX; ++j) {
      const int st = j % kStages;
      const int kbase = j * kBN;
      const int cbase = kbase + 64 * H;  // key of this half's first column
      if (!failed) failed = !mbar_wait_bounded(&s_full[X], j & 1);
      tc::fence_after_sync();
      const bool need_mask = (kbase + kBN - 1 > q0 + tX0) || (kbase + kBN > kvX);  // tile-uniform

      // pass 1: this half's row max (raw score units), exchanged with the other half
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c4 = 0; c4 < 2; ++c4) {
        float sv[32];
        tc::ld32_wait(tS + lane_off + 32 * c4, sv);
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kp = cbase + 32 * c4 + i;
            if (!(kp <= qpos && kp < kvX)) sv[i] = -INFINITY;
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], sv[i]);
      }
      const float pm = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      xch[j & 1][X][H][row] = pm;
      named_bar_sync(bar_id, 256);
      const float tmax = fmaxf(pm, xch[j & 1][X][H ^ 1][row]) * score_c;  // log2 units
      float alpha = 1.f;
      if (tmax > m_run + kLazy) {  // both halves take the same decision
        alpha = ex2(m_run - tmax);  // 0 on the first tile
        m_run = tmax;
      }
      // PV_X(j-1) done: the P buffer is free and O_X is stable
      if (j > 0 && !failed) failed = !mbar_wait_bounded(&pv_done[X], (j - 1) & 1);
      tc::fence_after_sync();

      // pass 2: p = 2^4 exp2(s c - m) in f16 (the argument rounded to f16, one
      // f16x2 exp2 per key pair), split in f16 into ph + pl, each converted to e4m3
      float psum = 0.f;
      const float moff = kPOff - m_run;
#pragma unroll 1
      for (int c4 = 0; c4 < 2; ++c4) {
        float sv[32];
        tc::ld32_wait(tS + lane_off + 32 * c4, sv);
        uint32_t acc2[4] = {0u, 0u, 0u, 0u};  // f16x2 partial sums
        uint32_t eh[16], el[16];                // e4m3 pairs (16-bit each)
#pragma unroll
        for (int pr = 0; pr < 16; ++pr) {
          float a = fmaf(sv[2 * pr], score_c, moff), b = fmaf(sv[2 * pr + 1], score_c, moff);
          if (need_mask) {
            const int kp = cbase + 32 * c4 + 2 * pr;
            if (!(kp <= qpos && kp < kvX)) a = -INFINITY;
            if (!(kp + 1 <= qpos && kp + 1 < kvX)) b = -INFINITY;
          }
          const uint32_t p2 = ex2_h2(pack_h2(a, b));
          acc2[pr & 3] = hadd2(acc2[pr & 3], p2);
          const uint32_t hi2 = (p2 + 0x00400040u) & 0xFF80FF80u;  // RN to 4 significant bits
          const uint32_t lo2 = hsub2(p2, hi2);                     // exact
          eh[pr] = e4m3x2_h2(hi2);
          el[pr] = e4m3x2_h2(lo2);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) psum += h2_sum_f32(acc2[q]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 hi = make_uint4(eh[8 * h + 0] | (eh[8 * h + 1] << 16), eh[8 * h + 2] | (eh[8 * h + 3] << 16),
                                      eh[8 * h + 4] | (eh[8 * h + 5] << 16), eh[8 * h + 6] | (eh[8 * h + 7] << 16));
          const uint4 lo = make_uint4(el[8 * h + 0] | (el[8 * h + 1] << 16), el[8 * h + 2] | (el[8 * h + 3] << 16),
                                      el[8 * h + 4] | (el[8 * h + 5] << 16), el[8 * h + 6] | (el[8 * h + 7] << 16));
          const int c = 4 * H + 2 * c4 + h;
          *reinterpret_cast<uint4*>(sPh + swz(row, c)) = hi;
          *reinterpret_cast<uint4*>(sPl + swz(row, c)) = lo;
        }
      }
      l_half = l_half * alpha + psum;

      // rescale this warp's O rows (this half's columns) when a row's max moved
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c4 = 0; c4 < 2; ++c4) {
          float o[32];
          tc::ld32_wait(tO + lane_off + 32 * c4, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tc::st32(tO + lane_off + 32 * c4, o);
        }
        tc::wait_st();
      }
      // last tile of the CTA: zero the V rows at or past its kv_hi (stale or
      // non-finite bytes); every warpgroup reading this tile writes the same zeros
      if (j == nmax - 1 && kbase + row >= kv_hi) {
        uint4* vr = reinterpret_cast<uint4*>(smem + kOffV + st * kOp + row * 128 + 64 * H);
#pragma unroll
        for (int c = 0; c < 4; ++c) vr[c] = make_uint4(0, 0, 0, 0);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[X]);
    }

    // ---- epilogue: O / l * v_scale -> bf16 (this half's 64 columns) -----------------
    if (nX > 0) {
      xch[nX & 1][X][H][row] = l_half;
      named_bar_sync(bar_id, 256);
      const float l_run = l_half + xch[nX & 1][X][H ^ 1][row];
      if (!failed) failed = !mbar_wait_bounded(&pv_done[X], (nX - 1) & 1);
      tc::fence_after_sync();
      const float inv = (l_run > 0.f) ? __ldg(p.v_scale) / l_run : 0.f;
      __nv_bfloat16* orow = p.out + (int64_t)(qstart + (valid ? tok : 0)) * p.o_st +
                            (int64_t)(kh * GQA + g) * p.o_sh + 64 * H;
#pragma unroll 1
      for (int c4 = 0; c4 < 2; ++c4) {
        float o[32];
        tc::ld32_wait(tO + lane_off + 32 * c4, o);
        if (valid && !failed) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 b =
                  __floats2bfloat162_rn(o[8 * q8 + 2 * e] * inv, o[8 * q8 + 2 * e + 1] * inv);
              w[e] = *reinterpret_cast<const uint32_t*>(&b);
            }
            *reinterpret_cast<uint4*>(orow + 32 * c4 + 8 * q8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, kTmemCols);
}

template <int GQA>
cudaError_t launch_fp8(const CUtensorMap& km, const CUtensorMap& vm, const Fp8PrefillParams& p,
                       int gx, int hkv, int gz, cudaStream_t st) {
  const size_t smem = (size_t)kSmemBytes + 1024;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_fp8_kernel<GQA>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const dim3 grid = p.head_fast ? dim3(hkv, gx, gz) : dim3(gx, hkv, gz);
  prefill_fp8_kernel<GQA><<<grid, kThreads, smem, st>>>(km, vm, p);
  return cudaGetLastError();
}

}  // namespace

// Returns a status code, or -1 when the call does not fit this path (the caller
// then takes the f16 path).  Arguments are validated by the caller.
int prefill_fp8_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                       const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                       int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                       const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                       const int32_t* block_table, int64_t bt_stride, const float* k_scale,
                       const float* v_scale, float sm_scale, int num_seqs, int qmax,
                       int q0_single, int qlen_single, int gqa, int hkv, int block_size,
                       int num_blocks, int only_multi, void* stream, int total_q) {
  if (block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128) return -1;
  if (num_blocks <= 0) return -1;
  CUtensorMap km, vm;
  if (!encode_paged_kv(&km, k_cache, kD, (uint32_t)hkv, (uint32_t)block_size, (uint64_t)num_blocks,
                       (uint64_t)sk2, (uint64_t)sk1, (uint64_t)sk0) ||
      !encode_paged_kv(&vm, v_cache, kD, (uint32_t)hkv, (uint32_t)block_size, (uint64_t)num_blocks,
                       (uint64_t)sv2, (uint64_t)sv1, (uint64_t)sv0))
    return -1;
  Fp8PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_st;
  p.q_sh = q_sh;
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
  p.pblk_shift = __builtin_ctz((unsigned)block_size);
  p.q0_single = q0_single;
  p.qlen_single = qlen_single;
  p.qpairs = cdiv(qmax, 2 * (kRows / gqa));
  p.only_multi = only_multi;
  p.num_seqs = num_seqs;
  // with the batch's token count known, the grid enumerates its tile pairs:
  // at most total / (2 tokens per tile x tiles) + one partial pair per sequence
  const int64_t dense = (int64_t)p.qpairs * num_seqs;
  const int64_t items = cu_seqlens_q && total_q > 0 ? cdiv(total_q, 2 * (kRows / gqa)) + (int64_t)num_seqs : dense;
  p.compact = items < dense && items <= 0x7fffffff;
  int grid_x = p.compact ? (int)items : p.qpairs, grid_z = p.compact ? 1 : num_seqs;
  p.head_fast = grid_x <= 65535;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (gqa) {
    case 1: e = launch_fp8<1>(km, vm, p, grid_x, hkv, grid_z, st); break;
    case 2: e = launch_fp8<2>(km, vm, p, grid_x, hkv, grid_z, st); break;
    case 4: e = launch_fp8<4>(km, vm, p, grid_x, hkv, grid_z, st); break;
    case 8: e = launch_fp8<8>(km, vm, p, grid_x, hkv, grid_z, st); break;
    default: return -1;
  }
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
