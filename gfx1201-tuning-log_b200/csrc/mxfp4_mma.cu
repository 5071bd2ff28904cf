// MXFP4 (e2m1 + e8m0) W4A16 matvec / skinny GEMM on block-scaled tcgen05 MMAs,
// sm_100a, 1 <= M <= 8.
//
// Same product as mxfp4_gemv.cu (the reference kernel h4mv/h4mv.cu:43-104):
//   out[m, n] = bf16_rn( sum_g 2^(S[n,g]-127) * sum_{j<32} e2m1(W[n,32g+j]) * x[m,32g+j] )
// with fp32 accumulation, computed by tcgen05.mma.kind::mxf8f6f4.block_scale.block32:
//  * A = a 128-row weight tile in e2m1, brought in by TMA from the packed
//    checkpoint layout and unpacked on the way into the tensor core's 4-bit
//    operand layout of this kind (16 codes per 16-byte chunk, 128-byte-swizzled
//    K-major rows of 128 k); the MMA applies the e8m0 weight scales itself.  A
//    stage issues up to 8 K-adjacent boxes back to back, so DRAM sees 128-512
//    contiguous bytes of every weight row per stage;
//  * B = the activations as two e4m3 terms with their own e8m0 scale per
//    32-element block (mxfp4_tc.cuh): exact for every bf16 element within 2^-13
//    of its block maximum, within 2^-21 of the block maximum below that.  Term
//    t of activation row m is B row 8 t + m (MMA N = 16), so one MMA computes
//    both products and the epilogue adds them;
//  * the weight scales come pre-packed (b200kv_mxfp4_pack_scales) in the
//    tensor core's 512-byte scale-factor atom per (128 rows x 128 k), copied to
//    tensor memory with tcgen05.cp -- a load-time repack, like the reference's
//    scale transpose (fp8kv_hipw4.py:32-43).
// One thread issues a block-scaled MMA about every 127 cycles whatever its N
// (measured on this part; two threads in different warps issue twice as many),
// and one MMA of K = 32 covers 2 KB of weights, which is slower than a fair
// share of HBM per SM: NI issuing warps (2 or 4) each take every NI-th box of
// a stage into an accumulator of their own, and the epilogue adds them.
// Work split: a thread-block cluster of ks CTAs splits K; clusters take 128-row
// tiles round-robin; each tile's partials are pushed (st.async into distributed
// shared memory) to one rank of the cluster, which adds them in a fixed order
// and stores the bf16 row, so no rank waits on a cluster-wide barrier at the
// end.  The kernel is launched with programmatic stream serialization: weights
// stream before it waits on the kernel that produces x.  Warp 0 streams
// (W boxes, scale atoms) stages through an mbarrier ring, warps 1..NI issue
// the MMAs, the last four warps turn x into its terms and drain the
// accumulators.
//
// Scale semantics are the MMA's (OCP MX: 2^(s-127)); the reference kernel
// differs for the bytes 0 (it gives 0.0) and 255 (inf), so weights holding those
// bytes stay on mxfp4_gemv.cu -- the packer reports them.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "b200kv.h"
#include "b200kv_common.cuh"
#include "mxfp4_tc.cuh"
#include "peer_comm.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200kv {
namespace {

constexpr int kTile = 128;           // weight rows per tile (MMA M)
constexpr int kStep = 128;           // K per W box and per scale atom (4 MMAs of K = 32)
constexpr int kBox = kTile * 128;    // W box in shared memory, unpacked: 16 KB
constexpr int kBoxTx = kTile * 64;   // bytes the TMA signals for it (the packed size)
constexpr int kAtom = mx::kAtom;
constexpr int kMaxM = 8;
constexpr int kNB = 16;              // B rows (MMA N): term t of activation row m is row 8 t + m
constexpr int kBBox = kNB * 128;     // B bytes per W box (K-major, 128-byte swizzle)
constexpr int kMaxStages = 4;
constexpr int kMaxSliceBoxes = 32;   // the x terms of a K-slice stay in shared memory
constexpr int kSmemMax = 227 * 1024;

// warp roles for NI issuing warps: 0 producer, 1..NI issuers, NI+1..NI+4 x split + epilogue
template <int NI>
struct Roles {
  static constexpr int kThreads = 32 * (NI + 5);
  static constexpr int kEw0 = NI + 1;
  // accumulator b of issuer i at tensor-memory column b * kDStride + 16 i (16 used)
  static constexpr int kDStride = NI * 16 < 32 ? 32 : NI * 16;
  static constexpr int kAtomCol = 2 * kDStride;  // scale atoms of the ring after the accumulators
};

// kEpiRopeKv: the qkv projection of a decode step with the rotary embedding
// and the paged KV-cache write as its epilogue (HF Llama, neox rotate_half,
// head_dim 128, fp8 e4m3 cache).  Tile i of the output is head i: q heads
// first, then k, then v.  q heads are rotated and stored; k heads are rotated
// and v heads taken as they are, both quantised (x / scale, satfinite, RN) into
// the cache slot of their token.
struct RopeKvArgs {
  const int32_t* pos;      // [M] token positions
  const float* cos_sin;    // [max_pos][128]: cos of the 64 frequencies, then sin
  int max_pos;
  const int64_t* slots;    // [M] cache slots (block * block_size + offset), < 0 skips
  uint8_t* kc;
  uint8_t* vc;
  int64_t sk0, sk1, sk2, sv0, sv1, sv2;  // bytes: block, slot in block, kv head
  const float* k_scale;
  const float* v_scale;
  int hq, hkv, block_size;
};

struct MmaArgs {
  const uint8_t* Sp;         // packed scale atoms [ntiles][K/128][512]
  const __nv_bfloat16* X;    // [M, K]
  __nv_bfloat16* Out;        // [M, N]
  int N, K, M;
  int nsteps;                // W boxes along K: K / 128
  int sps;                   // W boxes per K-slice
  int ntiles, nclusters, tmax, nstages, bps;
  int epilogue;              // kEpiStore: out[M, N]; kEpiSwiglu: out[M, N / 2]; kEpiAllreduce (below)
  PeerBufs peers;            // kEpiAllreduce: every rank's communication buffer (peer_comm.cuh)
  int rank, tp;
  RopeKvArgs rope;           // kEpiRopeKv
};

// Epilogues.  kEpiSwiglu takes gate_up weights whose 128-row tiles hold 64
// gate rows and then the 64 matching up rows (tile i: gate rows 64 i .. 64 i + 63,
// then the same up rows) and writes act[m, 64 i + r] = bf16(bf16(silu(g)) * u)
// with g, u the bf16-rounded products, HF Llama's act_fn(gate) * up with the
// rounding of b200kv_swiglu.
//
// kEpiAllreduce is the row-parallel product of tensor parallelism with its
// allreduce: every rank computes its [M, N] partial over its share of K, and
// as each 128-row tile is finished its bf16 partial goes straight into every
// rank's communication buffer (the line protocol of peer_comm.cuh, with one
// call counter per output tile), after which the same threads poll the
// local buffer for the other ranks' partials of that tile and store the sum
// in rank order -- bit for bit the plain product followed by the one-shot
// allreduce, without its launch, and with the transfer of a tile overlapping
// the products of the tiles still in flight.
constexpr int kEpiStore = 0, kEpiSwiglu = 1, kEpiAllreduce = 2, kEpiRopeKv = 3;

__device__ __forceinline__ uint8_t q8_e4m3(float v, float scale) {
  return (uint8_t)__nv_cvt_float_to_fp8(__fdiv_rn(v, scale), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Dynamic shared memory: the stage ring (a stage: bps W boxes, then their bps
// scale atoms), x's terms (B operand, one 2 KB box per W box of the slice) and
// their scale atoms, and the receive area of the K-slice reduction: tile i of
// a cluster is finished by rank i % ks, which receives every rank's partial of
// it in recv[i / ks][rank][row][m].
struct MmaLayout {
  int sps, tmax, nstages, ks, bps;
  __host__ __device__ int owned_max() const { return (tmax + ks - 1) / ks; }
  __host__ __device__ size_t stage() const { return (size_t)bps * (kBox + kAtom); }
  __host__ __device__ size_t xb() const { return (size_t)nstages * stage(); }
  __host__ __device__ size_t sfb() const { return xb() + (size_t)sps * kBBox; }
  __host__ __device__ size_t recv() const { return sfb() + (size_t)sps * kAtom; }
  __host__ __device__ size_t bytes(int m) const {
    return recv() + (size_t)owned_max() * ks * kTile * m * 4 + 1024;
  }
};

// tensor-memory columns: accumulators, then the A and B scale atoms of every
// (ring slot, box) pair
template <int NI>
__host__ __device__ constexpr int tmem_cols_needed(int nstages, int bps) {
  return Roles<NI>::kAtomCol + 8 * nstages * bps;
}

// x -> two e4m3 terms with an e8m0 scale per 32-element block, written as the
// B operand (term t of activation row m is B row 8 t + m of every box,
// 128-byte-swizzled K-major rows) and its scale atoms (byte 16 n + group).
// TPB threads share a block, EPT = 32 / TPB elements each; the next item's
// elements are loaded before the current one is converted.  B rows of absent
// activation rows are left as they are: they only reach accumulator columns
// the epilogue never reads.
template <int TPB>
__device__ __forceinline__ void split_terms(const MmaArgs& a, int et, int s_begin, int ns, uint8_t* xb,
                                            uint8_t* sfb) {
  constexpr int EPT = 32 / TPB;
  constexpr int NV = EPT / 8;  // 16-byte loads per item
  const int nblk = ns * 4;
  const int total = a.M * nblk * TPB;
  const int bound = (total + 31) & ~31;  // whole warps iterate together (shuffles)
  auto load = [&](int w, uint4 (&v)[NV]) {
    if (w < total) {
      const int q = w % TPB, wb = w / TPB;
      const int m = wb / nblk, blk = wb % nblk;
      const uint4* src = reinterpret_cast<const uint4*>(a.X + (size_t)m * a.K +
                                                        (size_t)(s_begin * kStep + blk * 32 + EPT * q));
#pragma unroll
      for (int i = 0; i < NV; ++i) v[i] = __ldg(src + i);
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i) v[i] = make_uint4(0, 0, 0, 0);
    }
  };
  uint4 cur[NV], nxt[NV];
  load(et, cur);
  for (int w = et; w < bound; w += 128) {
    load(w + 128, nxt);
    const bool live = w < total;
    const int q = w % TPB, wb = live ? w / TPB : 0;
    const int m = wb / nblk, blk = wb % nblk;
    const int j = blk >> 2, grp = blk & 3;
    float r[EPT];
#pragma unroll
    for (int i = 0; i < NV; ++i) mx::bf16x8_to_f32(cur[i], r + 8 * i);
    uint8_t* bj = xb + (size_t)j * kBBox;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      float mxv = 0.f;
#pragma unroll
      for (int e = 0; e < EPT; ++e) mxv = fmaxf(mxv, fabsf(r[e]));
#pragma unroll
      for (int o = 1; o < TPB; o <<= 1) mxv = fmaxf(mxv, __shfl_xor_sync(0xffffffffu, mxv, o));
      const int sb = mx::term_scale(mxv);
      uint32_t words[EPT / 4];
      mx::term_codes<EPT>(r, sb, words);
      if (live) {
        const int n = 8 * t + m;  // B row
        uint8_t* row = bj + n * 128;
        const int sw = n & 7;
        if constexpr (TPB == 1) {
          *reinterpret_cast<uint4*>(row + (((2 * grp) ^ sw) << 4)) = make_uint4(words[0], words[1], words[2], words[3]);
          *reinterpret_cast<uint4*>(row + (((2 * grp + 1) ^ sw) << 4)) =
              make_uint4(words[4], words[5], words[6], words[7]);
        } else if constexpr (TPB == 2) {
          *reinterpret_cast<uint4*>(row + (((2 * grp + q) ^ sw) << 4)) = make_uint4(words[0], words[1], words[2], words[3]);
        } else {
          *reinterpret_cast<uint2*>(row + (((2 * grp + (q >> 1)) ^ sw) << 4) + 8 * (q & 1)) =
              make_uint2(words[0], words[1]);
        }
        if (q == 0) sfb[(size_t)j * kAtom + 16 * n + grp] = (uint8_t)sb;  // rows < 32: byte 16 n + group
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) cur[i] = nxt[i];
  }
}

template <int NI, bool AR>
__global__ void __launch_bounds__(Roles<NI>::kThreads, 1)
    mxfp4_mma_kernel(const __grid_constant__ CUtensorMap wmap, const MmaArgs a) {
  using R = Roles<NI>;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages];
  __shared__ uint64_t d_full[2], d_free[2], x_ready, recv_bar;
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x;  // K-slice = rank in the cluster (cluster dims (ks, 1, 1))
  const int ksz = gridDim.x;
  const int cid = blockIdx.y;
  const int s_begin = rank * a.sps;
  const int ns = max(0, min(a.nsteps, s_begin + a.sps) - s_begin);  // W boxes in this slice
  const int bps = a.bps, nst = a.nstages;
  const int spt = (ns + bps - 1) / bps;                              // stages per tile
  const int my_tiles = cid < a.ntiles ? (a.ntiles - cid + a.nclusters - 1) / a.nclusters : 0;
  const int owned = my_tiles > rank ? (my_tiles - rank + ksz - 1) / ksz : 0;  // tiles i % ksz == rank
  const int nact = min(NI, min(ns, bps));  // issuers that get a box of every tile
  const MmaLayout L{a.sps, a.tmax, nst, ksz, bps};
  const size_t stage_bytes = L.stage();
  uint8_t* xb = dsm + L.xb();
  uint8_t* sfb = dsm + L.sfb();
  float* recv = reinterpret_cast<float*>(dsm + L.recv());  // [owned_max][ksz][128][M]
  const uint32_t recv_bytes = (uint32_t)(owned * (ksz - 1) * kTile * a.M * 4);
  const uint32_t tmem_cols = tmem_cols_needed<NI>(nst, bps) <= 256 ? 256 : 512;

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], max(nact, 1));
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&d_full[b], max(nact, 1));
      mbar_init(&d_free[b], 4);
    }
    mbar_init(&x_ready, 4);
    mbar_init(&recv_bar, 1);
    fence_mbar_init();
    if (recv_bytes) mbar_arrive_expect_tx(&recv_bar, recv_bytes);  // peers' pushes complete it
  }
  if (warp == 0) tc::tmem_alloc(&tmem_slot, tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_slot;
  if (ksz > 1) cluster_arrive_relaxed();  // recv_bar is initialised (peers wait before pushing)
  // The next kernel may launch now.  Weights and scale atoms are load-time
  // data, so the producer streams them before this grid waits on the previous
  // one; x is read, and the output written, only after griddep_wait().
  if (tid == 0) griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- producer: per stage up to bps (W box, its scale atom) ------------
    if (lane == 0 && ns > 0) {
      tma_prefetch_desc(&wmap);
      int s = 0;
      bool failed = false;
      for (int i = 0; i < my_tiles && !failed; ++i) {
        const int tile = cid + i * a.nclusters;
        for (int t = 0; t < spt; ++t, ++s) {
          const int slot = s % nst;
          if (s >= nst && !mbar_wait_bounded(&empty_bar[slot], ((s / nst) - 1) & 1)) {
            failed = true;  // stop issuing; drain what is in flight
            break;
          }
          uint8_t* st = dsm + (size_t)slot * stage_bytes;
          const int b0 = t * bps;
          const int nb = min(bps, ns - b0);
          const int g = s_begin + b0;  // first W box (along K) of this stage
          mbar_arrive_expect_tx(&full_bar[slot], (uint32_t)(nb * (kBoxTx + kAtom)));
          for (int q = 0; q < nb; ++q)  // adjacent K boxes back to back
            tma_load_2d(st + q * kBox, &wmap, (g + q) * kStep, tile * kTile, &full_bar[slot]);
          bulk_g2s(st + (size_t)bps * kBox, a.Sp + ((size_t)tile * a.nsteps + g) * kAtom, (uint32_t)(nb * kAtom),
                   &full_bar[slot]);
        }
      }
      // drain: every copy issued has landed before the CTA may exit
      for (int t = max(0, s - nst); t < s; ++t) mbar_wait_bounded(&full_bar[t % nst], (t / nst) & 1);
    }
  } else if (warp <= NI) {
    // ---------------- MMA issuers: issuer ii takes boxes q = ii, ii + NI, .. of a stage ----
    // A stage is "in" for an issuer once its bytes landed and the weight-scale
    // atoms of the issuer's boxes were copied to tensor memory.  Until x is
    // ready the issuer brings in the stages issued before this grid waited on
    // the previous kernel, so that afterwards only the MMAs remain.
    const int ii = warp - 1;
    if (lane == 0 && ii < nact) {
      const uint32_t a_ring = smem_u32(dsm), a_xb = smem_u32(xb), a_sfb = smem_u32(sfb);
      const int total = my_tiles * spt;  // stages of this CTA
      const uint32_t col_a = tbase + R::kAtomCol, col_b = col_a + 4 * nst * bps;
      bool failed = false;
      int s_in = 0;
      auto stage_in = [&](int s) {
        const int slot = s % nst;
        if (!mbar_wait_bounded(&full_bar[slot], (s / nst) & 1)) return false;
        const int nb = min(bps, ns - (s % spt) * bps);
        const uint32_t atoms = a_ring + (uint32_t)(slot * stage_bytes) + (uint32_t)bps * kBox;
        for (int q = ii; q < nb; q += NI)
          mx::tmem_cp_atom(col_a + 4 * (slot * bps + q), mx::sdesc_atom(atoms + (uint32_t)q * kAtom));
        return true;
      };
      bool xr = mbar_test(&x_ready, 0);
      while (!xr && !failed && s_in < min(total, nst)) {
        failed = !stage_in(s_in++);
        xr = mbar_test(&x_ready, 0);
      }
      if (!failed && !xr) failed = !mbar_wait_bounded(&x_ready, 0);
      tc::fence_after_sync();
      for (int s = 0; s < total && !failed; ++s) {
        const int i = s / spt, t = s % spt, b = i & 1;
        if (t == 0) {  // accumulator b is free once the epilogue drained tile i - 2
          if (i >= 2 && !mbar_wait_bounded(&d_free[b], ((i - 2) >> 1) & 1)) {
            failed = true;
            break;
          }
          tc::fence_after_sync();
        }
        if (s == s_in && !stage_in(s_in++)) {
          failed = true;  // issue nothing more
          break;
        }
        const int slot = s % nst;
        const uint32_t st = a_ring + (uint32_t)(slot * stage_bytes);
        const uint32_t tD = tbase + (uint32_t)(R::kDStride * b + 16 * ii);
        const int b0 = t * bps;
        const int nb = min(bps, ns - b0);
        for (int q = ii; q < nb; q += NI) {
          const uint32_t ta = col_a + 4 * (slot * bps + q), tb = col_b + 4 * (slot * bps + q);
          mx::tmem_cp_atom(tb, mx::sdesc_atom(a_sfb + (uint32_t)(b0 + q) * kAtom));
          const uint32_t abox = st + (uint32_t)q * kBox;
          const uint32_t bbox = a_xb + (uint32_t)(b0 + q) * kBBox;
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {  // K = 32 each; scale byte kq of the atoms
            const uint32_t sf = (uint32_t)kq;
            mx::mma_mxf8f6f4(tD, tc::sdesc_sw128(abox + kq * 32, 16, 1024), tc::sdesc_sw128(bbox + kq * 32, 16, 1024),
                             mx::idesc_mxf8f6f4(kTile, kNB, sf), (t > 0 || q > ii || kq > 0) ? 1u : 0u,
                             ta | (sf << 30), tb | (sf << 30));
          }
        }
        tc::commit(&empty_bar[slot]);
        if (t == spt - 1) tc::commit(&d_full[b]);
      }
    }
  } else {
    // ---------------- last four warps: x -> two e4m3 terms + scale atoms; epilogue ----------
    const int et = tid - 32 * R::kEw0;            // 0..127
    const int row = 32 * (warp & 3) + lane;       // tensor-memory lane of this thread
    griddep_wait();  // x is the previous kernel's output
    // 1, 2 or 4 threads per 32-element block of one activation row: the most
    // threads per block (shorter dependency chains, the block maximum reduced
    // across them) that still needs the fewest rounds of the 128 threads
    const int blocks = a.M * ns * 4;
    const int rounds1 = (blocks + 127) / 128;
    if ((4 * blocks + 127) / 128 == rounds1)
      split_terms<4>(a, et, s_begin, ns, xb, sfb);
    else if ((2 * blocks + 127) / 128 == rounds1)
      split_terms<2>(a, et, s_begin, ns, xb, sfb);
    else
      split_terms<1>(a, et, s_begin, ns, xb, sfb);
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&x_ready);

    // per tile: sum the issuers' accumulators and the two term columns of each
    // activation row and hand the partial to the tile's finishing rank
    // (i % ksz): its own receive slot, or a peer's through st.async counted on
    // the peer's recv_bar
    if (ksz > 1) cluster_wait();  // every peer's recv_bar is initialised
    const uint32_t rbar_local = smem_u32(&recv_bar);
    bool failed = false;
    for (int i = 0; i < my_tiles; ++i) {
      float v[kMaxM];
#pragma unroll
      for (int m = 0; m < kMaxM; ++m) v[m] = 0.f;
      if (ns > 0) {
        const int b = i & 1;
        if (!failed) failed = !mbar_wait_bounded(&d_full[b], (i >> 1) & 1);
        tc::fence_after_sync();
        const uint32_t tl = tbase + (uint32_t)(R::kDStride * b) + ((uint32_t)(32 * (warp & 3)) << 16);
#pragma unroll
        for (int h = 0; h < (NI + 1) / 2; ++h) {  // two accumulators per 32-column load
          float d[32];
          tc::ld32_wait(tl + 32 * h, d);
#pragma unroll
          for (int u = 0; u < 2; ++u)
            if (2 * h + u < nact)
#pragma unroll
              for (int m = 0; m < kMaxM; ++m) v[m] += d[16 * u + m] + d[16 * u + 8 + m];
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_free[b]);
      }
      const int owner = i % ksz;
      float* slot = recv + (((size_t)(i / ksz) * ksz + rank) * kTile + row) * a.M;
      if (owner == rank) {
#pragma unroll
        for (int m = 0; m < kMaxM; ++m)
          if (m < a.M) slot[m] = v[m];
      } else {
        const uint32_t raddr = map_to_rank(smem_u32(slot), owner);
        const uint32_t rbar = map_to_rank(rbar_local, owner);
#pragma unroll
        for (int m = 0; m < kMaxM; ++m)
          if (m < a.M) st_async_f32(raddr + 4 * m, v[m], rbar);
      }
    }

    // finish the owned tiles: fixed-order sum over the ranks' partials
    if (owned > 0) {
      bool ok = recv_bytes == 0 || mbar_wait_bounded(&recv_bar, 0);
      if (!AR && a.epilogue == kEpiStore) {
        for (int t = 0; ok && t < owned; ++t) {
          const int n = (cid + (rank + t * ksz) * a.nclusters) * kTile + row;
          const float* rs = recv + ((size_t)t * ksz * kTile + row) * a.M;
          for (int m = 0; m < a.M; ++m) {
            float acc = 0.f;
            for (int q = 0; q < ksz; ++q) acc += rs[(size_t)q * kTile * a.M + m];
            if (n < a.N) a.Out[(size_t)m * a.N + n] = __float2bfloat16_rn(acc);
          }
        }
      } else if constexpr (AR) {
        // lanes 2j and 2j + 1 hold output rows n and n + 1 of a tile: the even
        // lane sends the lines {out[m][n], out[m][n + 1]} of even m, the odd
        // lane those of odd m (line index (m N + n) / 2, the one-shot kernel's)
        const bool odd = (lane & 1) != 0;
        for (int t = 0; t < owned; ++t) {
          const int tile = cid + (rank + t * ksz) * a.nclusters;
          const int n = tile * kTile + row;
          const float* rs = recv + ((size_t)t * ksz * kTile + row) * a.M;
          volatile uint32_t* ctr = reinterpret_cast<volatile uint32_t*>(a.peers.p[a.rank]) + tile;
          const uint32_t call = *ctr;  // every thread reads it before the barrier below
          const uint32_t flag = call + 1;
          const int par = (int)(call & 1u);
          uint32_t mine[kMaxM];
#pragma unroll
          for (int m = 0; m < kMaxM; ++m) {
            float acc = 0.f;
            if (m < a.M)
              for (int q = 0; q < ksz; ++q) acc += rs[(size_t)q * kTile * a.M + m];
            mine[m] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc));
          }
          uint32_t data[kMaxM / 2];
#pragma unroll
          for (int m = 0; m < kMaxM; ++m) {
            const uint32_t other = __shfl_xor_sync(0xffffffffu, mine[m], 1);
            if ((m & 1) == (int)odd) data[m / 2] = odd ? (other | (mine[m] << 16)) : (mine[m] | (other << 16));
          }
          const int nl = (a.M + (odd ? 0 : 1)) / 2;  // lines of this lane: m = odd, odd + 2, ... < M
          for (int r = 0; r < a.tp; ++r) {
            uint2* dst = comm_lines(a.peers.p[r], par, a.rank);
#pragma unroll
            for (int j = 0; j < kMaxM / 2; ++j) {
              const int m = 2 * j + (odd ? 1 : 0);
              if (j < nl) comm_st_line(dst + ((size_t)m * a.N + (n & ~1)) / 2, data[j], flag);
            }
          }
          // poll the local buffer, line by line (a batched first load of every
          // (line, rank) took 161 registers and was slower: the CTA's footprint
          // matters more here than the round trips)
          uint8_t* own = a.peers.p[a.rank];
          bool late = false;
          for (int j = 0; j < nl; ++j) {
            const int m = 2 * j + (odd ? 1 : 0);
            const size_t li = ((size_t)m * a.N + (n & ~1)) / 2;
            float a0 = 0.f, a1 = 0.f;
            for (int r = 0; r < a.tp; ++r) {
              const uint2* l = comm_lines(own, par, r) + li;
              uint2 v = comm_ld_line(l);
              if (v.y != flag && !late) {
                const unsigned long long t0 = globaltimer_ns();
                while ((v = comm_ld_line(l)).y != flag) {
                  if (globaltimer_ns() - t0 > kCommTimeoutNs) {
                    atomicExch(&g_device_status, kDevPeerTimeout);
                    late = true;
                    break;
                  }
                }
              }
              a0 += __uint_as_float(v.x << 16);
              a1 += __uint_as_float(v.x & 0xFFFF0000u);
            }
            const __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
            *reinterpret_cast<__nv_bfloat162*>(a.Out + (size_t)m * a.N + (n & ~1)) = h;
          }
          named_bar_sync(1, 128);  // every thread has read the tile's counter
          if (row == 0) *ctr = flag;
        }
      } else if (a.epilogue == kEpiRopeKv) {
        // dims r and r + 64 of a head are a rotary pair: rows r and r + 64 of
        // its tile, the second written by another warp (one barrier of the four
        // epilogue warps, which also makes the decision to store uniform); the
        // sums and roundings are the plain store's, then b200kv_rope_kv_write's
        ok = named_bar_and(1, 128, ok);
        const RopeKvArgs& R = a.rope;
        const float ks = __ldg(R.k_scale), vs = __ldg(R.v_scale);
        for (int t = 0; ok && row < 64 && t < owned; ++t) {
          const int tile = cid + (rank + t * ksz) * a.nclusters;  // head
          const float* r1 = recv + ((size_t)t * ksz * kTile + row) * a.M;
          const float* r2 = r1 + (size_t)64 * a.M;
          for (int m = 0; m < a.M; ++m) {
            float s1 = 0.f, s2 = 0.f;
            for (int q = 0; q < ksz; ++q) {
              s1 += r1[(size_t)q * kTile * a.M + m];
              s2 += r2[(size_t)q * kTile * a.M + m];
            }
            const float x1 = round_bf(s1), x2 = round_bf(s2);
            const int64_t slot = R.slots[m];
            if (tile < R.hq + R.hkv) {
              const int pos = min(max(R.pos[m], 0), R.max_pos - 1);
              const float* cs = R.cos_sin + (size_t)pos * kTile;
              float y1, y2;
              rope_pair(x1, x2, cs[row], cs[64 + row], y1, y2);
              if (tile < R.hq) {
                a.Out[(size_t)m * a.N + tile * kTile + row] = __float2bfloat16_rn(y1);
                a.Out[(size_t)m * a.N + tile * kTile + 64 + row] = __float2bfloat16_rn(y2);
              } else if (slot >= 0) {
                uint8_t* dst = R.kc + (slot / R.block_size) * R.sk0 + (slot % R.block_size) * R.sk1 +
                               (int64_t)(tile - R.hq) * R.sk2;
                dst[row] = q8_e4m3(round_bf(y1), ks);
                dst[64 + row] = q8_e4m3(round_bf(y2), ks);
              }
            } else if (slot >= 0) {
              uint8_t* dst = R.vc + (slot / R.block_size) * R.sv0 + (slot % R.block_size) * R.sv1 +
                             (int64_t)(tile - R.hq - R.hkv) * R.sv2;
              dst[row] = q8_e4m3(x1, vs);
              dst[64 + row] = q8_e4m3(x2, vs);
            }
          }
        }
      } else {
        // the up row of gate row r is row r + 64 of the same tile, whose local
        // partial another warp wrote: one barrier of the four epilogue warps,
        // which also makes the decision to store uniform
        ok = named_bar_and(1, 128, ok);
        const int half = a.N / 2;
        for (int t = 0; ok && row < 64 && t < owned; ++t) {
          const int tile = cid + (rank + t * ksz) * a.nclusters;
          const float* rg = recv + ((size_t)t * ksz * kTile + row) * a.M;
          const float* ru = rg + (size_t)64 * a.M;
          for (int m = 0; m < a.M; ++m) {
            float g = 0.f, u = 0.f;
            for (int q = 0; q < ksz; ++q) {
              g += rg[(size_t)q * kTile * a.M + m];
              u += ru[(size_t)q * kTile * a.M + m];
            }
            const float gv = round_bf(g), uv = round_bf(u);
            const float sv = silu_bf16(gv);
            a.Out[(size_t)m * half + tile * 64 + row] = __float2bfloat16_rn(sv * uv);
          }
        }
      }
    }
  }

  griddep_wait();  // every thread waits before exit
  tc::fence_before_sync();
  __syncthreads();  // all tensor-memory reads are done
  if (warp == 0) tc::tmem_dealloc(tbase, tmem_cols);
}

// Scale packer: S (layout 0: [N, K/32] transposed, 1: [K/32, N] checkpoint) ->
// atoms [ntiles][K/128][512]; rows past N and groups past K/32 get 127 (2^0).
// *edge is set to 1 when any byte is 0 or 255.
__global__ void pack_scales_kernel(const uint8_t* __restrict__ S, int layout, uint8_t* __restrict__ Sp,
                                   int N, int K, int ntiles, int nsteps, int* edge) {
  const int ngroups = K >> 5;
  const size_t total = (size_t)ntiles * nsteps * kAtom;
  bool e = false;
  for (size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
    const int byte = (int)(o % kAtom);
    const size_t ts = o / kAtom;
    const int step = (int)(ts % nsteps), tile = (int)(ts / nsteps);
    const int dp = byte >> 4, jj = (byte >> 2) & 3, kb = byte & 3;
    const int n = tile * kTile + dp + 32 * jj;
    const int g = step * 4 + kb;
    uint8_t v = 127;
    if (n < N && g < ngroups) {
      v = layout == 0 ? S[(size_t)n * ngroups + g] : S[(size_t)g * N + n];
      e |= (v == 0 || v == 255);
    }
    Sp[o] = v;
  }
  if (e) atomicExch(edge, 1);
}

// The kernel's dynamic shared-memory limit, raised on demand (per process and
// instantiation; the attribute is per function, the same value on every device).
template <int NI, bool AR>
cudaError_t raise_smem_limit(size_t smem) {
  static std::mutex mu;
  static size_t limit = 0;
  std::lock_guard<std::mutex> g(mu);
  if (smem <= limit) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(mxfp4_mma_kernel<NI, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) limit = smem;
  return e;
}

template <int NI, bool AR>
cudaError_t launch_mma(const CUtensorMap& wm, const MmaArgs& a, int ks, cudaStream_t st) {
  const MmaLayout L{a.sps, a.tmax, a.nstages, ks, a.bps};
  const size_t smem = L.bytes(a.M);
  const cudaError_t e = raise_smem_limit<NI, AR>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, a.nclusters, 1);
  cfg.blockDim = dim3(Roles<NI>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, mxfp4_mma_kernel<NI, AR>, wm, a);
}

int env_or(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

// Clusters of ks CTAs with `smem` bytes each that the device can hold at once
// (cached per device, instantiation, size and smem).
template <int NI, bool AR>
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
  if (raise_smem_limit<NI, AR>(smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, 1, 1);
  cfg.blockDim = dim3(Roles<NI>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, mxfp4_mma_kernel<NI, AR>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

struct MmaPlan {
  int ks = 0, nst = 0, bps = 0, nc = 0;
};

// K-split ks (cluster size), boxes per stage, ring depth and cluster count.  The
// clusters are persistent: no more than can be resident at once (a cluster's
// CTAs must share a GPC), and the plan minimises the per-cluster work, tiles x
// boxes per slice, with a small price per CTA sharing an SM, per rank, and for
// rings that hold less than 64 KB of weights.  The ring holds at most what a
// CTA ever fills, so small shapes leave room for the next kernel's CTAs.
// Plans measured on B200 (148 SMs) for the 7B projections (qkv 6144 x 4096,
// o 4096 x 4096, gate_up 28672 x 4096, down 4096 x 14336) and their
// tensor-parallel shards over 2, 4 and 8 GPUs, at M = 1, 4 and 8: the fastest
// (K-split, boxes per stage, ring depth) of a sweep of all of them.  The
// cost model below misses what they show: a K-split that divides K evenly,
// deeper rings for gate_up, and fewer ranks as M grows (the cross-rank
// reduction carries M values per row).
struct PlanHint {
  int N, K, mb, ks, bps, nst;  // mb: 1 (M = 1..2), 4 (M = 3..5), 8 (M = 6..8)
};
constexpr PlanHint kHints[] = {
    {6144, 4096, 1, 4, 8, 1},   {4096, 4096, 1, 4, 8, 3},   {28672, 4096, 1, 4, 4, 3},  {4096, 14336, 1, 4, 4, 2},
    {3072, 4096, 1, 4, 8, 4},   {4096, 2048, 1, 2, 8, 2},   {14336, 4096, 1, 2, 4, 2},  {4096, 7168, 1, 4, 8, 1},
    {1536, 4096, 1, 5, 8, 4},   {4096, 1024, 1, 2, 4, 2},   {7168, 4096, 1, 4, 8, 1},   {4096, 3584, 1, 4, 8, 3},
    {4096, 512, 1, 2, 8, 3},    {3584, 4096, 1, 4, 8, 3},   {4096, 1792, 1, 2, 8, 1},
    {6144, 4096, 4, 4, 4, 2},   {4096, 4096, 4, 4, 8, 1},   {28672, 4096, 4, 2, 4, 2},  {4096, 14336, 4, 4, 4, 2},
    {6144, 4096, 8, 2, 8, 1},   {4096, 4096, 8, 4, 8, 1},   {28672, 4096, 8, 2, 4, 2},  {4096, 14336, 8, 4, 4, 2},
    {3072, 4096, 8, 4, 8, 4},   {4096, 2048, 8, 2, 8, 4},   {14336, 4096, 8, 2, 4, 2},  {4096, 7168, 8, 4, 8, 1},
    {1536, 4096, 8, 4, 8, 3},   {4096, 1024, 8, 2, 4, 2},   {7168, 4096, 8, 2, 8, 1},   {4096, 3584, 8, 4, 8, 2},
    {768, 4096, 8, 4, 8, 1},    {4096, 512, 8, 1, 8, 2},    {3584, 4096, 8, 4, 8, 2},   {4096, 1792, 8, 2, 8, 1},
};

const PlanHint* find_hint(int N, int K, int M) {
  const int want = M <= 2 ? 1 : (M <= 5 ? 4 : 8);
  const PlanHint* fallback = nullptr;
  for (const PlanHint& h : kHints) {
    if (h.N != N || h.K != K) continue;
    if (h.mb == want) return &h;
    if (want == 4 && h.mb == 8) fallback = &h;  // M = 3..5 without its own entry
  }
  return fallback;
}

template <int NI, bool AR>
MmaPlan plan_mma_forced(const MmaArgs& a, int sms, int force_ks, int force_st, int force_bps);

// The measured plan of the shape when there is one and it fits (more
// activation rows need more shared memory), else the cost model's.
template <int NI, bool AR>
MmaPlan plan_mma(const MmaArgs& a, int sms) {
  const int force_ks = env_or("B200KV_MMA_KSPLIT", 0);
  const int force_st = env_or("B200KV_MMA_STAGES", 0);
  const int force_bps = env_or("B200KV_MMA_BPS", 0);
  if (!force_ks && !force_st && !force_bps && env_or("B200KV_MMA_HINTS", 1)) {
    if (const PlanHint* h = find_hint(a.N, a.K, a.M)) {
      const MmaPlan p = plan_mma_forced<NI, AR>(a, sms, h->ks, h->nst, h->bps);
      if (p.ks) return p;
    }
  }
  return plan_mma_forced<NI, AR>(a, sms, force_ks, force_st, force_bps);
}

template <int NI, bool AR>
MmaPlan plan_mma_forced(const MmaArgs& a, int sms, int force_ks, int force_st, int force_bps) {
  // a footprint cap below half an SM lets the next kernel's CTAs share the SM
  // and start streaming while this one finishes
  const size_t smem_cap = (size_t)env_or("B200KV_MMA_SMEM_CAP", kSmemMax);
  MmaPlan best;
  double best_cost = 1e30;
  for (int ks = 1; ks <= 8; ++ks) {
    if (force_ks && ks != force_ks) continue;
    if (ks > a.nsteps) break;
    const int sps = cdiv(a.nsteps, ks);
    if (sps > kMaxSliceBoxes) continue;
    const int nc0 = max(1, min(a.ntiles, sms / ks));
    const int tslots = cdiv(a.ntiles, nc0) + 1;
    const int work = cdiv(a.ntiles, nc0) * sps;  // boxes a CTA streams (upper bound)
    for (int bps : {4, 8, 2}) {
      if (force_bps && bps != force_bps) continue;
      if (!force_bps && bps < NI && bps < sps) continue;  // an issuer would sit idle
      for (int nst0 = kMaxStages; nst0 >= 1; --nst0) {
        if (force_st && nst0 != force_st) continue;
        const int nst = min(nst0, cdiv(work, bps));
        if (nst * bps > 16) continue;  // 128 KB of weights in flight is plenty
        if (tmem_cols_needed<NI>(nst, bps) > 256) continue;
        const size_t smem = MmaLayout{sps, tslots, nst, ks, bps}.bytes(a.M);
        if (smem > std::min((size_t)kSmemMax, smem_cap)) continue;
        const int nc = min(a.ntiles, min(nc0, max_active_clusters<NI, AR>(ks, smem)));
        if (nc <= 0) continue;
        const int waves = cdiv(a.ntiles, nc);
        if (waves > tslots) continue;
        const int ctas = nc * ks;
        const double share = ctas > sms ? (double)ctas / sms : 1.0;
        // weights in flight per CTA below 64 KB (8 boxes) cost latency, and a
        // single-stage ring does not overlap copies with MMAs
        const int ring = nst * bps;  // boxes in flight
        const double latency = ring >= min(8, work) ? 0.0 : 2.0 * (min(8, work) - ring) / 8.0;
        const double cost = waves * sps * share + 0.25 * ks + latency + (nst == 1 && work > bps ? 1.0 : 0.0);
        if (cost < best_cost - 1e-9) {
          best_cost = cost;
          best.ks = ks;
          best.nst = nst;
          best.bps = bps;
          best.nc = nc;
        }
        break;  // the deepest ring that fits for this bps
      }
    }
  }
  return best;
}

template <int NI, bool AR>
int run_mma(const CUtensorMap& wm, MmaArgs a, int N, int K, int M, int sms, cudaStream_t st) {
  const MmaPlan p = plan_mma<NI, AR>(a, sms);
  if (p.ks == 0) return B200KV_ERR_UNSUPPORTED;
  a.nclusters = p.nc;
  a.sps = cdiv(a.nsteps, p.ks);
  a.tmax = cdiv(a.ntiles, a.nclusters);
  a.nstages = p.nst;
  a.bps = p.bps;
  if (env_or("B200KV_MMA_PLAN", 0))
    fprintf(stderr,
            "[b200kv] mxfp4_gemm N=%d K=%d M=%d: issuers=%d ks=%d clusters=%d stages=%d boxes/stage=%d "
            "tiles/cluster=%d boxes/slice=%d\n",
            N, K, M, NI, p.ks, a.nclusters, a.nstages, a.bps, a.tmax, a.sps);
  const cudaError_t e = launch_mma<NI, AR>(wm, a, p.ks, st);
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace

size_t mxfp4_packed_scales_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % kStep) return 0;
  return (size_t)cdiv(N, kTile) * (K / kStep) * kAtom;
}

int mxfp4_pack_scales_launch(const void* S, int layout, void* Sp, int N, int K, int* edge_flag,
                             void* stream) {
  if (!S || !Sp || !edge_flag || N <= 0 || K <= 0) return B200KV_ERR_INVALID_ARG;
  if (K % kStep) return B200KV_ERR_UNSUPPORTED;
  if (layout != 0 && layout != 1) return B200KV_ERR_INVALID_ARG;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  const int ntiles = cdiv(N, kTile), nsteps = K / kStep;
  const size_t total = (size_t)ntiles * nsteps * kAtom;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  pack_scales_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(S), layout, static_cast<uint8_t*>(Sp), N, K, ntiles, nsteps, edge_flag);
  return cudaGetLastError() == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

namespace {

int mma_launch(const void* W, const void* Sp, const void* X, void* Out, int N, int K, int M, int epilogue,
               void* stream, void* const* comm_bufs, int rank, int tp, const RopeKvArgs* rope) {
  if (!W || !Sp || !X || !Out) return B200KV_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || M <= 0) return B200KV_ERR_INVALID_ARG;
  if (epilogue != kEpiStore && epilogue != kEpiSwiglu && epilogue != kEpiAllreduce && epilogue != kEpiRopeKv)
    return B200KV_ERR_INVALID_ARG;
  if (epilogue == kEpiSwiglu && N % kTile) return B200KV_ERR_UNSUPPORTED;
  if (epilogue == kEpiRopeKv) {
    if (!rope) return B200KV_ERR_INVALID_ARG;
    if (N != (rope->hq + 2 * rope->hkv) * kTile) return B200KV_ERR_UNSUPPORTED;  // head_dim 128
  }
  PeerBufs pb = {};
  if (epilogue == kEpiAllreduce) {
    if (!comm_bufs || tp < 1 || tp > kCommMaxRanks || rank < 0 || rank >= tp) return B200KV_ERR_INVALID_ARG;
    for (int r = 0; r < tp; ++r) {
      if (!comm_bufs[r]) return B200KV_ERR_INVALID_ARG;
      pb.p[r] = static_cast<uint8_t*>(comm_bufs[r]);
    }
    // whole tiles (the line pairs and the per-tile counters), the partial within the line area
    if (N % kTile || N / kTile > kCommCounters || (size_t)M * N > (size_t)kCommMaxElems)
      return B200KV_ERR_UNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(Out) & 3) return B200KV_ERR_MISALIGNED;
  }
  if (M > kMaxM || K % kStep) return B200KV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(Sp) & 15) ||
      (reinterpret_cast<uintptr_t>(X) & 15))
    return B200KV_ERR_MISALIGNED;
  const int sms = num_sms_current_device();
  if (sms <= 0 || sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;

  MmaArgs a = {};
  a.Sp = static_cast<const uint8_t*>(Sp);
  a.X = static_cast<const __nv_bfloat16*>(X);
  a.Out = static_cast<__nv_bfloat16*>(Out);
  a.N = N;
  a.K = K;
  a.M = M;
  a.nsteps = K / kStep;
  a.ntiles = cdiv(N, kTile);
  a.epilogue = epilogue;
  a.peers = pb;
  a.rank = rank;
  a.tp = tp;
  if (rope) a.rope = *rope;

  CUtensorMap wm;
  if (!encode_e2m1_unpacked_2d(&wm, W, (uint64_t)K, (uint64_t)N, (uint64_t)(K / 2), kTile))
    return B200KV_ERR_UNSUPPORTED;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int ni = env_or("B200KV_MMA_ISSUERS", 4);
  // the allreduce epilogue is its own instantiation: its batched peer polls
  // take registers the other epilogues should not pay for
  if (epilogue == kEpiAllreduce) {
    if (ni == 1) return run_mma<1, true>(wm, a, N, K, M, sms, st);
    if (ni == 2) return run_mma<2, true>(wm, a, N, K, M, sms, st);
    return run_mma<4, true>(wm, a, N, K, M, sms, st);
  }
  if (ni == 1) return run_mma<1, false>(wm, a, N, K, M, sms, st);
  if (ni == 2) return run_mma<2, false>(wm, a, N, K, M, sms, st);
  return run_mma<4, false>(wm, a, N, K, M, sms, st);
}

}  // namespace

int mxfp4_mma_launch(const void* W, const void* Sp, const void* X, void* Out, int N, int K, int M,
                     int epilogue, void* stream, void* const* comm_bufs, int rank, int tp) {
  if (epilogue == kEpiRopeKv) return B200KV_ERR_INVALID_ARG;  // mxfp4_mma_rope_kv_launch
  return mma_launch(W, Sp, X, Out, N, K, M, epilogue, stream, comm_bufs, rank, tp, nullptr);
}

int mxfp4_mma_rope_kv_launch(const void* W, const void* Sp, const void* X, void* qkv, int N, int K, int M,
                             const int32_t* positions, const float* cos_sin, int max_pos,
                             const int64_t* slots, void* k_cache, void* v_cache, int64_t sk0, int64_t sk1,
                             int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, const float* k_scale,
                             const float* v_scale, int hq, int hkv, int block_size, int kv_dtype,
                             void* stream) {
  if (!positions || !cos_sin || !slots || !k_cache || !v_cache || !k_scale || !v_scale)
    return B200KV_ERR_INVALID_ARG;
  if (hq <= 0 || hkv <= 0 || block_size <= 0 || max_pos <= 0) return B200KV_ERR_INVALID_ARG;
  if (kv_dtype != B200KV_KV_FP8_E4M3) return B200KV_ERR_UNSUPPORTED;
  RopeKvArgs r;
  r.pos = positions;
  r.cos_sin = cos_sin;
  r.max_pos = max_pos;
  r.slots = slots;
  r.kc = static_cast<uint8_t*>(k_cache);
  r.vc = static_cast<uint8_t*>(v_cache);
  r.sk0 = sk0; r.sk1 = sk1; r.sk2 = sk2;
  r.sv0 = sv0; r.sv1 = sv1; r.sv2 = sv2;
  r.k_scale = k_scale;
  r.v_scale = v_scale;
  r.hq = hq;
  r.hkv = hkv;
  r.block_size = block_size;
  return mma_launch(W, Sp, X, qkv, N, K, M, kEpiRopeKv, stream, nullptr, 0, 1, &r);
}

}  // namespace b200kv
