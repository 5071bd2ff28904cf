// MXFP4 (e2m1 + e8m0) W4A16 matvec / skinny GEMM on block-scaled tcgen05 MMAs,
// sm_100a, 1 <= M <= 8.
//
// Same product as mxfp4_gemv.cu (the reference kernel h4mv/h4mv.cu:43-104):
//   out[m, n] = bf16_rn( sum_g 2^(S[n,g]-127) * sum_{j<32} e2m1(W[n,32g+j]) * x[m,32g+j] )
// with fp32 accumulation, computed by tcgen05.mma.kind::mxf4.block_scale.block32:
//  * A = a 128-row weight tile in packed e2m1 straight from memory: plain TMA
//    boxes of 128 rows x 128 bytes (256 k) land in the tensor core's 128-byte-
//    swizzled K-major layout unchanged (the checkpoint's low-nibble-first order
//    is the tensor core's), and the MMA applies the e8m0 group scales itself.
//    A stage issues 4 K-adjacent boxes back to back, so DRAM sees 512
//    contiguous bytes per row per stage: measured on this part, that streams at
//    6.3 TB/s where one 128-byte box per row and stage stays near 3.6 TB/s;
//  * B = the activations written as four e2m1 terms with their own e8m0
//    scales per 32-element block, x ~= t0 + t1 + t2 + t3, each term taking the
//    top 2-3 bits of what the previous ones left (greedy, round to nearest).
//    They sit in the N dimension (B row 8p + m = term p of activation row m),
//    so one MMA computes all four products and the epilogue adds them.  About
//    95 % of bf16 values come out exact; the worst case is 5e-4 of the block
//    maximum (modelled on config-2 data, where it moves the result by 1.4e-4 of
//    its maximum against the 5e-3 tolerance);
//  * the weight scales come pre-packed (b200kv_mxfp4_pack_scales) in the
//    tensor core's scale-factor atom: 512 bytes per (128 rows x 4 groups), byte
//    16*(row % 32) + 4*(row / 32) + group, copied to tensor memory with
//    tcgen05.cp 32x128b.warpx4 -- a load-time repack, like the reference's
//    scale transpose (fp8kv_hipw4.py:32-43).
// Packed 4-bit operands keep every TMA request at a full 128-byte row and every
// in-flight weight byte at one byte of shared memory (an unpacked 8-bit-container
// operand would halve both).  Work split: a thread-block cluster of ks CTAs
// splits K; clusters take 128-row tiles round-robin; each tile's partials are
// pushed (st.async into distributed shared memory) to one rank of the cluster,
// which adds them in a fixed order and stores the bf16 row, so no rank waits
// on a cluster-wide barrier at the end.  The kernel is launched with
// programmatic stream serialization: weights stream before it waits on the
// kernel that produces x.  Warp 0 streams (W box, 2 scale atoms)
// stages through an mbarrier ring, warp 1 issues the MMAs from one thread,
// warps 2-5 turn x into its four terms at the start and drain the accumulators.
//
// Scale semantics are the MMA's (OCP MX: 2^(s-127)); the reference kernel
// differs for the bytes 0 (it gives 0.0) and 255 (inf), so weights holding those
// bytes stay on mxfp4_gemv.cu -- the packer reports them.

#include <cuda.h>
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
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200kv {
namespace {

constexpr int kTile = 128;             // weight rows per tile (MMA M)
constexpr int kAtomK = 128;            // K covered by one scale atom (4 groups)
constexpr int kStep = 256;             // K per W box (128 B rows): 2 atoms, 4 MMAs
constexpr int kBoxesPerStage = 4;      // a stage reads 512 contiguous bytes of each row
constexpr int kTerms = 6;              // e2m1 terms of x
constexpr int kMaxM = 8;               // activation rows; term p of row m is B row S*p + m
// B rows (MMA N) for term stride S: kTerms * S rounded up to a multiple of 8
__host__ __device__ constexpr int nb_rows(int S) { return (kTerms * S + 7) / 8 * 8; }
// tensor-memory columns of one accumulator
__host__ __device__ constexpr int d_cols(int S) { return nb_rows(S) <= 32 ? 32 : 64; }
constexpr int kBox = kTile * 128;      // W box: 16 KB
constexpr int kAtom = 512;
constexpr int kStageBytes = kBoxesPerStage * (kBox + 2 * kAtom);  // 68 KB
constexpr int kMaxStages = 3;
constexpr int kThreads = 192;          // warp 0 TMA, warp 1 MMA, warps 2-5 x + epilogue
// tensor memory: D[2][DC] at 0 and DC (DC = d_cols(S)), A scales of ring slot r
// at 2 DC + 32 r, the activation scales at 2 DC + 32 nstages + 8 box; 256
// columns, or 512 when that does not fit (such CTAs no longer share an SM)
constexpr int kMaxSliceBoxes = 16;     // SFB of a K-slice stays in tensor memory: 8 columns a box

struct MmaArgs {
  const uint8_t* Sp;         // packed scale atoms [ntiles][K/128][512]
  const __nv_bfloat16* X;    // [M, K]
  __nv_bfloat16* Out;        // [M, N]
  int N, K, M;
  int nsteps;                // W boxes along K: K / 256
  int sps;                   // W boxes per K-slice
  int ntiles, nclusters, tmax, nstages;
};

// Dynamic shared memory: the stage ring, x's four terms (B operand), their
// scale atoms, and the receive area of the K-slice reduction: tile i of a
// cluster is finished by rank i % ks, which receives every rank's partial of it
// in recv[i / ks][rank][row][m].
struct MmaLayout {
  int sps, tmax, nstages, ks, S;  // S: B-row stride of the terms (M <= S, N = 4 S)
  __host__ __device__ int owned_max() const { return (tmax + ks - 1) / ks; }
  __host__ __device__ size_t xb() const { return (size_t)nstages * kStageBytes; }
  __host__ __device__ size_t sfb() const { return xb() + (size_t)sps * nb_rows(S) * 128; }
  __host__ __device__ size_t recv() const { return sfb() + (size_t)sps * 2 * kAtom; }
  __host__ __device__ size_t bytes(int m) const {
    return recv() + (size_t)owned_max() * ks * kTile * m * 4 + 1024;
  }
};



// instruction descriptor, kind::mxf4 block-scaled: A, B e2m1 (format 1 of this
// kind), both K-major, e8m0 scales, scale-factor byte ids (0 or 2: two bytes per MMA)
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N, uint32_t sf_id) {
  return (sf_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | (sf_id << 29);
}

// shared-memory descriptor of a 512-byte scale atom (32 rows x 16 B, no swizzle)
__device__ __forceinline__ uint64_t sdesc_atom(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16 >> 4) << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

__device__ __forceinline__ void tmem_cp_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void mma_mxf4(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t acc, uint32_t sfa, uint32_t sfb) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

// (a, b) -> one byte of two e2m1 codes, a in the low nibble
__device__ __forceinline__ uint32_t e2m1x2(float a, float b) {
  uint16_t r;
  asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n cvt.u16.u8 %0, t;\n}" : "=h"(r) : "f"(a), "f"(b));
  return (uint32_t)r;
}
// one byte of two e2m1 codes -> (low, high) values
__device__ __forceinline__ float2 e2m1x2_val(uint32_t byte) {
  uint32_t h;
  asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(h) : "r"(byte));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// x -> four e2m1 terms with e8m0 scales per 32-element block, written as the
// B operand (term t of activation row m is B row S*t + m, 128-byte-swizzled
// K-major rows, one 16-byte chunk per block) and its scale atoms.  TPB threads
// share a block, EPT = 32 / TPB elements each; the next item's elements are
// loaded before the current one is converted.  Term t of a block: residual
// maximum mx in [2^(E-127), 2^(E-126)) -> scale 2^(E-129), codes rounded to
// nearest (ties to even) and saturated at 6, residual -= code * scale.
template <int TPB, int S>
__device__ __forceinline__ void split_terms(const MmaArgs& a, int et, int s_begin, int ns,
                                            uint8_t* xb, uint8_t* sfb) {
  constexpr int EPT = 32 / TPB;
  constexpr int NV = EPT / 8;          // 16-byte loads per item
  constexpr uint32_t kBBox = nb_rows(S) * 128;
  const int nblk = ns * 8;
  const int total = a.M * nblk * TPB;
  const int bound = (total + 31) & ~31;  // whole warps iterate together (shuffles)
  auto load = [&](int w, uint4 (&v)[NV]) {
    if (w < total) {
      const int q = w % TPB, wb = w / TPB;
      const int m = wb / nblk, blk = wb % nblk;
      const uint4* src = reinterpret_cast<const uint4*>(
          a.X + (size_t)m * a.K + (size_t)(s_begin * kStep + blk * 32 + EPT * q));
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
    const int j = blk >> 3, kb8 = blk & 7;
    float r[EPT];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t u[4] = {cur[i].x, cur[i].y, cur[i].z, cur[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        r[8 * i + 2 * e] = __uint_as_float(u[e] << 16);
        r[8 * i + 2 * e + 1] = __uint_as_float(u[e] & 0xFFFF0000u);
      }
    }
    uint8_t* bj = xb + (size_t)j * kBBox;
#pragma unroll 1
    for (int t = 0; t < kTerms; ++t) {
      float mx = 0.f;
#pragma unroll
      for (int e = 0; e < EPT; ++e) mx = fmaxf(mx, fabsf(r[e]));
#pragma unroll
      for (int o = 1; o < TPB; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF);
      // term scale 2^(E-129): the block max maps into [4, 8) (6 is e2m1's top)
      const int sb = (mx == 0.f || E == 0xFF) ? 127 : max(E - 2, 1);
      const float inv = __uint_as_float((uint32_t)(254 - sb) << 23);  // 2^-(sb-127)
      const float scl = __uint_as_float((uint32_t)sb << 23);          // 2^(sb-127)
      uint32_t words[EPT / 8];
#pragma unroll
      for (int k = 0; k < EPT / 8; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * k + 2 * e;
          const uint32_t code = e2m1x2(r[i] * inv, r[i + 1] * inv);
          const float2 v = e2m1x2_val(code);
          r[i] = fmaf(-v.x, scl, r[i]);
          r[i + 1] = fmaf(-v.y, scl, r[i + 1]);
          word |= code << (8 * e);
        }
        words[k] = word;
      }
      if (live) {
        const int n = S * t + m;  // B row
        uint8_t* dst = bj + n * 128 + ((kb8 ^ (n & 7)) << 4) + (16 / TPB) * q;
        if constexpr (TPB == 1)
          *reinterpret_cast<uint4*>(dst) = make_uint4(words[0], words[1], words[2], words[3]);
        else if constexpr (TPB == 2)
          *reinterpret_cast<uint2*>(dst) = make_uint2(words[0], words[1]);
        else
          *reinterpret_cast<uint32_t*>(dst) = words[0];
        if (q == 0)  // scale-factor atom: byte 16 (n % 32) + 4 (n / 32) + group
          sfb[(size_t)(2 * j + (kb8 >> 2)) * kAtom + 16 * (n & 31) + 4 * (n >> 5) + (kb8 & 3)] = (uint8_t)sb;
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) cur[i] = nxt[i];
  }
}

// S = B-row stride of the activation terms: term p of activation row m is B
// row S*p + m, so the MMA's N is 4 S (8, 16 or 32 for M <= 2, 4, 8).
template <int S>
__global__ void __launch_bounds__(kThreads, 1)
    mxfp4_mma_kernel(const __grid_constant__ CUtensorMap wmap, const MmaArgs a) {
  constexpr int NB = nb_rows(S);            // MMA N
  constexpr int DC = d_cols(S);
  constexpr uint32_t kBBox = NB * 128;      // B bytes per W box (K-major, 128-byte swizzle)
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
  const int spt = (ns + kBoxesPerStage - 1) / kBoxesPerStage;       // stages per tile
  const int my_tiles = cid < a.ntiles ? (a.ntiles - cid + a.nclusters - 1) / a.nclusters : 0;
  const int owned = my_tiles > rank ? (my_tiles - rank + ksz - 1) / ksz : 0;  // tiles i % ksz == rank
  const MmaLayout L{a.sps, a.tmax, a.nstages, ksz, S};
  uint8_t* xb = dsm + L.xb();
  uint8_t* sfb = dsm + L.sfb();
  float* recv = reinterpret_cast<float*>(dsm + L.recv());  // [owned_max][ksz][128][M]
  const uint32_t recv_bytes = (uint32_t)(owned * (ksz - 1) * kTile * a.M * 4);
  const uint32_t tsfa_off = 2 * DC;
  const uint32_t tsfb_off = 2 * DC + 32 * a.nstages;
  const uint32_t tmem_cols = tsfb_off + 8 * a.sps <= 256 ? 256 : 512;

  if (tid == 0) {
    for (int i = 0; i < a.nstages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&d_full[b], 1);
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
    // ---------------- producer: per stage up to 4 (W box, its 2 scale atoms) -------------
    if (lane == 0 && ns > 0) {
      tma_prefetch_desc(&wmap);
      bool failed = false;
      int s = 0;
      const int atoms_per_tile = a.nsteps * 2;
      for (int i = 0; i < my_tiles && !failed; ++i) {
        const int tile = cid + i * a.nclusters;
        for (int t = 0; t < spt; ++t, ++s) {
          const int slot = s % a.nstages;
          if (s >= a.nstages && !mbar_wait_bounded(&empty_bar[slot], ((s / a.nstages) - 1) & 1)) {
            failed = true;  // stop issuing; drain what is in flight
            break;
          }
          uint8_t* st = dsm + (size_t)slot * kStageBytes;
          const int b0 = t * kBoxesPerStage;
          const int nb = min(kBoxesPerStage, ns - b0);
          const int g = s_begin + b0;  // first W box (along K) of this stage
          mbar_arrive_expect_tx(&full_bar[slot], (uint32_t)(nb * (kBox + 2 * kAtom)));
          for (int q = 0; q < nb; ++q)  // adjacent K boxes back to back: 512 B per row
            tma_load_2d(st + q * kBox, &wmap, (g + q) * (kStep / 2), tile * kTile, &full_bar[slot]);
          bulk_g2s(st + kBoxesPerStage * kBox, a.Sp + ((size_t)tile * atoms_per_tile + 2 * g) * kAtom,
                   (uint32_t)(nb * 2 * kAtom), &full_bar[slot]);
        }
      }
      // drain: every copy issued has landed before the CTA may exit
      for (int t = max(0, s - a.nstages); t < s; ++t)
        mbar_wait_bounded(&full_bar[t % a.nstages], (t / a.nstages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------------------------------------------
    // A stage is "in" once its bytes landed and its weight-scale atoms were copied
    // to tensor memory.  Until x is ready the issuer brings in the stages issued
    // before this grid waited on the previous kernel, so that afterwards only
    // the MMAs of those stages remain (an mbarrier wait and the atom copies cost
    // about as much issue time as the MMAs themselves).
    if (lane == 0 && ns > 0) {
      const uint32_t a_ring = smem_u32(dsm), a_xb = smem_u32(xb), a_sfb = smem_u32(sfb);
      const uint32_t tsfb = tbase + tsfb_off;  // the activation scales: all boxes of the slice
      const int total = my_tiles * spt;       // stages of this CTA
      bool failed = false;
      int s_in = 0;
      auto stage_in = [&](int s) {
        const int slot = s % a.nstages;
        if (!mbar_wait_bounded(&full_bar[slot], (s / a.nstages) & 1)) return false;
        const int nb = min(kBoxesPerStage, ns - (s % spt) * kBoxesPerStage);
        const uint32_t atoms = a_ring + (uint32_t)slot * kStageBytes + kBoxesPerStage * kBox;
        const uint32_t tsfa = tbase + tsfa_off + 32 * slot;
        for (int q = 0; q < 2 * nb; ++q) tmem_cp_atom(tsfa + 4 * q, sdesc_atom(atoms + (uint32_t)q * kAtom));
        return true;
      };
      bool xr = mbar_test(&x_ready, 0);
      while (!xr && !failed && s_in < min(total, a.nstages)) {
        failed = !stage_in(s_in++);
        xr = mbar_test(&x_ready, 0);
      }
      if (!failed && !xr) failed = !mbar_wait_bounded(&x_ready, 0);
      tc::fence_after_sync();
      if (!failed)
        for (int q = 0; q < 2 * ns; ++q) tmem_cp_atom(tsfb + 4 * q, sdesc_atom(a_sfb + (uint32_t)q * kAtom));
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
        const int slot = s % a.nstages;
        const uint32_t tsfa = tbase + tsfa_off + 32 * slot;
        const uint32_t st = a_ring + (uint32_t)slot * kStageBytes;
        const uint32_t tD = tbase + DC * b;
        const int b0 = t * kBoxesPerStage;
        const int nb = min(kBoxesPerStage, ns - b0);
        for (int q = 0; q < nb; ++q) {
          const uint32_t abox = st + (uint32_t)q * kBox;
          const uint32_t bbox = a_xb + (uint32_t)(b0 + q) * kBBox;
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {  // K = 64 each; scale bytes 2(kq&1).. of atom kq/2
            const uint32_t sf = 2u * (uint32_t)(kq & 1);
            mma_mxf4(tD, tc::sdesc_sw128(abox + kq * 32, 16, 1024),
                     tc::sdesc_sw128(bbox + kq * 32, 16, 1024), idesc_mxf4(kTile, NB, sf),
                     (t > 0 || q > 0 || kq > 0) ? 1u : 0u,
                     (tsfa + 8 * q + 4 * (kq >> 1)) | (sf << 30),
                     (tsfb + 8 * (b0 + q) + 4 * (kq >> 1)) | (sf << 30));
          }
        }
        tc::commit(&empty_bar[slot]);
        if (t == spt - 1) tc::commit(&d_full[b]);
      }
    }
  } else {
    // ---------------- warps 2-5: x -> 4 e2m1 terms + scale atoms; epilogue ----------
    const int et = tid - 64;                      // 0..127
    const int row = 32 * (warp & 3) + lane;       // TMEM lane of this thread
    // zero the B rows (rows of absent activation rows stay zero); scales 2^0
    for (int i = et; i < ns * (int)kBBox / 16; i += 128)
      reinterpret_cast<uint4*>(xb)[i] = make_uint4(0, 0, 0, 0);
    for (int i = et; i < ns * 2 * kAtom / 4; i += 128)
      reinterpret_cast<uint32_t*>(sfb)[i] = 0x7F7F7F7Fu;
    named_bar_sync(1, 128);
    griddep_wait();  // x is the previous kernel's output
    // 1, 2 or 4 threads per 32-element block of one activation row: the most
    // threads per block (shorter dependency chains, the block maximum reduced
    // across them) that still needs the fewest rounds of the 128 threads
    const int blocks = a.M * ns * 8;
    const int rounds1 = (blocks + 127) / 128;
    if ((4 * blocks + 127) / 128 == rounds1)
      split_terms<4, S>(a, et, s_begin, ns, xb, sfb);
    else if ((2 * blocks + 127) / 128 == rounds1)
      split_terms<2, S>(a, et, s_begin, ns, xb, sfb);
    else
      split_terms<1, S>(a, et, s_begin, ns, xb, sfb);
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&x_ready);

    // per tile: sum the four term columns of each activation row and hand the
    // partial to the tile's finishing rank (i % ksz): its own receive slot, or a
    // peer's through st.async counted on the peer's recv_bar
    if (ksz > 1) cluster_wait();  // every peer's recv_bar is initialised
    const uint32_t rbar_local = smem_u32(&recv_bar);
    bool failed = false;
    for (int i = 0; i < my_tiles; ++i) {
      float v[S];
#pragma unroll
      for (int m = 0; m < S; ++m) v[m] = 0.f;
      if (ns > 0) {
        const int b = i & 1;
        if (!failed) failed = !mbar_wait_bounded(&d_full[b], (i >> 1) & 1);
        tc::fence_after_sync();
        float d0[32], d1[32];
        const uint32_t tl = tbase + DC * b + ((uint32_t)(32 * (warp & 3)) << 16);
        tc::ld32_wait(tl, d0);
        if constexpr (DC == 64) tc::ld32_wait(tl + 32, d1);
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_free[b]);
#pragma unroll
        for (int m = 0; m < S; ++m) {
          float acc = 0.f;
#pragma unroll
          for (int t = 0; t < kTerms; ++t) acc += S * t + m < 32 ? d0[S * t + m] : d1[S * t + m - 32];
          v[m] = acc;
        }
      }
      const int owner = i % ksz;
      float* slot = recv + (((size_t)(i / ksz) * ksz + rank) * kTile + row) * a.M;
      if (owner == rank) {
#pragma unroll
        for (int m = 0; m < S; ++m)
          if (m < a.M) slot[m] = v[m];
      } else {
        const uint32_t raddr = map_to_rank(smem_u32(slot), owner);
        const uint32_t rbar = map_to_rank(rbar_local, owner);
#pragma unroll
        for (int m = 0; m < S; ++m)
          if (m < a.M) st_async_f32(raddr + 4 * m, v[m], rbar);
      }
    }

    // finish the owned tiles: fixed-order sum over the ranks' partials
    griddep_wait();  // before any output store
    if (owned > 0 && (recv_bytes == 0 || mbar_wait_bounded(&recv_bar, 0))) {
      for (int t = 0; t < owned; ++t) {
        const int n = (cid + (rank + t * ksz) * a.nclusters) * kTile + row;
        const float* rs = recv + ((size_t)t * ksz * kTile + row) * a.M;
        for (int m = 0; m < a.M; ++m) {
          float acc = 0.f;
          for (int q = 0; q < ksz; ++q) acc += rs[(size_t)q * kTile * a.M + m];
          if (n < a.N) a.Out[(size_t)m * a.N + n] = __float2bfloat16_rn(acc);
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
// atoms [ntiles][nsteps][512]; rows past N and groups past K/32 get 127 (2^0).
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
template <int S>
cudaError_t raise_smem_limit(size_t smem) {
  static std::mutex mu;
  static size_t limit = 0;
  std::lock_guard<std::mutex> g(mu);
  if (smem <= limit) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(mxfp4_mma_kernel<S>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) limit = smem;
  return e;
}

template <int S>
cudaError_t launch_mma(const CUtensorMap& wm, const MmaArgs& a, int ks, cudaStream_t st) {
  const MmaLayout L{a.sps, a.tmax, a.nstages, ks, S};
  const size_t smem = L.bytes(a.M);
  const cudaError_t e = raise_smem_limit<S>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, a.nclusters, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
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
  return cudaLaunchKernelEx(&cfg, mxfp4_mma_kernel<S>, wm, a);
}

int env_or(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

// Clusters of ks CTAs with `smem` bytes each that the device can hold at once
// (cached per device, size and smem).
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
  if (raise_smem_limit<kMaxM>(smem) != cudaSuccess) {
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
  if (cudaOccupancyMaxActiveClusters(&n, mxfp4_mma_kernel<kMaxM>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

}  // namespace

size_t mxfp4_packed_scales_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % kAtomK) return 0;
  return (size_t)cdiv(N, kTile) * (K / kAtomK) * kAtom;
}

int mxfp4_pack_scales_launch(const void* S, int layout, void* Sp, int N, int K, int* edge_flag,
                             void* stream) {
  if (!S || !Sp || !edge_flag || N <= 0 || K <= 0) return B200KV_ERR_INVALID_ARG;
  if (K % kAtomK) return B200KV_ERR_UNSUPPORTED;
  if (layout != 0 && layout != 1) return B200KV_ERR_INVALID_ARG;
  if (sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;
  const int ntiles = cdiv(N, kTile), nsteps = K / kAtomK;
  const size_t total = (size_t)ntiles * nsteps * kAtom;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  pack_scales_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(S), layout, static_cast<uint8_t*>(Sp), N, K, ntiles, nsteps, edge_flag);
  return cudaGetLastError() == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

int mxfp4_mma_launch(const void* W, const void* Sp, const void* X, void* Out, int N, int K, int M,
                     void* stream) {
  if (!W || !Sp || !X || !Out) return B200KV_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || M <= 0) return B200KV_ERR_INVALID_ARG;
  if (M > kMaxM || K % kStep) return B200KV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(Sp) & 15) ||
      (reinterpret_cast<uintptr_t>(X) & 15))
    return B200KV_ERR_MISALIGNED;
  const int sms = num_sms_current_device();
  if (sms <= 0 || sm_major_current_device() < 10) return B200KV_ERR_NO_DEVICE;

  MmaArgs a;
  a.Sp = static_cast<const uint8_t*>(Sp);
  a.X = static_cast<const __nv_bfloat16*>(X);
  a.Out = static_cast<__nv_bfloat16*>(Out);
  a.N = N;
  a.K = K;
  a.M = M;
  a.nsteps = K / kStep;
  a.ntiles = cdiv(N, kTile);
  // K-split ks (cluster size), ring depth and cluster count.  The clusters are
  // persistent: no more than can be resident at once (a cluster's CTAs must
  // share a GPC, so fewer clusters than SMs / ks fit when a CTA fills an SM),
  // and the plan minimises the per-cluster work, tiles x steps per slice.
  const int force_ks = env_or("B200KV_MMA_KSPLIT", 0);
  const int force_st = env_or("B200KV_MMA_STAGES", 0);
  const int S = M <= 2 ? 2 : (M <= 4 ? 4 : 8);  // term stride: N = 4 S
  int best_ks = 1, best_st = 4, best_nc = 1;
  double best_cost = 1e30;
  for (int ks = 1; ks <= 8; ++ks) {
    if (force_ks && ks != force_ks) continue;
    if (ks > a.nsteps) break;
    const int sps = cdiv(a.nsteps, ks);
    for (int nst0 : {2, 3}) {
      if (force_st && nst0 != force_st) continue;
      const int nc0 = max(1, min(a.ntiles, sms / ks));
      const int tslots = cdiv(a.ntiles, nc0) + 1;
      if (sps > kMaxSliceBoxes) continue;
      // no more ring stages than a CTA ever fills (a small footprint lets the
      // next kernel's CTAs share the SM and start streaming early)
      const int nst = min(nst0, cdiv(a.ntiles, nc0) * cdiv(sps, kBoxesPerStage));
      const size_t smem = MmaLayout{sps, tslots, nst, ks, S}.bytes(M);
      if (smem > 227 * 1024) continue;
      const int nc = min(a.ntiles, min(nc0, max_active_clusters(ks, smem)));
      if (nc <= 0) continue;
      const int waves = cdiv(a.ntiles, nc);
      if (waves > tslots) continue;
      // per-cluster work, plus a small price per CTA sharing an SM and per rank
      const int ctas = nc * ks;
      const double share = ctas > sms ? (double)ctas / sms : 1.0;
      const double cost = waves * sps * share + 0.25 * ks;
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best_ks = ks;
        best_st = nst;
        best_nc = nc;
      }
    }
  }
  if (best_cost >= 1e30) return B200KV_ERR_UNSUPPORTED;
  const int ks = best_ks;
  a.nclusters = best_nc;
  a.sps = cdiv(a.nsteps, ks);
  a.tmax = cdiv(a.ntiles, a.nclusters);
  a.nstages = best_st;
  if (env_or("B200KV_MMA_PLAN", 0))
    fprintf(stderr, "[b200kv] mxfp4_gemm N=%d K=%d M=%d: ks=%d clusters=%d stages=%d tiles/cluster=%d steps/slice=%d\n",
            N, K, M, ks, a.nclusters, a.nstages, a.tmax, a.sps);

  CUtensorMap wm;
  if (!encode_u8_2d(&wm, W, (uint64_t)(K / 2), (uint64_t)N, (uint64_t)(K / 2), 128, kTile, true))
    return B200KV_ERR_UNSUPPORTED;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = S == 2 ? launch_mma<2>(wm, a, ks, st)
                               : (S == 4 ? launch_mma<4>(wm, a, ks, st) : launch_mma<8>(wm, a, ks, st));
  return e == cudaSuccess ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
