// The element-wise steps of a decoder layer around the hot path, for the 7B
// decode loop (HF Llama semantics, the model family of the reference's
// benchmarks): residual add + RMSNorm, rotary embedding of q and k fused with
// the paged fp8 KV write, and the SwiGLU activation.  All HBM/latency-bound
// one-pass kernels, launched with programmatic stream serialization like the
// hot-path kernels (inputs read after griddep_wait()).

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace b200kv {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float bf(uint32_t w, int hi) {
  return __uint_as_float(hi ? (w & 0xFFFF0000u) : (w << 16));
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float round_bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// h <- bf16(h + delta) (when delta is given); x = w * bf16(h * rsqrt(mean(h^2) + eps))
// (HF LlamaRMSNorm: statistics in fp32, normalised value rounded to the model
// dtype before the weight multiply).  One CTA per row, 8 elements per 16-byte
// access, hidden % 8 == 0 and hidden <= 8 * 8 * kNormThreads.  The norm
// weight is load-time data: it is read before this grid waits on the previous
// kernel, so that load leaves the critical path.
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_residual_kernel(__nv_bfloat16* h, const __nv_bfloat16* delta, const __nv_bfloat16* w,
                            __nv_bfloat16* x, int hidden, float eps) {
  __shared__ float red[kNormThreads / 32];
  if (threadIdx.x == 0) griddep_launch_dependents();
  const int row = blockIdx.x;
  const int nv = hidden / 8;
  constexpr int kMaxV = 8;  // vectors per thread
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4 wvs[kMaxV];
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    wvs[j] = i < nv ? __ldg(wr + i) : make_uint4(0, 0, 0, 0);
  }
  griddep_wait();
  uint4* hr = reinterpret_cast<uint4*>(h + (size_t)row * hidden);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + (size_t)row * hidden) : nullptr;
  uint4 hv[kMaxV];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nv) {
      uint4 v = hr[i];
      if (dr) {
        const uint4 d = dr[i];
        const uint32_t a[4] = {v.x, v.y, v.z, v.w}, b[4] = {d.x, d.y, d.z, d.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = pack_bf2(bf(a[e], 0) + bf(b[e], 0), bf(a[e], 1) + bf(b[e], 1));
        v = make_uint4(o[0], o[1], o[2], o[3]);
        hr[i] = v;
      }
      hv[j] = v;
      const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) ss += bf(a[e], 0) * bf(a[e], 0) + bf(a[e], 1) * bf(a[e], 1);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)hidden + eps);
  uint4* xr = reinterpret_cast<uint4*>(x + (size_t)row * hidden);
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nv) {
      const uint4 v = hv[j], wv = wvs[j];
      const uint32_t a[4] = {v.x, v.y, v.z, v.w}, b[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = pack_bf2(round_bf(bf(a[e], 0) * r) * bf(b[e], 0), round_bf(bf(a[e], 1) * r) * bf(b[e], 1));
      xr[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

struct RopeKvParams {
  __nv_bfloat16* qkv;
  int64_t qkv_st;          // elements between tokens
  const int32_t* pos;
  const float* cos_sin;    // [max_pos][head_dim]: cos of the d/2 frequencies, then sin
  int max_pos;
  const int64_t* slots;
  uint8_t* kc;
  uint8_t* vc;
  int64_t sk0, sk1, sk2, sv0, sv1, sv2;  // bytes
  const float* k_scale;
  const float* v_scale;
  int hq, hkv, d, block_size;
};

// Neox-style rotary embedding (rotate the two halves of each head, as HF
// Llama's rotate_half) of every q and k head of one token, in fp32 from bf16,
// one rounding; q is written back in place, k and v go to the paged cache
// (fp8: cvt.rn.satfinite.e4m3(x / scale), as the KV write).  One CTA per token.
template <bool FP8>
__global__ void __launch_bounds__(256) rope_kv_write_kernel(const RopeKvParams p) {
  if (threadIdx.x == 0) griddep_launch_dependents();
  griddep_wait();
  const int t = blockIdx.x;
  const int half = p.d / 2;
  const int pos = min(max(p.pos[t], 0), p.max_pos - 1);
  const float* cs = p.cos_sin + (size_t)pos * p.d;
  __nv_bfloat16* row = p.qkv + (size_t)t * p.qkv_st;
  const int64_t slot = p.slots[t];
  const int64_t blk = slot >= 0 ? slot / p.block_size : 0;
  const int64_t off = slot >= 0 ? slot % p.block_size : 0;
  const float ks = FP8 ? __ldg(p.k_scale) : 1.f;
  const float vs = FP8 ? __ldg(p.v_scale) : 1.f;
  // rotary pairs of q and k heads
  const int pairs = (p.hq + p.hkv) * half;
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int head = i / half, j = i - head * half;
    __nv_bfloat16* hp = row + (size_t)head * p.d;
    const float x1 = __bfloat162float(hp[j]), x2 = __bfloat162float(hp[j + half]);
    float y1, y2;
    rope_pair(x1, x2, cs[j], cs[half + j], y1, y2);
    if (head < p.hq) {
      hp[j] = __float2bfloat16_rn(y1);
      hp[j + half] = __float2bfloat16_rn(y2);
    } else if (slot >= 0) {
      const int kh = head - p.hq;
      uint8_t* dst = p.kc + blk * p.sk0 + off * p.sk1 + kh * p.sk2;
      if constexpr (FP8) {
        dst[j] = __nv_cvt_float_to_fp8(__fdiv_rn(round_bf(y1), ks), __NV_SATFINITE, __NV_E4M3);
        dst[j + half] = __nv_cvt_float_to_fp8(__fdiv_rn(round_bf(y2), ks), __NV_SATFINITE, __NV_E4M3);
      } else {
        reinterpret_cast<__nv_bfloat16*>(dst)[j] = __float2bfloat16_rn(y1);
        reinterpret_cast<__nv_bfloat16*>(dst)[j + half] = __float2bfloat16_rn(y2);
      }
    }
  }
  // v rows straight to the cache
  if (slot >= 0) {
    const __nv_bfloat16* vrow = row + (size_t)(p.hq + p.hkv) * p.d;
    for (int i = threadIdx.x; i < p.hkv * p.d; i += blockDim.x) {
      const int vh = i / p.d, e = i - vh * p.d;
      uint8_t* dst = p.vc + blk * p.sv0 + off * p.sv1 + vh * p.sv2;
      if constexpr (FP8)
        dst[e] = __nv_cvt_float_to_fp8(__fdiv_rn(__bfloat162float(vrow[i]), vs), __NV_SATFINITE, __NV_E4M3);
      else
        reinterpret_cast<__nv_bfloat16*>(dst)[e] = vrow[i];
    }
  }
}

// act[r, i] = bf16(bf16(silu(g)) * u) with g = gate_up[r, i], u = gate_up[r, inter + i]
// (HF: act_fn(gate) * up in the model dtype).  Two elements per thread.
__global__ void __launch_bounds__(256)
    swiglu_kernel(const __nv_bfloat16* gu, __nv_bfloat16* act, int rows, int inter) {
  if (threadIdx.x == 0) griddep_launch_dependents();
  griddep_wait();
  const int pairs = inter / 2;
  const int64_t total = (int64_t)rows * pairs;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(k / pairs), i = (int)(k - (int64_t)r * pairs);
    const uint32_t g = reinterpret_cast<const uint32_t*>(gu + (size_t)r * 2 * inter)[i];
    const uint32_t u = reinterpret_cast<const uint32_t*>(gu + (size_t)r * 2 * inter + inter)[i];
    float o[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float gv = bf(g, e);
      const float s = silu_bf16(gv);
      o[e] = s * bf(u, e);
    }
    reinterpret_cast<uint32_t*>(act + (size_t)r * inter)[i] = pack_bf2(o[0], o[1]);
  }
}

// The bookkeeping that opens a decode step, for sequence b = blockIdx.x at
// position p = positions[b]: seq_lens[b] = p + 1, slots[b] = the cache slot of
// position p through the block table, and h[b, :] = embed[tokens[b], :] (the
// embedding lookup).  One CTA per sequence.  Ids and positions outside their
// tables read nothing: a zero row, slot -1, and the device status records it.
__global__ void __launch_bounds__(256)
    decode_step_prep_kernel(const int32_t* pos, const int64_t* tokens, const uint4* embed, int hidden_v,
                            int vocab, const int32_t* bt, int64_t bt_stride, int max_blocks, int block_size,
                            int32_t* seq_lens, int64_t* slots, uint4* h) {
  if (threadIdx.x == 0) griddep_launch_dependents();
  griddep_wait();  // positions and tokens are the previous step's
  const int b = blockIdx.x;
  const int p = max(pos[b], 0);
  const int64_t tok = tokens[b];
  const bool tok_ok = tok >= 0 && tok < vocab;
  if (threadIdx.x == 0) {
    seq_lens[b] = p + 1;
    const int page = p / block_size;
    slots[b] = page < max_blocks ? (int64_t)bt[(int64_t)b * bt_stride + page] * block_size + p % block_size : -1;
    if (page >= max_blocks || !tok_ok) atomicExch(&g_device_status, kDevIndexRange);
  }
  uint4* dst = h + (size_t)b * hidden_v;
  if (!tok_ok) {
    for (int i = threadIdx.x; i < hidden_v; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = embed + (size_t)tok * hidden_v;
  for (int i = threadIdx.x; i < hidden_v; i += blockDim.x) dst[i] = __ldg(src + i);
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelExC(&lc, fn, args);
}

}  // namespace

int rmsnorm_residual_launch(void* h, const void* delta, const void* weight, void* x, int rows,
                            int hidden, float eps, void* stream) {
  if (!h || !weight || !x || rows <= 0 || hidden <= 0) return B200KV_ERR_INVALID_ARG;
  if (hidden % 8 || hidden > 8 * 8 * kNormThreads) return B200KV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(delta) |
       reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(x)) & 15)
    return B200KV_ERR_MISALIGNED;
  __nv_bfloat16* hp = static_cast<__nv_bfloat16*>(h);
  const __nv_bfloat16* dp = static_cast<const __nv_bfloat16*>(delta);
  const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(weight);
  __nv_bfloat16* xp = static_cast<__nv_bfloat16*>(x);
  void* args[] = {&hp, &dp, &wp, &xp, &hidden, &eps};
  return launch_pdl(reinterpret_cast<const void*>(rmsnorm_residual_kernel), dim3(rows),
                    dim3(kNormThreads), args, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? B200KV_OK : B200KV_ERR_LAUNCH;
}

int rope_kv_write_launch(void* qkv, int64_t qkv_st, const int32_t* positions, const float* cos_sin,
                         int max_pos, const int64_t* slots, void* k_cache, void* v_cache,
                         int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0, int64_t sv1,
                         int64_t sv2, const float* k_scale, const float* v_scale, int num_tokens,
                         int hq, int hkv, int head_dim, int block_size, int kv_dtype, void* stream) {
  if (!qkv || !positions || !cos_sin || !slots || !k_cache || !v_cache) return B200KV_ERR_INVALID_ARG;
  if (num_tokens < 0 || hq <= 0 || hkv <= 0 || head_dim <= 0 || head_dim % 2 || block_size <= 0 ||
      max_pos <= 0)
    return B200KV_ERR_INVALID_ARG;
  if (kv_dtype != B200KV_KV_FP8_E4M3 && kv_dtype != B200KV_KV_BF16) return B200KV_ERR_UNSUPPORTED;
  const bool fp8 = kv_dtype == B200KV_KV_FP8_E4M3;
  if (fp8 && (!k_scale || !v_scale)) return B200KV_ERR_INVALID_ARG;
  if (num_tokens == 0) return B200KV_OK;
  const int esz = fp8 ? 1 : 2;
  RopeKvParams p;
  p.qkv = static_cast<__nv_bfloat16*>(qkv);
  p.qkv_st = qkv_st;
  p.pos = positions;
  p.cos_sin = cos_sin;
  p.max_pos = max_pos;
  p.slots = slots;
  p.kc = static_cast<uint8_t*>(k_cache);
  p.vc = static_cast<uint8_t*>(v_cache);
  p.sk0 = sk0 * esz; p.sk1 = sk1 * esz; p.sk2 = sk2 * esz;
  p.sv0 = sv0 * esz; p.sv1 = sv1 * esz; p.sv2 = sv2 * esz;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.hq = hq;
  p.hkv = hkv;
  p.d = head_dim;
  p.block_size = block_size;
  void* args[] = {&p};
  const void* fn = fp8 ? reinterpret_cast<const void*>(rope_kv_write_kernel<true>)
                       : reinterpret_cast<const void*>(rope_kv_write_kernel<false>);
  return launch_pdl(fn, dim3(num_tokens), dim3(256), args, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? B200KV_OK : B200KV_ERR_LAUNCH;
}

int decode_step_prep_launch(const int32_t* positions, const int64_t* tokens, const void* embed, int hidden,
                            int vocab, const int32_t* block_table, int64_t bt_stride, int max_blocks,
                            int block_size, int num_seqs, int32_t* seq_lens, int64_t* slots, void* h,
                            void* stream) {
  if (!positions || !tokens || !embed || !block_table || !seq_lens || !slots || !h) return B200KV_ERR_INVALID_ARG;
  if (hidden <= 0 || vocab <= 0 || max_blocks <= 0 || block_size <= 0 || num_seqs <= 0)
    return B200KV_ERR_INVALID_ARG;
  if (hidden % 8 || ((reinterpret_cast<uintptr_t>(embed) | reinterpret_cast<uintptr_t>(h)) & 15))
    return B200KV_ERR_MISALIGNED;
  const uint4* e = static_cast<const uint4*>(embed);
  uint4* hp = static_cast<uint4*>(h);
  int hv = hidden / 8;
  void* args[] = {&positions, &tokens, &e,   &hv,    &vocab, &block_table, &bt_stride,
                  &max_blocks, &block_size, &seq_lens, &slots, &hp};
  return launch_pdl(reinterpret_cast<const void*>(decode_step_prep_kernel), dim3(num_seqs), dim3(256), args,
                    static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? B200KV_OK : B200KV_ERR_LAUNCH;
}

int swiglu_launch(const void* gate_up, void* act, int rows, int inter, void* stream) {
  if (!gate_up || !act || rows <= 0 || inter <= 0) return B200KV_ERR_INVALID_ARG;
  if (inter % 2 || (reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(act)) & 3)
    return B200KV_ERR_MISALIGNED;
  const __nv_bfloat16* g = static_cast<const __nv_bfloat16*>(gate_up);
  __nv_bfloat16* a = static_cast<__nv_bfloat16*>(act);
  const int64_t total = (int64_t)rows * (inter / 2);
  const int blocks = (int)((total + 255) / 256 < 1184 ? (total + 255) / 256 : 1184);
  void* args[] = {&g, &a, &rows, &inter};
  return launch_pdl(reinterpret_cast<const void*>(swiglu_kernel), dim3(blocks), dim3(256), args,
                    static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? B200KV_OK : B200KV_ERR_LAUNCH;
}

}  // namespace b200kv
