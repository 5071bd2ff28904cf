/*
 * b200kv.h — C ABI of libb200kv.so, the sm_100a (B200) implementation of the
 * pty819/gfx1201-tuning-log inference hot path:
 *
 *   - MXFP4 (e2m1 weights + e8m0 group scales) W4A16 matvec / skinny GEMM
 *   - fp8-e4m3 (or bf16) paged-KV split-K decode attention
 *   - fp8-e4m3 paged-KV causal (varlen) prefill attention on tcgen05
 *   - the paged KV-cache write (bf16 -> fp8 quantise + scatter)
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless stated otherwise; the caller owns
 *     every buffer. Nothing here allocates device memory.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call is asynchronous on that stream and never synchronises the host,
 *     so calls can be captured into CUDA graphs.
 *   - Entry points return 0 (B200KV_OK) or a B200KV_ERR_* code; on error nothing
 *     was launched. b200kv_status_string() names a code.
 *   - Strides are in ELEMENTS of the tensor's own dtype (torch's Tensor.stride()),
 *     innermost stride 1.
 *   - No global mutable host state beyond a cached device-attribute table and the
 *     thread-local last error of the void-returning h4mv_launch().
 */
#ifndef B200KV_H
#define B200KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define B200KV_OK                 0
#define B200KV_ERR_INVALID_ARG    1  /* null pointer, negative/zero size, bad stride */
#define B200KV_ERR_UNSUPPORTED    2  /* shape/dtype outside what the kernels implement */
#define B200KV_ERR_MISALIGNED     3  /* pointer or stride violates a 16-byte rule */
#define B200KV_ERR_WORKSPACE      4  /* workspace missing or smaller than required */
#define B200KV_ERR_LAUNCH         5  /* the CUDA launch itself failed */
#define B200KV_ERR_NO_DEVICE      6  /* no sm_100 device current */

/* dtype tags for KV caches */
#define B200KV_KV_FP8_E4M3        0  /* 1 byte/elem, per-tensor fp32 k/v scales */
#define B200KV_KV_BF16            1  /* 2 bytes/elem, scales ignored             */

/* Library version (major*10000 + minor*100 + patch). */
int b200kv_version(void);

/* Human-readable name of a status code (static string). */
const char* b200kv_status_string(int status);

/* Status of the most recent h4mv_launch() on the calling host thread. */
int b200kv_last_error(void);

/*
 * Device-side status word written by kernels that hit a bounded wait limit.
 * 0 = clean; B200KV_DEV_MBARRIER_TIMEOUT: an mbarrier (a copy or a peer warp)
 * never completed; B200KV_DEV_PEER_TIMEOUT: a peer GPU's allreduce flag did not
 * arrive; B200KV_DEV_CHAIN_TIMEOUT: an input tile of a chained GEMV
 * (b200kv_mxfp4_chain) was not ready in time; B200KV_DEV_INDEX_RANGE: a token
 * id or position outside its table (b200kv_decode_step_prep).  Reading it
 * synchronises the given stream.  b200kv_reset_device_status() clears it
 * (async on stream).
 */
#define B200KV_DEV_MBARRIER_TIMEOUT 0x101
#define B200KV_DEV_PEER_TIMEOUT     0x103
#define B200KV_DEV_CHAIN_TIMEOUT    0x104
#define B200KV_DEV_INDEX_RANGE      0x105
int b200kv_get_device_status(void* stream, int* status_out);
int b200kv_reset_device_status(void* stream);

/* ---- MXFP4 W4A16 matvec ------------------------------------------------------
 *
 * out[m, n] = bf16_rn( sum_g scale(St[n, g]) * sum_{j<32} e2m1(W[n, 32g+j]) * X[m, 32g+j] )
 *
 *   W   uint8 [N, K/2]   two e2m1 codes per byte, low nibble = even k; 16-B aligned
 *   St  uint8 [N, K/32]  e8m0 group scales, already transposed from the checkpoint's
 *                        [K/32, N] layout; scale(b) = 2^(b-127) for 1<=b<=254,
 *                        scale(0) = 0 and scale(255) = inf (the bit pattern b<<23
 *                        read as fp32, exactly as the reference kernel does)
 *   X   bf16  [M, K]     contiguous, 16-B aligned
 *   out bf16  [M, N]     contiguous
 *   1 <= M <= 8, K % 32 == 0, N >= 1.
 *
 * Replaces h4mv/h4mv.cu:106-122 (h4mv_launch) of the reference, with a status
 * return.  Accumulation is fp32; products e2m1 x bf16 are exact.
 */
int b200kv_mxfp4_gemv(const void* W, const void* St, const void* X, void* out,
                      int N, int K, int M, void* stream);

/*
 * Drop-in for the reference's own symbol (h4mv/h4mv.cu:106-107), same
 * signature and argument meaning, loadable through the same ctypes binding
 * (h4mv/fp8kv_hipw4.py:21-23).  Unlike the reference it does NOT silently run
 * M>8 as M=8: invalid arguments launch nothing and set b200kv_last_error().
 */
void h4mv_launch(const void* W, const void* St, const void* Xb, void* Out,
                 int N, int K, int M, void* stream);

/* ---- fp8 paged-KV decode attention ------------------------------------------
 *
 * For every sequence s < num_seqs and query head h (GQA = num_q_heads/num_kv_heads,
 * kv head kh = h / GQA), with L = seq_lens[s] and token t = qsl[s]:
 *
 *   score[j] = (q[t, h, :] . K[j, kh, :]) * sm_scale * k_scale      j < L
 *   out[r, h, :] = v_scale * softmax(score) @ V[:L, kh, :]           (bf16)
 *
 * where K[j] lives in block block_table[s, j / block_size] at slot j % block_size:
 *   key element (j, kh, d) = k_cache[blk*sk0 + slot*sk1 + kh*sk2 + d]
 * and r = qsl[s] when out_by_qsl != 0 (fp8kv_kernel.py:70), r = s otherwise
 * (fp8kv_v3.py:112).  Sequences with L == 0 produce zeros.
 *
 * Replaces the Python entry points vllm-fp8kv/fp8kv_v3.py:116-139 (split +
 * reduce Triton kernels) and vllm-fp8kv/fp8kv_kernel.py:75-88.
 *
 *   q            bf16 [*, num_q_heads, head_dim]   strides (q_stride_tok, q_stride_head, 1)
 *   k/v_cache    fp8 e4m3 or bf16 (kv_dtype), strides (s*0, s*1, s*2, 1) in elements
 *   out          bf16, strides (out_stride_tok, out_stride_head, 1)
 *   qsl          int32 [num_seqs+1]; seq_lens int32 [num_seqs]
 *   block_table  int32 [num_seqs, >= max_blocks_per_seq], row stride bt_stride
 *   k/v_scale    device fp32 scalars (ignored for bf16 KV)
 *   head_dim must be 128; GQA must be 1, 2, 4 or 8.
 *   num_blocks   blocks in the cache (its first dimension), 0 if unknown.  fp8
 *                caches with block_size 16/32/64/128 and num_blocks > 0 have their
 *                pages loaded by TMA (block ids outside [0, num_blocks) read as
 *                zeros); other caches take a per-row asynchronous-copy gather.
 *   num_splits   CTAs (a thread-block cluster) that share one (sequence, kv head):
 *                0 = choose from the SM count and the context bound (max_seq_len_hint,
 *                or max_blocks_per_seq*block_size when the hint is 0); otherwise a
 *                request, rounded up to a power of two, at most 16.
 * No workspace: the split partials are merged through distributed shared memory.
 */
int b200kv_decode_attn(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                       const void* k_cache, const void* v_cache,
                       int64_t sk0, int64_t sk1, int64_t sk2,
                       int64_t sv0, int64_t sv1, int64_t sv2,
                       void* out, int64_t out_stride_tok, int64_t out_stride_head,
                       const int32_t* qsl, const int32_t* seq_lens,
                       const int32_t* block_table, int64_t bt_stride,
                       const float* k_scale, const float* v_scale, float sm_scale,
                       int num_seqs, int num_q_heads, int num_kv_heads, int head_dim,
                       int block_size, int num_blocks, int max_blocks_per_seq,
                       int max_seq_len_hint, int kv_dtype, int out_by_qsl, int num_splits,
                       void* stream);

/* ---- MXFP4 on block-scaled tensor cores (load-time packed scales) -------------
 *
 * The same product as b200kv_mxfp4_gemv, computed by tcgen05
 * kind::mxf8f6f4.block_scale MMAs: the packed e2m1 weights go to the tensor
 * core straight from memory (unpacked to one code per byte by the TMA) and the
 * MMA applies the e8m0 scales itself.  The scales must first be packed once per
 * weight (a load-time repack, as the reference transposes its scales once,
 * h4mv/fp8kv_hipw4.py:32-43) into 512-byte atoms, one per (128 rows x 4
 * groups).  No counterpart call in the reference.
 *
 *   b200kv_mxfp4_packed_scales_bytes  size of the packed buffer (0 if K % 128).
 *   b200kv_mxfp4_pack_scales  scales: layout 0 = St [N, K/32] (transposed, as
 *       b200kv_mxfp4_gemv takes them), 1 = S [K/32, N] (checkpoint layout).
 *       *edge_flag (device int, set to 1, never cleared) reports scale bytes 0
 *       or 255, whose meaning differs between the MMA (2^-127, NaN) and the
 *       reference kernel (0.0, inf): such weights belong on b200kv_mxfp4_gemv.
 *   b200kv_mxfp4_gemm  out[M, N] bf16 for 1 <= M <= 8, K % 128 == 0, W 16-byte
 *       aligned.  x enters as two e4m3 terms with per-32 block scales, split
 *       inside the kernel (every bf16 element within 2^-13 of its block
 *       maximum is exact, smaller ones within 2^-21 of it); fp32 accumulation.
 */
size_t b200kv_mxfp4_packed_scales_bytes(int N, int K);
int b200kv_mxfp4_pack_scales(const void* scales, int layout, void* packed, int N, int K,
                             int* edge_flag, void* stream);
int b200kv_mxfp4_gemm(const void* W, const void* packed_scales, const void* X, void* out, int N,
                      int K, int M, void* stream);

/* The gate_up projection with the MLP activation as its epilogue (the
 * reference's engine fuses the same SiLU * mul into its linear).  W holds the
 * 2 I gate and up rows interleaved in 64-row groups: its 128-row tile w is gate
 * rows 64 w .. 64 w + 63 followed by the same up rows (a load-time row
 * permutation; pack the scales after permuting).  act[M, I] =
 * bf16(bf16(silu(g)) * u), g and u the bf16-rounded products: bit for bit the
 * plain GEMM followed by b200kv_swiglu on the unpermuted weights, when the
 * plain GEMM splits K the same way (the order of the fp32 sum).  N = 2 I,
 * N % 128 == 0.  b200kv_mxfp4_gemm_swiglu: 1 <= M <= 8, as b200kv_mxfp4_gemm,
 * with the same plan; b200kv_mxfp4_gemm_wide_swiglu: any M, as
 * b200kv_mxfp4_gemm_wide with K unsplit across CTAs; act 16-byte aligned. */
int b200kv_mxfp4_gemm_swiglu(const void* W, const void* packed_scales, const void* X, void* act, int N,
                             int K, int M, void* stream);
int b200kv_mxfp4_gemm_wide_swiglu(const void* W, const void* packed_scales, const void* X, int64_t x_stride,
                                  void* workspace, size_t workspace_bytes, void* act, int N, int K, int M,
                                  void* stream);

/* The qkv projection of a decode step with the rotary embedding and the paged
 * KV-cache write as its epilogue: one launch in place of b200kv_mxfp4_gemm
 * followed by b200kv_rope_kv_write (no counterpart in the reference, whose
 * engine runs them as separate kernels).  W holds the [q heads | k heads |
 * v heads] rows of one rank (N = (num_q_heads + 2 num_kv_heads) * 128,
 * head_dim 128); 1 <= M <= 8 tokens, with the plan of b200kv_mxfp4_gemm.  The
 * q columns of qkv [M, N] receive the rotated q, bit for bit what the two
 * calls leave there; k (rotated) and v go to the fp8 e4m3 cache at
 * slot_mapping[m] exactly as b200kv_rope_kv_write writes them (arguments as
 * there: cos_sin [max_pos][128], positions clamped to [0, max_pos), strides
 * in elements, slots < 0 skipped).  The k and v columns of qkv are not
 * written.  kv_dtype must be B200KV_KV_FP8_E4M3. */
int b200kv_mxfp4_gemm_rope_kv(const void* W, const void* packed_scales, const void* X, void* qkv, int N,
                              int K, int M, const int32_t* positions, const float* cos_sin, int max_pos,
                              const int64_t* slot_mapping, void* k_cache, void* v_cache,
                              int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2,
                              const float* k_scale, const float* v_scale, int num_q_heads, int num_kv_heads,
                              int block_size, int kv_dtype, void* stream);

/* Wide batches (prefill chunks, batched decode; any M >= 1, meant for M > 8):
 * the same product on tcgen05 kind::mxf8f6f4.block_scale MMAs, weights as e2m1
 * with the packed scale atoms above, x as two e4m3 terms with per-32 block
 * scales written by a pre-pass into the caller's workspace (exact for every
 * element within 2^-13 of its block maximum, within 2^-21 of it otherwise);
 * fp32 accumulation.  The reference's counterpart is its dequant + matmul
 * path for M > 8 (h4mv/fp8kv_hipw4.py:62-94).
 *   b200kv_mxfp4_gemm_wide_workspace_bytes  workspace size for (M, K): 128 B
 *       rows of 2 K bytes per 64 tokens plus scale atoms (0 if K % 128).
 *   b200kv_mxfp4_gemm_wide  out[M, N] bf16; x rows x_stride elements apart
 *       (a multiple of 8, >= K), K % 128 == 0, W / packed / x 16-byte aligned,
 *       workspace 128-byte aligned.  Two launches on `stream` (pre-pass, GEMM);
 *       calls that share a workspace must be ordered on one stream. */
size_t b200kv_mxfp4_gemm_wide_workspace_bytes(int M, int K);
int b200kv_mxfp4_gemm_wide(const void* W, const void* packed_scales, const void* X, int64_t x_stride,
                           void* workspace, size_t workspace_bytes, void* out, int N, int K, int M,
                           void* stream);

/* b200kv_mxfp4_gemm_wide without a caller workspace, for callers that cannot
 * allocate device memory: a serving engine that has already given all free HBM
 * to its KV-cache pool, or a host that binds this C ABI and has no device
 * allocator.  No counterpart in the reference.  The activation terms go to a
 * scratch array inside this library (4.3 MB, held on every GPU that loads the
 * library until exit), so M <= 128 and K <= 16384; larger sizes return
 * B200KV_ERR_WORKSPACE.  Allocates nothing.  Its first call on a device looks
 * up the array's device address (make that call before any stream capture).
 * All calls on a device share the array: calls that overlap on the GPU (on
 * different streams) race, calls ordered on one stream do not.  Each call
 * rewrites all of the scratch it reads, so nothing has to start at zero. */
int b200kv_mxfp4_gemm_wide_noalloc(const void* W, const void* packed_scales, const void* X,
                                   int64_t x_stride, void* out, int N, int K, int M, void* stream);

/* A chain of dependent MXFP4 matvecs (1 <= M <= 8) in one persistent launch:
 * op j computes the product of b200kv_mxfp4_gemm on (weight_j, packed scales,
 * x_j), where x_j is an input of the call or op x_from's output, so a decode
 * step's o -> gate_up -> down -> next qkv runs without a launch boundary
 * between the products.  Every SM streams its share of every op's weights
 * without waiting (load-time data) and waits, per 128-k box, only for the
 * tiles of the producing op that hold that slice of x; a tile whose K range is
 * split over several SMs is reduced in a fixed order through the workspace.
 * Arithmetic per op as b200kv_mxfp4_gemm (x as two exact e4m3 terms, fp32
 * accumulation, bf16 output).  No counterpart call in the reference, whose
 * engine launches one h4mv per linear (h4mv/fp8kv_hipw4.py:62-94).
 *   epilogue B200KV_CHAIN_STORE: out[m, n] (bf16, rows out_stride apart).
 *   epilogue B200KV_CHAIN_SWIGLU: the op's weight rows are interleaved in
 *     blocks of 64 (rows 128 t .. 128 t + 63 = gate rows 64 t .., the next 64 =
 *     the matching up rows), N % 128 == 0, and out[m, i] = bf16(bf16(silu(g)) * u)
 *     for i < N / 2 (the rounding of b200kv_swiglu).
 *   x_from = -1: x (bf16, rows x_stride apart, 16-byte aligned, x_stride % 8 == 0)
 *     is read from `x`; x_from = i < j: x is op i's output (x, x_stride ignored).
 *   K % 128 == 0, at most 8 ops.  The workspace (b200kv_mxfp4_chain_workspace_bytes,
 *   256-byte aligned) holds per-tile counters and ready flags that persist
 *   across calls: zero it once before the first call and keep one workspace
 *   per chain that is replayed (a call that reported B200KV_DEV_CHAIN_TIMEOUT
 *   leaves it inconsistent: zero it again).  One CTA per SM, cooperative. */
#define B200KV_CHAIN_STORE  0
#define B200KV_CHAIN_SWIGLU 1
typedef struct b200kv_chain_op {
  const void* weight;          /* uint8 [N, K/2], e2m1 pairs, 16-byte aligned */
  const void* packed_scales;   /* b200kv_mxfp4_pack_scales output for (N, K) */
  const void* x;               /* bf16 [M, K] when x_from == -1 */
  int64_t x_stride;            /* elements between x rows */
  void* out;                   /* bf16 [M, N] (N / 2 for SWIGLU) */
  int64_t out_stride;          /* elements between output rows */
  int32_t N, K;
  int32_t x_from;              /* -1, or the index of an earlier op whose output is x */
  int32_t epilogue;            /* B200KV_CHAIN_STORE or B200KV_CHAIN_SWIGLU */
} b200kv_chain_op;
size_t b200kv_mxfp4_chain_workspace_bytes(const b200kv_chain_op* ops, int nops, int M);
int b200kv_mxfp4_chain(const b200kv_chain_op* ops, int nops, int M, void* workspace, size_t workspace_bytes,
                       void* stream);

/* ---- fp8 paged-KV causal prefill attention -----------------------------------
 *
 * For every sequence s with query rows cu_seqlens_q[s] .. cu_seqlens_q[s+1]-1
 * (qlen of them) and kv length L = seq_lens[s], query i sits at position
 * q0 + i with q0 = L - qlen and attends keys 0 .. q0 + i of the same kv head:
 *
 *   out[row, h, :] = v_scale * softmax_j<=q0+i((q . K[j]) * sm_scale * k_scale) @ V
 *
 * Keys are gathered through block_table[s, :] exactly as in b200kv_decode_attn.
 * When cu_seqlens_q and seq_lens are both NULL the call is the reference's
 * single-sequence form (vllm-fp8kv/fp8kv_prefill.py:124-144, `run(..., q0, qlen)`):
 * num_seqs must be 1, rows 0 .. qlen_single-1, q0 = q0_single, table row 0.
 *
 * Replaces the reference's Triton kernel vllm-fp8kv/fp8kv_prefill.py:32-121,
 * generalised to varlen batches.  Runs on tcgen05 tensor cores with fp32
 * accumulation in tensor memory: fp8 caches with block_size 16/32/64/128 take
 * the fp8 MMA path (pages gathered by TMA straight from the cache, query and
 * probabilities split into two e4m3 terms each, so both products keep a
 * bf16-sized significand); other caches take an f16 path.  head_dim 128,
 * GQA 1/2/4/8.
 *   max_qlen   upper bound of the per-sequence query lengths (grid size);
 *              ignored in the single-sequence form.
 *   num_blocks number of blocks in the cache (its first dimension): block
 *              ids outside [0, num_blocks) read as zeros on the fp8 path.
 *   num_tokens the batch's query rows, cu_seqlens_q[num_seqs] (0 if not
 *              known on the host): sizes the grid to the batch's query tiles
 *              instead of num_seqs x max_qlen's, so short and one-token
 *              sequences cost no CTAs.
 */
int b200kv_prefill_attn(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                        const void* k_cache, const void* v_cache,
                        int64_t sk0, int64_t sk1, int64_t sk2,
                        int64_t sv0, int64_t sv1, int64_t sv2,
                        void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                        const int32_t* block_table, int64_t bt_stride,
                        const float* k_scale, const float* v_scale, float sm_scale,
                        int num_seqs, int max_qlen, int q0_single, int qlen_single,
                        int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                        int num_blocks, int kv_dtype, int num_tokens, void* stream);

/* Mixed batches (decode tokens and prefills in one varlen batch, as vLLM's
 * TritonAttentionImpl.forward receives them, vllm-fp8kv/fp8kv_prefill.py:156-198
 * takes the whole batch through its prefill kernel): the same result as
 * b200kv_prefill_attn over the batch, with the work split on the device by
 * each sequence's query count, without a host sync.  Sequences with one query
 * token run on the split-K decode kernel (that token attends its whole
 * context, as a one-token prefill does), the others on the varlen prefill
 * kernel; each kernel leaves the other's sequences untouched (two launches on
 * `stream`).  No counterpart call in the reference.
 *   max_seq_len  upper bound of seq_lens (sizes the decode kernel's split);
 *   max_blocks_per_seq  block_table row capacity;  other arguments (num_tokens
 *   included) as b200kv_prefill_attn's varlen form (cu_seqlens_q and seq_lens
 *   required). */
int b200kv_attn_varlen_mixed(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                             const void* k_cache, const void* v_cache,
                             int64_t sk0, int64_t sk1, int64_t sk2,
                             int64_t sv0, int64_t sv1, int64_t sv2,
                             void* out, int64_t out_stride_tok, int64_t out_stride_head,
                             const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                             const int32_t* block_table, int64_t bt_stride,
                             const float* k_scale, const float* v_scale, float sm_scale,
                             int num_seqs, int max_qlen, int max_seq_len,
                             int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                             int num_blocks, int max_blocks_per_seq, int kv_dtype, int num_tokens,
                             void* stream);

/* ---- paged KV-cache write ------------------------------------------------------
 *
 * For every token t < num_tokens with slot = slot_mapping[t] >= 0:
 *   k_cache[slot / block_size, slot % block_size, h, :] = q8(key[t, h, :] / k_scale)
 *   v_cache[...same...]                                 = q8(value[t, h, :] / v_scale)
 * where q8 is fp32 IEEE division then round-to-nearest-even e4m3 with saturation to
 * +-448 (kv_dtype FP8_E4M3), or a plain copy (kv_dtype BF16, scales ignored).
 * Negative slots (padding tokens) are skipped.
 *
 * Replaces vLLM's reshape_and_cache_flash custom op, which the reference's engine
 * runs ahead of its attention kernels (profiling/prof_h4mv.txt:9); same slot and
 * quantisation semantics.
 *
 *   key/value   bf16 [num_tokens, num_kv_heads, head_dim], strides (st, sh, 1)
 *   k/v_cache   [NB, block_size, num_kv_heads, head_dim], strides (s*0, s*1, s*2, 1)
 *   slot_mapping int64 [num_tokens]; k/v_scale device fp32 scalars
 *   head_dim % 16 == 0; cache rows 16-byte aligned.
 */
int b200kv_kv_write(const void* key, int64_t key_stride_tok, int64_t key_stride_head,
                    const void* value, int64_t value_stride_tok, int64_t value_stride_head,
                    void* k_cache, void* v_cache,
                    int64_t sk0, int64_t sk1, int64_t sk2,
                    int64_t sv0, int64_t sv1, int64_t sv2,
                    const int64_t* slot_mapping, const float* k_scale, const float* v_scale,
                    int num_tokens, int num_kv_heads, int head_dim, int block_size,
                    int kv_dtype, void* stream);

/* The bookkeeping that opens a decode step, one launch: for each sequence
 * b < num_seqs at position p = positions[b] (int32; negative taken as 0):
 * seq_lens[b] = p + 1, slot_mapping[b] = block_table[b, p / block_size] *
 * block_size + p % block_size, and h[b, :] = embed[tokens[b], :] (bf16
 * [vocab, hidden] rows, hidden % 8 == 0, 16-byte aligned).  A token id
 * outside [0, vocab) gives a zero row, a position past the row's
 * max_blocks_per_seq pages gives slot -1 (skipped by the KV writes); both
 * record B200KV_DEV_INDEX_RANGE.  No counterpart in the reference (its engine
 * prepares these on the host). */
int b200kv_decode_step_prep(const int32_t* positions, const int64_t* tokens, const void* embed, int hidden,
                            int vocab, const int32_t* block_table, int64_t bt_stride, int max_blocks_per_seq,
                            int block_size, int num_seqs, int32_t* seq_lens, int64_t* slot_mapping, void* h,
                            void* stream);

/* ---- greedy argmax over logits rows ---------------------------------------------
 *
 * For each row r < rows of x (fp32, row stride ld elements): max_val[r] = the
 * largest of x[r, 0 .. cols) and max_idx[r] = the lowest index holding it
 * (torch.max(x, dim=1) on NaN-free rows).  max_val may be NULL.  One launch,
 * a cluster of 8 CTAs per row, no scratch.  No counterpart in the reference
 * (its engine's sampler does this). */
int b200kv_argmax_rows(const float* x, int64_t ld, int rows, int cols, float* max_val, int64_t* max_idx,
                       void* stream);

/* ---- Decoder-layer glue for the 7B decode loop --------------------------------------
 *
 * The element-wise steps around the hot path (HF Llama semantics; the
 * reference left them to vLLM's own kernels, profiling/prof_h4mv.txt:11-15).
 * All bf16, launched on `stream`, no synchronisation.
 *
 * b200kv_rmsnorm_residual: per row, h <- bf16(h + delta) when delta != NULL
 *   (in place), then x = weight * bf16(h * rsqrt(mean(h^2) + eps)) with fp32
 *   statistics.  hidden % 8 == 0, <= 16384; 16-byte aligned rows.
 * b200kv_rope_kv_write: per token t (row stride qkv_stride_tok of the fused
 *   [q | k | v] projection, heads of head_dim), rotary embedding at
 *   positions[t] (neox halves; cos_sin = fp32 [max_pos][head_dim], the cos of
 *   the head_dim/2 frequencies then their sin) of the q heads in place and of
 *   the k heads, which go with v to the paged cache slot slot_mapping[t]
 *   (< 0: skipped) exactly as b200kv_kv_write stores them.
 * b200kv_swiglu: act[r, i] = bf16(bf16(silu(g)) * u), g = gate_up[r, i],
 *   u = gate_up[r, inter + i]; inter even.
 */
int b200kv_rmsnorm_residual(void* h, const void* delta, const void* weight, void* x, int rows,
                            int hidden, float eps, void* stream);
int b200kv_rope_kv_write(void* qkv, int64_t qkv_stride_tok, const int32_t* positions,
                         const float* cos_sin, int max_pos, const int64_t* slot_mapping,
                         void* k_cache, void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2,
                         int64_t sv0, int64_t sv1, int64_t sv2, const float* k_scale,
                         const float* v_scale, int num_tokens, int num_q_heads, int num_kv_heads,
                         int head_dim, int block_size, int kv_dtype, void* stream);
int b200kv_swiglu(const void* gate_up, void* act, int rows, int inter, void* stream);

/* ---- Tensor-parallel allreduce over peer memory ---------------------------------
 *
 * Sum of a bf16 vector of n elements (n % 8 == 0, n <= 32768: one [M <= 8, 4096]
 * partial of the row-parallel o / down projections) over tp <= 8 GPUs of one
 * node, one rank per GPU, through NVLink peer stores and flags -- the
 * collective of the tensor-parallel layout (no counterpart in the reference,
 * which runs on one GPU).  Each rank allocates one communication buffer
 * (b200kv_comm_alloc, 64-byte CUDA IPC handle out), exchanges the handles over
 * any host channel, opens the peers' (b200kv_comm_open; its own stays as
 * allocated) and passes all tp buffer pointers, in rank order, to every call.
 * All ranks must make the same sequence of calls; a call waits at most 200 ms
 * for the peers and then reports B200KV_DEV_PEER_TIMEOUT through the device
 * status word.  in == out is allowed.  Capturable in CUDA graphs.
 */
size_t b200kv_comm_buffer_bytes(void);
int b200kv_comm_alloc(void** buf, void* ipc_handle64);
int b200kv_comm_open(const void* ipc_handle64, void** peer_buf);
int b200kv_comm_close(void* peer_buf);
int b200kv_comm_free(void* buf);
int b200kv_allreduce_oneshot(const void* in, void* out, int n, void* const* bufs, int rank, int tp,
                             void* stream);

/* The row-parallel MXFP4 product with its allreduce in the epilogue (o and
 * down under tensor parallelism, 1 <= M <= 8): each rank passes its K shard
 * (W [N, K/2], packed scales, X [M, K]) and every rank gets out[M, N] = the sum
 * over ranks of the partials, bit for bit b200kv_mxfp4_gemm followed by
 * b200kv_allreduce_oneshot.  Each finished 128-row tile's bf16 partial goes
 * into every rank's buffer as the tile completes, and the tile's threads then
 * sum the ranks' partials in rank order; one launch, no allreduce kernel.
 * comm_bufs: tp buffers from b200kv_comm_alloc / _open as for the one-shot
 * allreduce, but a set of its own (its counters are per output tile).  N %
 * 128 == 0, N <= 8192, M N <= 32768, out 4-byte aligned.  All ranks make the
 * same sequence of calls; a rank waits at most 200 ms for a peer's tile, then
 * reports B200KV_DEV_PEER_TIMEOUT.  Capturable in CUDA graphs. */
int b200kv_mxfp4_gemm_allreduce(const void* W, const void* packed_scales, const void* X, void* out, int N,
                                int K, int M, void* const* comm_bufs, int rank, int tp, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200KV_H */
