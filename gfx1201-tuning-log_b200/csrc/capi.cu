// Exported C ABI of libb200kv.so (declared in include/b200kv.h).
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "b200kv.h"
#include "b200kv_common.cuh"

namespace b200kv {

__device__ int g_device_status = 0;

namespace {
constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices];    // 0 = not cached yet
int g_major[kMaxDevices];

int current_device_slot() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return -1;
  }
  if (g_sms[dev] == 0) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    g_major[dev] = major;
    g_sms[dev] = sms;  // written last: a racing reader sees 0 and recomputes
  }
  return dev;
}

thread_local int t_last_error = B200KV_OK;
}  // namespace

int num_sms_current_device() {
  const int d = current_device_slot();
  return d < 0 ? 0 : g_sms[d];
}

int sm_major_current_device() {
  const int d = current_device_slot();
  return d < 0 ? 0 : g_major[d];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("B200KV_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int mxfp4_gemv_launch(const void* W, const void* St, const void* X, void* out, int N, int K,
                      int M, void* stream);
int rmsnorm_residual_launch(void* h, const void* delta, const void* weight, void* x, int rows,
                            int hidden, float eps, void* stream);
int rope_kv_write_launch(void* qkv, int64_t qkv_st, const int32_t* positions, const float* cos_sin,
                         int max_pos, const int64_t* slots, void* k_cache, void* v_cache,
                         int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0, int64_t sv1,
                         int64_t sv2, const float* k_scale, const float* v_scale, int num_tokens,
                         int hq, int hkv, int head_dim, int block_size, int kv_dtype, void* stream);
int swiglu_launch(const void* gate_up, void* act, int rows, int inter, void* stream);
int decode_step_prep_launch(const int32_t* positions, const int64_t* tokens, const void* embed, int hidden,
                            int vocab, const int32_t* block_table, int64_t bt_stride, int max_blocks,
                            int block_size, int num_seqs, int32_t* seq_lens, int64_t* slots, void* h,
                            void* stream);
size_t comm_buffer_bytes();
int comm_alloc(void** buf, void* ipc_handle);
int comm_open(const void* ipc_handle, void** peer);
int comm_close(void* peer);
int comm_free(void* buf);
int allreduce_oneshot_launch(const void* in, void* out, int n, void* const* bufs, int rank, int tp,
                             void* stream);
int argmax_rows_launch(const float* x, int64_t ld, int rows, int cols, float* max_val, int64_t* max_idx,
                       void* stream);
int decode_attn_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                       const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                       int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                       const int32_t* qsl, const int32_t* seq_lens, const int32_t* bt,
                       int64_t bt_stride, const float* k_scale, const float* v_scale,
                       float sm_scale, int num_seqs, int hq, int hkv, int head_dim,
                       int block_size, int num_blocks, int max_blocks, int hint, int kv_dtype,
                       int out_by_qsl, int num_splits, void* stream);

int kv_write_launch(const void* key, int64_t k_st, int64_t k_sh, const void* value, int64_t v_st,
                    int64_t v_sh, void* k_cache, void* v_cache, int64_t sk0, int64_t sk1,
                    int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, const int64_t* slots,
                    const float* k_scale, const float* v_scale, int num_tokens, int hkv,
                    int head_dim, int block_size, int kv_dtype, void* stream);

size_t mxfp4_packed_scales_bytes(int N, int K);
int mxfp4_pack_scales_launch(const void* S, int layout, void* Sp, int N, int K, int* edge_flag,
                             void* stream);
int mxfp4_mma_launch(const void* W, const void* Sp, const void* X, void* Out, int N, int K, int M,
                     int epilogue, void* stream, void* const* comm_bufs = nullptr, int rank = 0, int tp = 1);
int mxfp4_mma_rope_kv_launch(const void* W, const void* Sp, const void* X, void* qkv, int N, int K, int M,
                             const int32_t* positions, const float* cos_sin, int max_pos,
                             const int64_t* slots, void* k_cache, void* v_cache, int64_t sk0, int64_t sk1,
                             int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, const float* k_scale,
                             const float* v_scale, int hq, int hkv, int block_size, int kv_dtype,
                             void* stream);
size_t mxfp4_gemm_wide_workspace_bytes(int M, int K);
size_t mxfp4_chain_workspace_bytes(const b200kv_chain_op* ops, int nops, int M);
int mxfp4_chain_launch(const b200kv_chain_op* ops, int nops, int M, void* ws, size_t ws_bytes, void* stream);
int mxfp4_gemm_wide_launch(const void* W, const void* Sp, const void* X, int64_t x_ld, void* ws,
                           size_t ws_bytes, void* Out, int N, int K, int M, int epilogue, void* stream);
int mxfp4_gemm_wide_noalloc_launch(const void* W, const void* Sp, const void* X, int64_t x_ld, void* Out, int N,
                                   int K, int M, void* stream);

int prefill_attn_launch(const void* q, int64_t q_st, int64_t q_sh, const void* k_cache,
                        const void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2, int64_t sv0,
                        int64_t sv1, int64_t sv2, void* out, int64_t o_st, int64_t o_sh,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                        const int32_t* block_table, int64_t bt_stride, const float* k_scale,
                        const float* v_scale, float sm_scale, int num_seqs, int max_qlen,
                        int q0_single, int qlen_single, int hq, int hkv, int head_dim,
                        int block_size, int num_blocks, int kv_dtype, int only_multi, void* stream,
                        int total_q);

void set_last_error(int e) { t_last_error = e; }

}  // namespace b200kv

extern "C" {

int b200kv_version(void) { return 100; }

const char* b200kv_status_string(int status) {
  switch (status) {
    case B200KV_OK: return "ok";
    case B200KV_ERR_INVALID_ARG: return "invalid argument";
    case B200KV_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case B200KV_ERR_MISALIGNED: return "misaligned pointer or stride";
    case B200KV_ERR_WORKSPACE: return "workspace missing or too small";
    case B200KV_ERR_LAUNCH: return "kernel launch failed";
    case B200KV_ERR_NO_DEVICE: return "no sm_100 device is current";
    default: return "unknown status";
  }
}

int b200kv_last_error(void) { return b200kv::t_last_error; }

int b200kv_get_device_status(void* stream, int* status_out) {
  if (!status_out) return B200KV_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, b200kv::g_device_status, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    return B200KV_ERR_LAUNCH;
  }
  *status_out = v;
  return B200KV_OK;
}

int b200kv_reset_device_status(void* stream) {
  static const int zero = 0;
  if (cudaMemcpyToSymbolAsync(b200kv::g_device_status, &zero, sizeof(int), 0,
                              cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    cudaGetLastError();
    return B200KV_ERR_LAUNCH;
  }
  return B200KV_OK;
}

int b200kv_mxfp4_gemv(const void* W, const void* St, const void* X, void* out, int N, int K, int M,
                      void* stream) {
  return b200kv::mxfp4_gemv_launch(W, St, X, out, N, K, M, stream);
}

void h4mv_launch(const void* W, const void* St, const void* Xb, void* Out, int N, int K, int M,
                 void* stream) {
  b200kv::set_last_error(b200kv::mxfp4_gemv_launch(W, St, Xb, Out, N, K, M, stream));
}

int b200kv_decode_attn(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                       const void* k_cache, const void* v_cache, int64_t sk0, int64_t sk1,
                       int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, void* out,
                       int64_t out_stride_tok, int64_t out_stride_head, const int32_t* qsl,
                       const int32_t* seq_lens, const int32_t* block_table, int64_t bt_stride,
                       const float* k_scale, const float* v_scale, float sm_scale, int num_seqs,
                       int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                       int num_blocks, int max_blocks_per_seq, int max_seq_len_hint, int kv_dtype,
                       int out_by_qsl, int num_splits, void* stream) {
  return b200kv::decode_attn_launch(
      q, q_stride_tok, q_stride_head, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2, out,
      out_stride_tok, out_stride_head, qsl, seq_lens, block_table, bt_stride, k_scale, v_scale,
      sm_scale, num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
      max_blocks_per_seq, max_seq_len_hint, kv_dtype, out_by_qsl ? 1 : 0, num_splits, stream);
}

int b200kv_decode_step_prep(const int32_t* positions, const int64_t* tokens, const void* embed, int hidden,
                            int vocab, const int32_t* block_table, int64_t bt_stride, int max_blocks_per_seq,
                            int block_size, int num_seqs, int32_t* seq_lens, int64_t* slot_mapping, void* h,
                            void* stream) {
  return b200kv::decode_step_prep_launch(positions, tokens, embed, hidden, vocab, block_table, bt_stride,
                                         max_blocks_per_seq, block_size, num_seqs, seq_lens, slot_mapping, h,
                                         stream);
}

int b200kv_argmax_rows(const float* x, int64_t ld, int rows, int cols, float* max_val, int64_t* max_idx,
                       void* stream) {
  return b200kv::argmax_rows_launch(x, ld, rows, cols, max_val, max_idx, stream);
}

int b200kv_prefill_attn(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                        const void* k_cache, const void* v_cache, int64_t sk0, int64_t sk1,
                        int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, void* out,
                        int64_t out_stride_tok, int64_t out_stride_head,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                        const int32_t* block_table, int64_t bt_stride, const float* k_scale,
                        const float* v_scale, float sm_scale, int num_seqs, int max_qlen,
                        int q0_single, int qlen_single, int num_q_heads, int num_kv_heads,
                        int head_dim, int block_size, int num_blocks, int kv_dtype, int num_tokens,
                        void* stream) {
  return b200kv::prefill_attn_launch(
      q, q_stride_tok, q_stride_head, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2, out,
      out_stride_tok, out_stride_head, cu_seqlens_q, seq_lens, block_table, bt_stride, k_scale,
      v_scale, sm_scale, num_seqs, max_qlen, q0_single, qlen_single, num_q_heads, num_kv_heads,
      head_dim, block_size, num_blocks, kv_dtype, 0, stream, num_tokens);
}

int b200kv_attn_varlen_mixed(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                             const void* k_cache, const void* v_cache, int64_t sk0, int64_t sk1,
                             int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2, void* out,
                             int64_t out_stride_tok, int64_t out_stride_head,
                             const int32_t* cu_seqlens_q, const int32_t* seq_lens,
                             const int32_t* block_table, int64_t bt_stride, const float* k_scale,
                             const float* v_scale, float sm_scale, int num_seqs, int max_qlen,
                             int max_seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                             int block_size, int num_blocks, int max_blocks_per_seq, int kv_dtype,
                             int num_tokens, void* stream) {
  if (!cu_seqlens_q || !seq_lens || max_qlen < 1) return B200KV_ERR_INVALID_ARG;
  // one-token sequences on the split-K decode kernel (output row = the token's row)
  int r = b200kv::decode_attn_launch(
      q, q_stride_tok, q_stride_head, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2, out,
      out_stride_tok, out_stride_head, cu_seqlens_q, seq_lens, block_table, bt_stride, k_scale,
      v_scale, sm_scale, num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
      max_blocks_per_seq, max_seq_len, kv_dtype, 1 | 2, 0, stream);
  if (r != B200KV_OK || max_qlen == 1) return r;
  // the rest on the varlen kernel
  return b200kv::prefill_attn_launch(
      q, q_stride_tok, q_stride_head, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2, out,
      out_stride_tok, out_stride_head, cu_seqlens_q, seq_lens, block_table, bt_stride, k_scale,
      v_scale, sm_scale, num_seqs, max_qlen, 0, 0, num_q_heads, num_kv_heads, head_dim, block_size,
      num_blocks, kv_dtype, 1, stream, num_tokens);
}

size_t b200kv_mxfp4_packed_scales_bytes(int N, int K) {
  return b200kv::mxfp4_packed_scales_bytes(N, K);
}

int b200kv_mxfp4_pack_scales(const void* scales, int layout, void* packed, int N, int K,
                             int* edge_flag, void* stream) {
  return b200kv::mxfp4_pack_scales_launch(scales, layout, packed, N, K, edge_flag, stream);
}

int b200kv_mxfp4_gemm(const void* W, const void* packed_scales, const void* X, void* out, int N,
                      int K, int M, void* stream) {
  return b200kv::mxfp4_mma_launch(W, packed_scales, X, out, N, K, M, 0, stream);
}

int b200kv_mxfp4_gemm_swiglu(const void* W, const void* packed_scales, const void* X, void* act, int N, int K,
                             int M, void* stream) {
  return b200kv::mxfp4_mma_launch(W, packed_scales, X, act, N, K, M, 1, stream);
}

int b200kv_mxfp4_gemm_rope_kv(const void* W, const void* packed_scales, const void* X, void* qkv, int N,
                              int K, int M, const int32_t* positions, const float* cos_sin, int max_pos,
                              const int64_t* slot_mapping, void* k_cache, void* v_cache, int64_t sk0,
                              int64_t sk1, int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2,
                              const float* k_scale, const float* v_scale, int num_q_heads, int num_kv_heads,
                              int block_size, int kv_dtype, void* stream) {
  // cache strides in elements, as b200kv_rope_kv_write (fp8: bytes)
  return b200kv::mxfp4_mma_rope_kv_launch(W, packed_scales, X, qkv, N, K, M, positions, cos_sin, max_pos,
                                          slot_mapping, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2,
                                          k_scale, v_scale, num_q_heads, num_kv_heads, block_size, kv_dtype,
                                          stream);
}

int b200kv_mxfp4_gemm_allreduce(const void* W, const void* packed_scales, const void* X, void* out, int N,
                                int K, int M, void* const* comm_bufs, int rank, int tp, void* stream) {
  return b200kv::mxfp4_mma_launch(W, packed_scales, X, out, N, K, M, 2, stream, comm_bufs, rank, tp);
}

size_t b200kv_mxfp4_gemm_wide_workspace_bytes(int M, int K) {
  return b200kv::mxfp4_gemm_wide_workspace_bytes(M, K);
}

int b200kv_mxfp4_gemm_wide(const void* W, const void* packed_scales, const void* X, int64_t x_stride,
                           void* workspace, size_t workspace_bytes, void* out, int N, int K, int M,
                           void* stream) {
  return b200kv::mxfp4_gemm_wide_launch(W, packed_scales, X, x_stride, workspace, workspace_bytes, out, N,
                                        K, M, 0, stream);
}

int b200kv_mxfp4_gemm_wide_swiglu(const void* W, const void* packed_scales, const void* X, int64_t x_stride,
                                  void* workspace, size_t workspace_bytes, void* act, int N, int K, int M,
                                  void* stream) {
  return b200kv::mxfp4_gemm_wide_launch(W, packed_scales, X, x_stride, workspace, workspace_bytes, act, N,
                                        K, M, 1, stream);
}

int b200kv_mxfp4_gemm_wide_noalloc(const void* W, const void* packed_scales, const void* X, int64_t x_stride,
                                   void* out, int N, int K, int M, void* stream) {
  return b200kv::mxfp4_gemm_wide_noalloc_launch(W, packed_scales, X, x_stride, out, N, K, M, stream);
}

size_t b200kv_mxfp4_chain_workspace_bytes(const b200kv_chain_op* ops, int nops, int M) {
  return b200kv::mxfp4_chain_workspace_bytes(ops, nops, M);
}

int b200kv_mxfp4_chain(const b200kv_chain_op* ops, int nops, int M, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return b200kv::mxfp4_chain_launch(ops, nops, M, workspace, workspace_bytes, stream);
}

int b200kv_kv_write(const void* key, int64_t key_stride_tok, int64_t key_stride_head,
                    const void* value, int64_t value_stride_tok, int64_t value_stride_head,
                    void* k_cache, void* v_cache, int64_t sk0, int64_t sk1, int64_t sk2,
                    int64_t sv0, int64_t sv1, int64_t sv2, const int64_t* slot_mapping,
                    const float* k_scale, const float* v_scale, int num_tokens, int num_kv_heads,
                    int head_dim, int block_size, int kv_dtype, void* stream) {
  return b200kv::kv_write_launch(key, key_stride_tok, key_stride_head, value, value_stride_tok,
                                 value_stride_head, k_cache, v_cache, sk0, sk1, sk2, sv0, sv1,
                                 sv2, slot_mapping, k_scale, v_scale, num_tokens, num_kv_heads,
                                 head_dim, block_size, kv_dtype, stream);
}

}  // extern "C"

// ---- tensor-parallel allreduce over peer memory ------------------------------------
extern "C" size_t b200kv_comm_buffer_bytes(void) { return b200kv::comm_buffer_bytes(); }
extern "C" int b200kv_comm_alloc(void** buf, void* ipc_handle) { return b200kv::comm_alloc(buf, ipc_handle); }
extern "C" int b200kv_comm_open(const void* ipc_handle, void** peer_buf) {
  return b200kv::comm_open(ipc_handle, peer_buf);
}
extern "C" int b200kv_comm_close(void* peer_buf) { return b200kv::comm_close(peer_buf); }
extern "C" int b200kv_comm_free(void* buf) { return b200kv::comm_free(buf); }
extern "C" int b200kv_allreduce_oneshot(const void* in, void* out, int n, void* const* bufs, int rank,
                                        int tp, void* stream) {
  return b200kv::allreduce_oneshot_launch(in, out, n, bufs, rank, tp, stream);
}

// ---- decoder-layer glue ------------------------------------------------------------
extern "C" int b200kv_rmsnorm_residual(void* h, const void* delta, const void* weight, void* x,
                                       int rows, int hidden, float eps, void* stream) {
  return b200kv::rmsnorm_residual_launch(h, delta, weight, x, rows, hidden, eps, stream);
}
extern "C" int b200kv_rope_kv_write(void* qkv, int64_t qkv_stride_tok, const int32_t* positions,
                                    const float* cos_sin, int max_pos, const int64_t* slot_mapping,
                                    void* k_cache, void* v_cache, int64_t sk0, int64_t sk1,
                                    int64_t sk2, int64_t sv0, int64_t sv1, int64_t sv2,
                                    const float* k_scale, const float* v_scale, int num_tokens,
                                    int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                                    int kv_dtype, void* stream) {
  return b200kv::rope_kv_write_launch(qkv, qkv_stride_tok, positions, cos_sin, max_pos, slot_mapping,
                                      k_cache, v_cache, sk0, sk1, sk2, sv0, sv1, sv2, k_scale, v_scale,
                                      num_tokens, num_q_heads, num_kv_heads, head_dim, block_size,
                                      kv_dtype, stream);
}
extern "C" int b200kv_swiglu(const void* gate_up, void* act, int rows, int inter, void* stream) {
  return b200kv::swiglu_launch(gate_up, act, rows, inter, stream);
}
