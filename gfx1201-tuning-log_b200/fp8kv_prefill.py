"""fp8-KV causal prefill attention -- drop-in for the reference module
vllm-fp8kv/fp8kv_prefill.py: `run` (:124-144) with the same signature, backed
by the tcgen05 kernel in csrc/prefill_attn.cu, plus `prefill_attention`, the
varlen generalisation (several sequences packed with cu_seqlens, each with
its own block-table row and kv length), and `_install`, which with
FP8KV_PREFILL=1 (:147-198) makes the TritonAttentionImpl.forward patch of
fp8kv_override route prefill batches here as well.

BM / BN / warps / stages tuned the Triton tile and are accepted and ignored:
the B200 kernel always uses 128-row query tiles (GQA heads packed with
tokens, as the reference packs them) and 128-key KV tiles.
"""
import os
import sys

import torch

from _b200kv import KV_BF16, KV_FP8_E4M3, check, lib


def _scale(s, device):
    if torch.is_tensor(s):
        return s.to(device=device, dtype=torch.float32).reshape(-1)[:1].contiguous()
    return torch.tensor([float(s)], device=device, dtype=torch.float32)


def _kv_dtype(t):
    if t.dtype == torch.float8_e4m3fn:
        return KV_FP8_E4M3
    if t.dtype == torch.bfloat16:
        return KV_BF16
    raise TypeError(f"unsupported KV cache dtype {t.dtype}")


def _launch(q, k_cache, v_cache, out, cu, lens, bt, kscale, vscale, sm_scale, num_seqs,
            max_qlen, q0_single, qlen_single):
    if q.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise TypeError("q and out must be bfloat16")
    if bt.dtype != torch.int32 or bt.stride(-1) != 1:
        raise TypeError("block_table must be int32 with contiguous rows")
    dev = q.device
    ks, vs = _scale(kscale, dev), _scale(vscale, dev)
    check(lib.b200kv_prefill_attn(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        out.data_ptr(), out.stride(0), out.stride(1),
        cu.data_ptr() if cu is not None else None,
        lens.data_ptr() if lens is not None else None,
        bt.data_ptr(), bt.stride(0), ks.data_ptr(), vs.data_ptr(), float(sm_scale),
        num_seqs, max_qlen, q0_single, qlen_single, q.shape[1], k_cache.shape[2], q.shape[2],
        k_cache.shape[1], k_cache.shape[0], _kv_dtype(k_cache),
        q.shape[0] if cu is not None else 0,  # rows of q bound the batch's query rows
        torch.cuda.current_stream(dev).cuda_stream),
        "b200kv_prefill_attn")
    return out


def run(q, k_cache, v_cache, out, bt, kscale, vscale, sm_scale, q0, qlen,
        BM=64, BN=32, warps=2, stages=2):
    """Single-sequence causal prefill (reference signature): query rows 0..qlen-1
    at positions q0..q0+qlen-1 over keys 0..q0+qlen-1 through block_table row 0."""
    return _launch(q, k_cache, v_cache, out, None, None, bt, kscale, vscale, sm_scale,
                   1, int(qlen), int(q0), int(qlen))


def prefill_attention(q, k_cache, v_cache, out, cu_seqlens_q, seq_lens, block_table,
                      k_scale, v_scale, sm_scale, max_qlen=None):
    """Varlen causal prefill: sequence s owns query rows cu[s]..cu[s+1]-1 and
    kv length seq_lens[s]; the last qlen keys are its own tokens (q0 = L - qlen)."""
    if cu_seqlens_q.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("cu_seqlens_q and seq_lens must be int32")
    if max_qlen is None:  # host sync; callers on the hot path pass it
        max_qlen = int((cu_seqlens_q[1:] - cu_seqlens_q[:-1]).max().item())
    num_seqs = cu_seqlens_q.shape[0] - 1
    if seq_lens.shape[0] < num_seqs or block_table.shape[0] < num_seqs:
        raise ValueError("seq_lens and block_table need a row per sequence of cu_seqlens_q")
    return _launch(q, k_cache, v_cache, out, cu_seqlens_q, seq_lens, block_table, k_scale,
                   v_scale, sm_scale, num_seqs, int(max_qlen), 0, 0)


def mixed_attention(q, k_cache, v_cache, out, cu_seqlens_q, seq_lens, block_table,
                    k_scale, v_scale, sm_scale, max_qlen, max_seq_len):
    """prefill_attention's result for a batch that mixes decode tokens and
    prefills, split on the device by query count: one-token sequences on the
    split-K decode kernel, the rest on the varlen kernel (no host sync)."""
    if q.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise TypeError("q and out must be bfloat16")
    if cu_seqlens_q.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("cu_seqlens_q and seq_lens must be int32")
    if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise TypeError("block_table must be int32 with contiguous rows")
    num_seqs = cu_seqlens_q.shape[0] - 1
    if seq_lens.shape[0] < num_seqs or block_table.shape[0] < num_seqs:
        raise ValueError("seq_lens and block_table need a row per sequence of cu_seqlens_q")
    dev = q.device
    ks, vs = _scale(k_scale, dev), _scale(v_scale, dev)
    check(lib.b200kv_attn_varlen_mixed(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        out.data_ptr(), out.stride(0), out.stride(1),
        cu_seqlens_q.data_ptr(), seq_lens.data_ptr(), block_table.data_ptr(), block_table.stride(0),
        ks.data_ptr(), vs.data_ptr(), float(sm_scale),
        num_seqs, int(max_qlen), int(max_seq_len), q.shape[1], k_cache.shape[2], q.shape[2],
        k_cache.shape[1], min(k_cache.shape[0], v_cache.shape[0]), block_table.shape[1],
        _kv_dtype(k_cache), q.shape[0], torch.cuda.current_stream(dev).cuda_stream),
        "b200kv_attn_varlen_mixed")
    return out


def _install():
    """FP8KV_PREFILL=1: prefill batches (max_query_len > 1) go to this kernel
    through the fp8kv_override patch of TritonAttentionImpl.forward; the gate
    and the fallback to vLLM's own forward are that module's."""
    if os.environ.get("FP8KV_PREFILL", "0") != "1":
        return False
    import fp8kv_override
    fp8kv_override.enable_prefill()
    ok = fp8kv_override._install()
    if ok:
        sys.stderr.write("[fp8kv-prefill] installed\n")
    return ok


_install()
