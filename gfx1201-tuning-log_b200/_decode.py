"""Host side of the paged-KV decode attention: argument mapping from torch
tensors to the C ABI entry b200kv_decode_attn.

Shared by fp8kv_v3.run (reference vllm-fp8kv/fp8kv_v3.py:116-139) and
fp8kv_kernel.run (reference vllm-fp8kv/fp8kv_kernel.py:75-88).  The kernel
needs no workspace: the split partials of a (sequence, kv head) are merged
inside a thread-block cluster through distributed shared memory.
"""
import torch

from _b200kv import KV_BF16, KV_FP8_E4M3, check, lib


def _scale_tensor(s, device):
    if torch.is_tensor(s):
        if s.dtype != torch.float32 or s.device != device:
            s = s.to(device=device, dtype=torch.float32)
        return s.reshape(-1)[:1].contiguous()
    return torch.tensor([float(s)], device=device, dtype=torch.float32)


def decode_attention(q, k_cache, v_cache, out, qsl, seq_lens, block_table,
                     k_scale, v_scale, sm_scale, *, out_by_qsl, num_splits=0,
                     max_seq_len_hint=0):
    """Launch the decode kernel on the current stream.

    q [T, HQ, D] bf16; k_cache/v_cache [NB, PBLK, HKV, D] (fp8 e4m3 or bf16, any
    strides with the innermost 1); out [*, HQ, D] bf16; qsl int32 [NS+1];
    seq_lens int32 [NS]; block_table int32 [NS, maxblk].  num_splits = CTAs per
    (sequence, kv head), 0 = automatic, at most 16.
    """
    if q.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise TypeError("q and out must be bfloat16")
    if k_cache.dtype == torch.float8_e4m3fn:
        kv_dtype = KV_FP8_E4M3
    elif k_cache.dtype == torch.bfloat16:
        kv_dtype = KV_BF16
    else:
        raise TypeError(f"unsupported KV cache dtype {k_cache.dtype}")
    if v_cache.dtype != k_cache.dtype:
        raise TypeError("k_cache and v_cache dtypes differ")
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("out", out)):
        if t.stride(-1) != 1:
            raise ValueError(f"{name} must have unit innermost stride")
    for name, t in (("qsl", qsl), ("seq_lens", seq_lens), ("block_table", block_table)):
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32")
    if not (qsl.is_contiguous() and seq_lens.is_contiguous() and block_table.stride(1) == 1):
        raise ValueError("qsl/seq_lens must be contiguous, block_table rows contiguous")
    dev = q.device
    ks = _scale_tensor(k_scale, dev)
    vs = _scale_tensor(v_scale, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    check(lib.b200kv_decode_attn(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        out.data_ptr(), out.stride(0), out.stride(1),
        qsl.data_ptr(), seq_lens.data_ptr(), block_table.data_ptr(), block_table.stride(0),
        ks.data_ptr(), vs.data_ptr(), float(sm_scale),
        block_table.shape[0], q.shape[1], k_cache.shape[2], q.shape[2], k_cache.shape[1],
        min(k_cache.shape[0], v_cache.shape[0]),
        block_table.shape[1], int(max_seq_len_hint),
        kv_dtype, 1 if out_by_qsl else 0, int(num_splits), stream), "b200kv_decode_attn")
    return out
