"""Paged KV-cache write: bf16 key/value rows -> fp8 e4m3 (or bf16) cache slots.

`reshape_and_cache_flash` keeps the argument order and meaning of vLLM's
custom op of the same name (torch.ops._C_cache_ops.reshape_and_cache_flash),
which the reference's engine runs before its attention kernels; the work is
done by csrc/kv_write.cu through b200kv_kv_write.
"""
import torch

from _b200kv import KV_BF16, KV_FP8_E4M3, check, lib


def _scale(s, device):
    if torch.is_tensor(s):
        return s.to(device=device, dtype=torch.float32).reshape(-1)[:1].contiguous()
    return torch.tensor([float(s)], device=device, dtype=torch.float32)


def reshape_and_cache_flash(key, value, key_cache, value_cache, slot_mapping,
                            kv_cache_dtype="fp8", k_scale=1.0, v_scale=1.0):
    """key/value [T, HKV, D] bf16; key/value_cache [NB, PBLK, HKV, D] (fp8 e4m3 or
    bf16, any strides with unit innermost); slot_mapping int64 [T] (-1 = skip)."""
    if key.dtype != torch.bfloat16 or value.dtype != torch.bfloat16:
        raise TypeError("key/value must be bfloat16")
    if key_cache.dtype in (torch.float8_e4m3fn, torch.uint8) and kv_cache_dtype != "auto":
        kv_dtype = KV_FP8_E4M3
    elif key_cache.dtype == torch.bfloat16:
        kv_dtype = KV_BF16
    else:
        raise TypeError(f"unsupported cache dtype {key_cache.dtype} / {kv_cache_dtype}")
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise TypeError("slot_mapping must be a contiguous int64 tensor")
    dev = key.device
    ks, vs = _scale(k_scale, dev), _scale(v_scale, dev)
    T = slot_mapping.numel()
    check(lib.b200kv_kv_write(
        key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
        slot_mapping.data_ptr(), ks.data_ptr(), vs.data_ptr(),
        T, key_cache.shape[2], key_cache.shape[3], key_cache.shape[1], kv_dtype,
        torch.cuda.current_stream(dev).cuda_stream), "b200kv_kv_write")
