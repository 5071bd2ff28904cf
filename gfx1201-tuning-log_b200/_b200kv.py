"""ctypes binding of libb200kv.so (the sm_100a kernels behind this directory's
drop-in modules).

The library is the product path: there is no CPU or Triton fallback.  If the
shared object is missing, importing this module raises ImportError with the
build command, so a mis-deployed drop-in fails loudly instead of silently
falling back (the reference's fallbacks exist only in the vLLM override layer,
where they route to vLLM's own stock kernels).

Entry points mirror include/b200kv.h; every call returns a status that
`check()` turns into a RuntimeError naming the call.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("B200KV_LIB", os.path.join(_HERE, "libb200kv.so"))

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"libb200kv.so not found at {LIB_PATH}; build it with `make -C {_HERE}` "
        "(nvcc, sm_100a) or python -c 'import __graft_entry__ as g; g.build()'")

lib = ctypes.CDLL(LIB_PATH)

_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

lib.b200kv_version.restype = _i32
lib.b200kv_version.argtypes = []
lib.b200kv_status_string.restype = ctypes.c_char_p
lib.b200kv_status_string.argtypes = [_i32]
lib.b200kv_last_error.restype = _i32
lib.b200kv_last_error.argtypes = []
lib.b200kv_get_device_status.restype = _i32
lib.b200kv_get_device_status.argtypes = [_vp, ctypes.POINTER(_i32)]
lib.b200kv_reset_device_status.restype = _i32
lib.b200kv_reset_device_status.argtypes = [_vp]

lib.b200kv_mxfp4_gemv.restype = _i32
lib.b200kv_mxfp4_gemv.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]
# identical to the reference binding h4mv/fp8kv_hipw4.py:21-23
lib.h4mv_launch.restype = None
lib.h4mv_launch.argtypes = [_vp] * 4 + [_i32] * 3 + [_vp]

lib.b200kv_decode_attn.restype = _i32
lib.b200kv_decode_attn.argtypes = (
    [_vp, _i64, _i64,                 # q, strides
     _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,  # caches, strides
     _vp, _i64, _i64,                 # out, strides
     _vp, _vp, _vp, _i64,             # qsl, seq_lens, block_table, bt stride
     _vp, _vp, _f32,                  # k_scale, v_scale, sm_scale
     _i32, _i32, _i32, _i32,          # num_seqs, hq, hkv, head_dim
     _i32, _i32, _i32, _i32,          # block_size, num_blocks, max_blocks, max_seq_len_hint
     _i32, _i32, _i32,                # kv_dtype, out_by_qsl, num_splits
     _vp])                            # stream

lib.b200kv_mxfp4_gemm_rope_kv.restype = _i32
lib.b200kv_mxfp4_gemm_rope_kv.argtypes = (
    [_vp, _vp, _vp, _vp, _i32, _i32, _i32,      # W, packed scales, x, qkv, N, K, M
     _vp, _vp, _i32, _vp, _vp, _vp,            # positions, cos_sin, max_pos, slots, k/v cache
     _i64, _i64, _i64, _i64, _i64, _i64,      # cache strides (elements)
     _vp, _vp, _i32, _i32, _i32, _i32, _vp])  # k/v scale, hq, hkv, block_size, kv_dtype, stream

lib.b200kv_decode_step_prep.restype = _i32
lib.b200kv_decode_step_prep.argtypes = [_vp, _vp, _vp, _i32, _i32, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                                        _vp]
lib.b200kv_argmax_rows.restype = _i32
lib.b200kv_argmax_rows.argtypes = [_vp, _i64, _i32, _i32, _vp, _vp, _vp]

lib.b200kv_rmsnorm_residual.restype = _i32
lib.b200kv_rmsnorm_residual.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _f32, _vp]
lib.b200kv_rope_kv_write.restype = _i32
lib.b200kv_rope_kv_write.argtypes = (
    [_vp, _i64, _vp, _vp, _i32, _vp,  # qkv, stride, positions, cos_sin, max_pos, slots
     _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,  # caches, strides (elements)
     _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,  # scales, tokens, hq, hkv, d, block, kv dtype
     _vp])
lib.b200kv_swiglu.restype = _i32
lib.b200kv_swiglu.argtypes = [_vp, _vp, _i32, _i32, _vp]

lib.b200kv_comm_buffer_bytes.restype = ctypes.c_size_t
lib.b200kv_comm_buffer_bytes.argtypes = []
lib.b200kv_comm_alloc.restype = _i32
lib.b200kv_comm_alloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), _vp]
lib.b200kv_comm_open.restype = _i32
lib.b200kv_comm_open.argtypes = [_vp, ctypes.POINTER(ctypes.c_void_p)]
lib.b200kv_comm_close.restype = _i32
lib.b200kv_comm_close.argtypes = [_vp]
lib.b200kv_comm_free.restype = _i32
lib.b200kv_comm_free.argtypes = [_vp]
lib.b200kv_allreduce_oneshot.restype = _i32
lib.b200kv_allreduce_oneshot.argtypes = [_vp, _vp, _i32, ctypes.POINTER(ctypes.c_void_p), _i32, _i32, _vp]

lib.b200kv_prefill_attn.restype = _i32
lib.b200kv_prefill_attn.argtypes = (
    [_vp, _i64, _i64,                 # q, strides
     _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,  # caches, strides
     _vp, _i64, _i64,                 # out, strides
     _vp, _vp, _vp, _i64,             # cu_seqlens_q, seq_lens, block_table, bt stride
     _vp, _vp, _f32,                  # k_scale, v_scale, sm_scale
     _i32, _i32, _i32, _i32,          # num_seqs, max_qlen, q0_single, qlen_single
     _i32, _i32, _i32, _i32,          # hq, hkv, head_dim, block_size
     _i32, _i32, _i32,                # num_blocks, kv_dtype, num_tokens
     _vp])
lib.b200kv_attn_varlen_mixed.restype = _i32
lib.b200kv_attn_varlen_mixed.argtypes = (
    [_vp, _i64, _i64,                 # q, strides
     _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,  # caches, strides
     _vp, _i64, _i64,                 # out, strides
     _vp, _vp, _vp, _i64,             # cu_seqlens_q, seq_lens, block_table, bt stride
     _vp, _vp, _f32,                  # k_scale, v_scale, sm_scale
     _i32, _i32, _i32,                # num_seqs, max_qlen, max_seq_len
     _i32, _i32, _i32, _i32,          # hq, hkv, head_dim, block_size
     _i32, _i32, _i32, _i32,          # num_blocks, max_blocks_per_seq, kv_dtype, num_tokens
     _vp])

lib.b200kv_mxfp4_packed_scales_bytes.restype = ctypes.c_size_t
lib.b200kv_mxfp4_packed_scales_bytes.argtypes = [_i32, _i32]
lib.b200kv_mxfp4_pack_scales.restype = _i32
lib.b200kv_mxfp4_pack_scales.argtypes = [_vp, _i32, _vp, _i32, _i32, _vp, _vp]
lib.b200kv_mxfp4_gemm.restype = _i32
lib.b200kv_mxfp4_gemm.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]
lib.b200kv_mxfp4_gemm_wide_workspace_bytes.restype = ctypes.c_size_t
lib.b200kv_mxfp4_gemm_wide_workspace_bytes.argtypes = [_i32, _i32]
lib.b200kv_mxfp4_gemm_wide.restype = _i32
lib.b200kv_mxfp4_gemm_wide.argtypes = [_vp, _vp, _vp, _i64, _vp, ctypes.c_size_t, _vp, _i32, _i32, _i32, _vp]
lib.b200kv_mxfp4_gemm_swiglu.restype = _i32
lib.b200kv_mxfp4_gemm_swiglu.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]
lib.b200kv_mxfp4_gemm_wide_swiglu.restype = _i32
lib.b200kv_mxfp4_gemm_wide_swiglu.argtypes = [_vp, _vp, _vp, _i64, _vp, ctypes.c_size_t, _vp, _i32, _i32, _i32,
                                              _vp]
lib.b200kv_mxfp4_gemm_allreduce.restype = _i32
lib.b200kv_mxfp4_gemm_allreduce.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _i32, _i32, _vp]
lib.b200kv_mxfp4_gemm_wide_noalloc.restype = _i32
lib.b200kv_mxfp4_gemm_wide_noalloc.argtypes = [_vp, _vp, _vp, _i64, _vp, _i32, _i32, _i32, _vp]



class ChainOp(ctypes.Structure):
    """b200kv_chain_op (include/b200kv.h)."""
    _fields_ = [("weight", _vp), ("packed_scales", _vp), ("x", _vp), ("x_stride", _i64),
                ("out", _vp), ("out_stride", _i64), ("N", ctypes.c_int32), ("K", ctypes.c_int32),
                ("x_from", ctypes.c_int32), ("epilogue", ctypes.c_int32)]


lib.b200kv_mxfp4_chain_workspace_bytes.restype = ctypes.c_size_t
lib.b200kv_mxfp4_chain_workspace_bytes.argtypes = [ctypes.POINTER(ChainOp), _i32, _i32]
lib.b200kv_mxfp4_chain.restype = _i32
lib.b200kv_mxfp4_chain.argtypes = [ctypes.POINTER(ChainOp), _i32, _i32, _vp, ctypes.c_size_t, _vp]
CHAIN_STORE = 0
CHAIN_SWIGLU = 1

lib.b200kv_kv_write.restype = _i32
lib.b200kv_kv_write.argtypes = ([_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp] + [_i64] * 6 +
                                [_vp, _vp, _vp] + [_i32] * 5 + [_vp])

KV_FP8_E4M3 = 0
KV_BF16 = 1


class B200KVError(RuntimeError):
    def __init__(self, what, status):
        self.status = status
        msg = lib.b200kv_status_string(status).decode()
        super().__init__(f"{what} failed: {msg} (status {status})")


def check(status, what):
    if status != 0:
        raise B200KVError(what, status)


def device_status(stream=0):
    """Device-side status word (0 = no kernel hit a bounded-wait limit)."""
    v = _i32(0)
    check(lib.b200kv_get_device_status(_vp(stream), ctypes.byref(v)), "b200kv_get_device_status")
    return v.value


def reset_device_status(stream=0):
    check(lib.b200kv_reset_device_status(_vp(stream)), "b200kv_reset_device_status")
