"""fp8 paged-KV split-K decode attention -- drop-in for the reference module
vllm-fp8kv/fp8kv_v3.py (`run` at :116-139), backed by the sm_100a kernel in
csrc/decode_attn.cu instead of the two Triton kernels.

Same signature and argument meaning.  Differences a caller can observe:
  * TILE / warps / stages are accepted and ignored (they tuned the Triton
    kernel's tile shape); `nsplit` is a split-count request -- None (default)
    lets the library size the splits for the B200's 148 SMs, an int asks for
    that many spans of the context bound, each capped at 256 tokens.
  * `scratch` may be a DecodeWorkspace (or None for the per-device default).
    The reference's 3-tuple of fp32 buffers is accepted and ignored: the
    partials live in the library workspace.
  * Sequences with seq_len == 0 produce zeros (the reference divides 0 by 0).
Like the reference, the output row of sequence s is `out[s]` (fp8kv_v3.py:112).
"""
from _decode import DecodeWorkspace, decode_attention


def run(q, k_cache, v_cache, out, qsl, slens, bt, kscale, vscale, sm_scale,
        TILE=32, warps=4, stages=3, nsplit=None, scratch=None, max_seq_len=0):
    ws = scratch if isinstance(scratch, DecodeWorkspace) else None
    decode_attention(q, k_cache, v_cache, out, qsl, slens, bt, kscale, vscale, sm_scale,
                     out_by_qsl=False, num_splits=int(nsplit or 0),
                     max_seq_len_hint=int(max_seq_len or 0), workspace=ws)
