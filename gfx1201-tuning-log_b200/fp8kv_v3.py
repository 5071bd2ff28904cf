"""fp8 paged-KV split-K decode attention -- drop-in for the reference module
vllm-fp8kv/fp8kv_v3.py (`run` at :116-139), backed by sm_100a kernels instead
of the two Triton kernels: csrc/decode_tma.cu (TMA page tiles) for fp8 caches,
csrc/decode_attn.cu (per-row gathers) for bf16 caches and for fp8 layouts that
no tensor map describes.

Same signature and argument meaning.  Differences a caller can observe:
  * TILE / warps / stages are accepted and ignored (they tuned the Triton
    kernel's tile shape); `nsplit` is a split-count request -- None (default)
    lets the library size the splits for the B200's 148 SMs, an int asks for
    that many CTAs per (sequence, kv head), rounded up to a power of two <= 16.
  * `scratch` is accepted and ignored: the split partials are merged inside a
    thread-block cluster through distributed shared memory, so the kernel
    needs no global scratch.
  * `max_seq_len` (extra, optional) is a host-side bound on seq_lens used to
    size the splits; without it the block table width bounds the context.
  * Sequences with seq_len == 0 produce zeros (the reference divides 0 by 0).
Like the reference, the output row of sequence s is `out[s]` (fp8kv_v3.py:112).
"""
from _decode import decode_attention


def run(q, k_cache, v_cache, out, qsl, slens, bt, kscale, vscale, sm_scale,
        TILE=32, warps=4, stages=3, nsplit=None, scratch=None, max_seq_len=0):
    decode_attention(q, k_cache, v_cache, out, qsl, slens, bt, kscale, vscale, sm_scale,
                     out_by_qsl=False, num_splits=int(nsplit or 0),
                     max_seq_len_hint=int(max_seq_len or 0))
