"""Single-call fp8/bf16 paged-KV decode attention -- drop-in for the reference
module vllm-fp8kv/fp8kv_kernel.py (`run` at :75-88).

The reference ran one CTA per (sequence, kv head) and folded k_scale on the
host with float(kscale), a device->host sync (fp8kv_kernel.py:82).  Here the
same call goes to the sm_100a split-K kernel (csrc/decode_attn.cu), which reads
both scales on the device, so the call never synchronises and is CUDA-graph
capturable.  KV caches may be fp8 e4m3 (scales applied) or bf16 (scales
ignored), as in the reference's K_FP8 switch.  The output row of sequence s is
out[qsl[s]] (fp8kv_kernel.py:70).  TILE / warps / stages are accepted and
ignored.
"""
from _decode import decode_attention


def run(q, k_cache, v_cache, out, qsl, slens, bt, kscale, vscale, sm_scale,
        TILE=64, warps=4, stages=3):
    decode_attention(q, k_cache, v_cache, out, qsl, slens, bt, kscale, vscale, sm_scale,
                     out_by_qsl=True)
