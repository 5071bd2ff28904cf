"""Route fp8 per-tensor KV attention in vLLM through the B200 kernels -- the
drop-in for the reference module vllm-fp8kv/fp8kv_override.py.

Importing this module (sitecustomize does it at interpreter start) patches
vllm.v1.attention.backends.triton_attn.TritonAttentionImpl.forward, as the
reference does (fp8kv_override.py:48-109):

  * the gate of fp8kv_override.py:51-62 -- fp8 per-tensor KV, head_size 128,
    no tensor-descriptor path, no sliding window, sinks, ALiBi or soft cap --
    plus what the B200 kernels need (bf16 queries, GQA 1/2/4/8);
  * decode-only batches (max_query_len == 1) run the split-K decode kernel
    (fp8kv_v3.run), the reference's fast path;
  * with FP8KV_PREFILL=1 (the reference's switch, fp8kv_prefill.py:148),
    batches that carry prefill tokens run the varlen causal prefill kernel for
    their prefills and the split-K decode kernel for their one-token
    sequences, split on the device (a decode token is a one-token prefill at
    position seq_len - 1, so the result is the varlen kernel's for the batch),
    where the reference's gate took exactly one sequence
    (fp8kv_prefill.py:159-172);
  * anything else, or any exception, falls back to the wrapped forward;
  * with FP8KV_KVWRITE=1 (not in the reference, which kept vLLM's Triton cache
    write) do_kv_cache_update writes the fp8 cache with csrc/kv_write.cu.

The reference's other patch, swapping vLLM's Triton _cast_kv_tile helper for
a faster fp8 cast on gfx1201 (fp8kv_override.py:15-24), tuned the stock Triton
kernel; here eligible calls never reach that kernel, so it is not needed.
Counters, the one-time diag / ENGAGED lines and the FP8KV_FORCE_TRITON
selector override keep the reference's names (fp8kv_override.py:25-36,65-74,
98-101,122-129).
"""
import os
import sys
import threading

_state = {"installed": False, "counts": None, "prefill": False, "installing": False}


def kv_views(kv_cache, head_size, fp8_dtype):
    """(key_cache, value_cache) views of a vLLM cache tensor.

    vLLM 0.22 stores [NB, 2, PBLK, HKV, D] and splits with unbind(1); the fork
    the reference targeted stored [NB, PBLK, 2, HKV*...] and split the last dim
    after a transpose (fp8kv_override.py:82-85).  Both give stride-generic views
    with unit innermost stride, which is what the kernels take.
    """
    import torch
    if kv_cache.dim() == 5 and kv_cache.shape[1] == 2:
        k, v = kv_cache.unbind(1)
    else:
        k, v = kv_cache.transpose(1, 2).split(head_size, dim=-1)
    if k.dtype != torch.bfloat16 and k.dtype != fp8_dtype:
        k = k.view(fp8_dtype)
        v = v.view(fp8_dtype)
    return k, v


def gate(impl, attn_metadata, query, kv_mode_fp8_per_tensor):
    """The reference's eligibility test (fp8kv_override.py:51-62) plus the B200
    kernel's own limits.  Returns None when eligible, else a short reason."""
    import torch
    try:
        if attn_metadata is None:
            return "no metadata"
        if impl._kv_quant_mode != kv_mode_fp8_per_tensor:
            return "kv quant mode"
        if impl.head_size != 128 or impl.num_kv_heads <= 0:
            return "head size"
        if getattr(impl, "use_td", False):
            return "tensor descriptors"
        if impl.sliding_window[0] >= 0:
            return "sliding window"
        if impl.sinks is not None or impl.alibi_slopes is not None:
            return "sinks/alibi"
        if impl.logits_soft_cap not in (0, None):
            return "soft cap"
        if getattr(attn_metadata, "use_cascade", False):
            return "cascade"
        if getattr(attn_metadata, "mm_prefix_range_tensor", None) is not None:
            return "multimodal prefix range"
        if getattr(impl, "chunk_lookback", -1) != -1:
            return "chunk lookback"
        if getattr(getattr(impl, "attn_type", None), "name", "DECODER") != "DECODER":
            return "attention type"
        if query.dtype != torch.bfloat16:
            return "query dtype"
        if impl.num_queries_per_kv not in (1, 2, 4, 8):
            return "gqa"
    except AttributeError as e:
        return f"missing attribute {e}"
    return None


def kv_write_gate(impl, key, kv_mode_fp8_per_tensor):
    """Eligibility of the cache write (do_kv_cache_update) for csrc/kv_write.cu."""
    import torch
    try:
        if impl._kv_quant_mode != kv_mode_fp8_per_tensor:
            return "kv quant mode"
        if getattr(getattr(impl, "attn_type", None), "name", "DECODER") != "DECODER":
            return "attention type"
        if key.dtype != torch.bfloat16 or impl.head_size % 16:
            return "key dtype / head size"
    except AttributeError as e:
        return f"missing attribute {e}"
    return None


def _install():
    """Patch TritonAttentionImpl once.  fp8kv_prefill._install calls back into
    this function while it is importing (the two modules import each other),
    so a nested call returns at once and the outer call does the work."""
    if _state["installing"]:
        return True
    _state["installing"] = True
    try:
        return _install_impl()
    finally:
        _state["installing"] = False


def _install_impl():
    try:
        from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl
        from vllm.v1.kv_cache_interface import KVQuantMode
    except Exception as e:  # vLLM absent: nothing to patch
        sys.stderr.write(f"[fp8kv-override] install skipped: {e}\n")
        return False
    if getattr(TritonAttentionImpl, "_b200kv_patched", False):
        return True
    import fp8kv_prefill
    import fp8kv_v3

    counts = {"decode": 0, "prefill": 0, "fallback": 0, "fallback_reasons": {}}
    prefill_on = os.environ.get("FP8KV_PREFILL", "0") == "1"
    decode_on = os.environ.get("FP8KV_OVERRIDE", "1") == "1"
    _state["counts"] = counts
    orig = TritonAttentionImpl.forward
    engaged = [0]

    # On CUDA, vLLM 0.22 quantises the query to fp8 before the backend when the
    # KV cache is fp8 and the backend says it takes such queries
    # (supports_quant_query_input, true on CUDA, false on ROCm where the
    # reference ran).  The kernels here take bf16 queries, as the reference's
    # did, so the layers are built without query quantisation; vLLM's own
    # Triton kernel, the fallback, takes bf16 queries too.
    orig_init = TritonAttentionImpl.__init__

    def _init(self, *args, **kwargs):
        orig_init(self, *args, **kwargs)
        self.supports_quant_query_input = False

    _init._b200kv_orig = orig_init
    TritonAttentionImpl.__init__ = _init

    def _forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                 output_scale=None, output_block_scale=None):
        why = gate(self, attn_metadata, query, KVQuantMode.FP8_PER_TENSOR)
        if output_scale is not None or output_block_scale is not None:
            why = why or "output quantisation"
        if why is None and attn_metadata.max_query_len > 1 and not (prefill_on or _state["prefill"]):
            why = "prefill (FP8KV_PREFILL off)"
        if why is None and attn_metadata.max_query_len == 1 and not decode_on:
            why = "decode (FP8KV_OVERRIDE off)"
        if engaged[0] == 0 and attn_metadata is not None:  # the first real batch (not the profiling run)
            engaged[0] = -1
            sys.stderr.write(f"[fp8kv-override] diag: mode={getattr(self, '_kv_quant_mode', None)!r} "
                             f"maxq={getattr(attn_metadata, 'max_query_len', None)} "
                             f"hs={getattr(self, 'head_size', None)} fast_ok={why is None}"
                             f"{'' if why is None else ' (' + why + ')'}\n")
        if why is not None:
            counts["fallback"] += 1
            reasons = counts["fallback_reasons"]
            if why not in reasons and why != "no metadata" and len(reasons) < 16:
                sys.stderr.write(f"[fp8kv-override] fallback: {why}\n")
            reasons[why] = reasons.get(why, 0) + 1
            return orig(self, layer, query, key, value, kv_cache, attn_metadata, output,
                        output_scale, output_block_scale)
        try:
            n = attn_metadata.num_actual_tokens
            hs = self.head_size
            kc, vc = kv_views(kv_cache, hs, self.fp8_dtype)
            q = query[:n]
            out = output[:n]
            if out.dim() == 2:
                out = out.view(n, -1, hs)
            if q.dim() == 2:
                q = q.view(n, -1, hs)
            # the split count is sized from the longest context on the host; a CUDA
            # graph keeps the count it was captured with, so under capture size it
            # for the block table's full width (any context a replay can see)
            import torch
            capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
            hint = 0 if capturing else attn_metadata.max_seq_len
            if attn_metadata.max_query_len == 1:
                fp8kv_v3.run(q, kc, vc, out, attn_metadata.query_start_loc, attn_metadata.seq_lens,
                             attn_metadata.block_table, layer._k_scale, layer._v_scale, self.scale,
                             max_seq_len=hint)
                counts["decode"] += 1
            else:
                # decode tokens of a mixed batch go to the split-K decode kernel,
                # the prefills to the varlen kernel (split on the device)
                fp8kv_prefill.mixed_attention(
                    q, kc, vc, out, attn_metadata.query_start_loc, attn_metadata.seq_lens,
                    attn_metadata.block_table, layer._k_scale, layer._v_scale, self.scale,
                    max_qlen=attn_metadata.max_query_len, max_seq_len=hint)
                counts["prefill"] += 1
            if engaged[0] <= 0:
                engaged[0] = 1
                sys.stderr.write(f"[fp8kv-override] ENGAGED: NS={attn_metadata.query_start_loc.shape[0] - 1} "
                                 f"HKV={self.num_kv_heads} hs={hs} GQA={self.num_queries_per_kv}\n")
            return output
        except Exception as e:
            sys.stderr.write(f"[fp8kv-override] fast path failed ({e!r}), falling back\n")
            counts["fallback"] += 1
            return orig(self, layer, query, key, value, kv_cache, attn_metadata, output,
                        output_scale, output_block_scale)

    _forward._b200kv_orig = orig
    TritonAttentionImpl.forward = _forward
    TritonAttentionImpl._b200kv_patched = True

    if os.environ.get("FP8KV_KVWRITE", "0") == "1" and hasattr(TritonAttentionImpl, "do_kv_cache_update"):
        import kv_cache
        orig_write = TritonAttentionImpl.do_kv_cache_update
        counts["kv_write"] = 0

        def _kv_update(self, layer, key, value, kv_cache_t, slot_mapping):
            if kv_write_gate(self, key, KVQuantMode.FP8_PER_TENSOR) is None:
                try:
                    kc, vc = kv_views(kv_cache_t, self.head_size, self.fp8_dtype)
                    kv_cache.reshape_and_cache_flash(key, value, kc, vc, slot_mapping,
                                                     self.kv_cache_dtype, layer._k_scale, layer._v_scale)
                    counts["kv_write"] += 1
                    return None
                except Exception as e:
                    sys.stderr.write(f"[fp8kv-override] kv write failed ({e!r}), falling back\n")
            return orig_write(self, layer, key, value, kv_cache_t, slot_mapping)

        _kv_update._b200kv_orig = orig_write
        TritonAttentionImpl.do_kv_cache_update = _kv_update

    if os.environ.get("FP8KV_COUNTERS"):
        def _report():
            import time
            while True:
                time.sleep(15)
                sys.stderr.write(f"[fp8kv-override] counters: {counts}\n")
        threading.Thread(target=_report, daemon=True).start()

    if os.environ.get("FP8KV_FORCE_TRITON"):
        try:
            import vllm.v1.attention.selector as _sel
            from vllm.v1.attention.backends.triton_attn import TritonAttentionBackend as _TB
            _sel.get_attn_backend = lambda *a, **kw: _TB
            sys.stderr.write("[fp8kv-override] selector forced to TritonAttentionBackend\n")
        except Exception as e:
            sys.stderr.write(f"[fp8kv-override] force-triton fail {e}\n")

    _state["installed"] = True
    sys.stderr.write("[fp8kv-override] installed\n")
    return True


def enable_prefill():
    """Route prefill batches too (what fp8kv_prefill._install switches on)."""
    _state["prefill"] = True


def uninstall():
    """Restore vLLM's own forward (used by tests)."""
    try:
        from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl
    except Exception:
        return
    f = TritonAttentionImpl.forward
    if getattr(TritonAttentionImpl, "_b200kv_patched", False) and hasattr(f, "_b200kv_orig"):
        TritonAttentionImpl.forward = f._b200kv_orig
        if hasattr(TritonAttentionImpl.__init__, "_b200kv_orig"):
            TritonAttentionImpl.__init__ = TritonAttentionImpl.__init__._b200kv_orig
        TritonAttentionImpl._b200kv_patched = False
        _state["installed"] = False
    w = getattr(TritonAttentionImpl, "do_kv_cache_update", None)
    if w is not None and hasattr(w, "_b200kv_orig"):
        TritonAttentionImpl.do_kv_cache_update = w._b200kv_orig


if os.environ.get("FP8KV_OVERRIDE", "1") == "1":
    _install()
