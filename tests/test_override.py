"""The vLLM drop-in layer on CPU: gates, dispatch and fallback of the
TritonAttentionImpl.forward patch, the radiance::mxfp4_linear override, the
profiler hook and the sitecustomize chain.  Kernel calls are replaced by
recorders here; the kernels themselves are covered by the -m gpu tests."""
import os
import subprocess
import sys
import types

import pytest
import torch

from conftest import PKG

pytest.importorskip("vllm")


def _impl(**kw):
    from vllm.v1.kv_cache_interface import KVQuantMode
    d = dict(_kv_quant_mode=KVQuantMode.FP8_PER_TENSOR, head_size=128, num_kv_heads=8,
             num_queries_per_kv=4, use_td=False, sliding_window=(-1, -1), sinks=None,
             alibi_slopes=None, logits_soft_cap=0, chunk_lookback=-1,
             attn_type=types.SimpleNamespace(name="DECODER"), fp8_dtype=torch.float8_e4m3fn,
             scale=0.088, kv_cache_dtype="fp8")
    d.update(kw)
    return types.SimpleNamespace(**d)


def _meta(ns=2, maxq=1, **kw):
    qsl = torch.arange(ns + 1, dtype=torch.int32) * maxq
    d = dict(num_actual_tokens=ns * maxq, max_query_len=maxq, query_start_loc=qsl,
             max_seq_len=100, seq_lens=torch.full((ns,), 100, dtype=torch.int32),
             block_table=torch.zeros((ns, 8), dtype=torch.int32), use_cascade=False,
             mm_prefix_range_tensor=None, slot_mapping=torch.arange(ns * maxq))
    d.update(kw)
    return types.SimpleNamespace(**d)


@pytest.fixture
def override(libpath, monkeypatch):
    """fp8kv_override installed over a recording stand-in of vLLM's forward."""
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl
    import fp8kv_override
    fp8kv_override.uninstall()
    real_fwd = TritonAttentionImpl.forward
    real_kvu = TritonAttentionImpl.do_kv_cache_update
    calls = {"orig": 0, "decode": [], "prefill": [], "kvw": [], "orig_kvw": 0}

    def fake_orig(self, layer, query, key, value, kv_cache, md, output, os_=None, obs=None):
        calls["orig"] += 1
        return output

    def fake_orig_kvw(self, layer, key, value, kv_cache, slot_mapping):
        calls["orig_kvw"] += 1

    TritonAttentionImpl.forward = fake_orig
    TritonAttentionImpl.do_kv_cache_update = fake_orig_kvw
    import fp8kv_prefill
    import fp8kv_v3
    import kv_cache
    monkeypatch.setattr(fp8kv_v3, "run", lambda *a, **k: calls["decode"].append((a, k)))
    monkeypatch.setattr(fp8kv_prefill, "mixed_attention", lambda *a, **k: calls["prefill"].append((a, k)))
    monkeypatch.setattr(kv_cache, "reshape_and_cache_flash", lambda *a, **k: calls["kvw"].append(a))
    monkeypatch.setenv("FP8KV_KVWRITE", "1")
    assert fp8kv_override._install()
    yield fp8kv_override, TritonAttentionImpl, calls
    fp8kv_override.uninstall()
    fp8kv_override._state["prefill"] = False
    TritonAttentionImpl.forward = real_fwd
    TritonAttentionImpl.do_kv_cache_update = real_kvu


def _tensors(ntok, hq=32, hkv=8, nb=4):
    q = torch.zeros((ntok, hq, 128), dtype=torch.bfloat16)
    kv = torch.zeros((nb, 2, 16, hkv, 128), dtype=torch.uint8)
    out = torch.zeros((ntok, hq, 128), dtype=torch.bfloat16)
    layer = types.SimpleNamespace(_k_scale=torch.ones(1), _v_scale=torch.ones(1))
    return q, kv, out, layer


def test_gate_accepts_reference_case():
    import fp8kv_override
    from vllm.v1.kv_cache_interface import KVQuantMode
    q = torch.zeros((2, 32, 128), dtype=torch.bfloat16)
    assert fp8kv_override.gate(_impl(), _meta(), q, KVQuantMode.FP8_PER_TENSOR) is None


@pytest.mark.parametrize("field,value,reason", [
    ("head_size", 64, "head size"),
    ("use_td", True, "tensor descriptors"),
    ("sliding_window", (127, 0), "sliding window"),
    ("sinks", torch.zeros(32), "sinks/alibi"),
    ("alibi_slopes", torch.zeros(32), "sinks/alibi"),
    ("logits_soft_cap", 30.0, "soft cap"),
    ("chunk_lookback", 4, "chunk lookback"),
    ("num_queries_per_kv", 16, "gqa"),
    ("attn_type", types.SimpleNamespace(name="ENCODER_ONLY"), "attention type"),
])
def test_gate_rejects(field, value, reason):
    import fp8kv_override
    from vllm.v1.kv_cache_interface import KVQuantMode
    q = torch.zeros((2, 32, 128), dtype=torch.bfloat16)
    assert fp8kv_override.gate(_impl(**{field: value}), _meta(), q, KVQuantMode.FP8_PER_TENSOR) == reason


def test_gate_rejects_metadata_and_dtype():
    import fp8kv_override
    from vllm.v1.kv_cache_interface import KVQuantMode
    q = torch.zeros((2, 32, 128), dtype=torch.bfloat16)
    mode = KVQuantMode.FP8_PER_TENSOR
    assert fp8kv_override.gate(_impl(), None, q, mode) == "no metadata"
    assert fp8kv_override.gate(_impl(), _meta(use_cascade=True), q, mode) == "cascade"
    assert fp8kv_override.gate(_impl(), _meta(mm_prefix_range_tensor=torch.zeros(1)), q, mode) \
        == "multimodal prefix range"
    assert fp8kv_override.gate(_impl(), _meta(), q.half(), mode) == "query dtype"
    other = [m for m in KVQuantMode if m != mode][0]
    assert fp8kv_override.gate(_impl(_kv_quant_mode=other), _meta(), q, mode) == "kv quant mode"


def test_kv_views_vllm_layout():
    import fp8kv_override
    kv = torch.zeros((5, 2, 16, 8, 128), dtype=torch.uint8)
    k, v = fp8kv_override.kv_views(kv, 128, torch.float8_e4m3fn)
    assert k.shape == v.shape == (5, 16, 8, 128)
    assert k.dtype == torch.float8_e4m3fn and k.stride(-1) == 1
    assert v.data_ptr() - k.data_ptr() == 16 * 8 * 128
    kb = torch.zeros((5, 2, 16, 8, 128), dtype=torch.bfloat16)
    k2, _ = fp8kv_override.kv_views(kb, 128, torch.float8_e4m3fn)
    assert k2.dtype == torch.bfloat16


def test_decode_batch_routed_to_decode_kernel(override):
    mod, cls, calls = override
    q, kv, out, layer = _tensors(2)
    md = _meta(ns=2, maxq=1)
    r = cls.forward(_impl(), layer, q, None, None, kv, md, out)
    assert r is out and calls["orig"] == 0 and len(calls["decode"]) == 1
    a, k = calls["decode"][0]
    assert a[0].shape == (2, 32, 128) and a[1].dtype == torch.float8_e4m3fn
    assert a[4] is md.query_start_loc and a[5] is md.seq_lens and a[6] is md.block_table
    assert k["max_seq_len"] == 100
    assert mod._state["counts"]["decode"] == 1


def test_2d_output_view(override):
    _, cls, calls = override
    q, kv, out, layer = _tensors(2)
    out2 = out.view(2, -1)
    cls.forward(_impl(), layer, q.view(2, -1), None, None, kv, _meta(ns=2, maxq=1), out2)
    a, _ = calls["decode"][0]
    assert a[0].shape == (2, 32, 128) and a[3].shape == (2, 32, 128)


def test_prefill_falls_back_unless_enabled(override):
    mod, cls, calls = override
    q, kv, out, layer = _tensors(8)
    md = _meta(ns=2, maxq=4)
    cls.forward(_impl(), layer, q, None, None, kv, md, out)
    assert calls["orig"] == 1 and not calls["prefill"]
    mod.enable_prefill()
    cls.forward(_impl(), layer, q, None, None, kv, md, out)
    assert calls["orig"] == 1 and len(calls["prefill"]) == 1
    a, k = calls["prefill"][0]
    assert a[4] is md.query_start_loc and k["max_qlen"] == 4 and k["max_seq_len"] == md.max_seq_len


def test_ineligible_and_failing_calls_fall_back(override, monkeypatch):
    _, cls, calls = override
    q, kv, out, layer = _tensors(2)
    cls.forward(_impl(head_size=64), layer, q, None, None, kv, _meta(), out)
    assert calls["orig"] == 1
    cls.forward(_impl(), layer, q, None, None, kv, _meta(), out, torch.ones(1))
    assert calls["orig"] == 2

    import fp8kv_v3

    def boom(*a, **k):
        raise RuntimeError("kernel refused")
    monkeypatch.setattr(fp8kv_v3, "run", boom)
    cls.forward(_impl(), layer, q, None, None, kv, _meta(), out)
    assert calls["orig"] == 3


def test_kv_cache_update_patch(override):
    _, cls, calls = override
    key = torch.zeros((3, 8, 128), dtype=torch.bfloat16)
    kv = torch.zeros((4, 2, 16, 8, 128), dtype=torch.uint8)
    layer = types.SimpleNamespace(_k_scale=torch.ones(1), _v_scale=torch.ones(1))
    slots = torch.arange(3)
    cls.do_kv_cache_update(_impl(), layer, key, key, kv, slots)
    assert len(calls["kvw"]) == 1 and calls["orig_kvw"] == 0
    a = calls["kvw"][0]
    assert a[2].shape == (4, 16, 8, 128) and a[2].dtype == torch.float8_e4m3fn and a[4] is slots
    cls.do_kv_cache_update(_impl(), layer, key.half(), key.half(), kv, slots)
    assert calls["orig_kvw"] == 1


def test_install_is_idempotent_and_uninstall_restores(override):
    mod, cls, _ = override
    fwd = cls.forward
    assert mod._install()
    assert cls.forward is fwd
    orig = fwd._b200kv_orig
    mod.uninstall()
    assert cls.forward is orig


def test_hipw4_gate_and_repack(libpath):
    import fp8kv_hipw4 as hw
    N, K = 64, 256
    w = torch.zeros((N, K // 2), dtype=torch.uint8)
    s = torch.arange(K // 32 * N, dtype=torch.int64).remainder(255).to(torch.uint8).view(K // 32, N)
    x = torch.zeros((2, K), dtype=torch.bfloat16)
    assert hw.eligible(x, w, s, 4)
    assert not hw.eligible(torch.zeros((5, K), dtype=torch.bfloat16), w, s, 4)
    assert not hw.eligible(x.half(), w, s, 4)
    assert not hw.eligible(torch.zeros((2, 2 * K), dtype=torch.bfloat16)[:, ::2], w, s, 4)
    assert not hw.eligible(x, w, s[:-1], 4)
    assert not hw.eligible(x, torch.zeros((4, K // 2), dtype=torch.uint8), torch.zeros((K // 32, 4), dtype=torch.uint8), 4)
    st = hw.scale_t_for(s)
    assert st.shape == (N, K // 32) and st.is_contiguous() and torch.equal(st, s.t())
    assert hw.scale_t_for(s) is st


def test_hipw4_patched_routes(libpath, monkeypatch):
    """Weights whose scales cannot take the tensor-core path (packed_scales_for
    gives False) run the CUDA-core kernel with the transposed scales."""
    import fp8kv_hipw4 as hw
    import h4mv
    seen = {"fast": [], "body": 0}
    monkeypatch.setattr(hw, "packed_scales_for", lambda s, N, K: False)
    monkeypatch.setattr(h4mv, "mxfp4_gemv", lambda x, w, st: seen["fast"].append((x.shape, st.shape)) or "fast")

    def body(x, w, s, wref):
        seen["body"] += 1
        return "body"
    f = hw.make_patched(body, 4)
    N, K = 32, 128
    w = torch.zeros((N, K // 2), dtype=torch.uint8)
    s = torch.zeros((K // 32, N), dtype=torch.uint8)
    assert f(torch.zeros((1, K), dtype=torch.bfloat16), w, s, None) == "fast"
    assert seen["fast"][0] == ((1, K), (N, K // 32))
    assert f(torch.zeros((16, K), dtype=torch.bfloat16), w, s, None) == "body"

    def boom(*a):
        raise RuntimeError("launch failed")
    monkeypatch.setattr(h4mv, "mxfp4_gemv", boom)
    assert f(torch.zeros((1, K), dtype=torch.bfloat16), w, s, None) == "body"
    assert seen["body"] == 2


def test_hipw4_prefers_tensor_core_path(libpath, monkeypatch):
    import fp8kv_hipw4 as hw
    import h4mv
    seen = []
    packed = torch.zeros(4, dtype=torch.uint8)
    monkeypatch.setattr(hw, "packed_scales_for", lambda s, N, K: packed)
    monkeypatch.setattr(h4mv, "mxfp4_gemm", lambda x, w, p: seen.append(p is packed) or "tc")
    monkeypatch.setattr(h4mv, "mxfp4_gemv", lambda *a, **k: "cuda-core")
    f = hw.make_patched(lambda *a: "body", 4)
    N, K = 32, 256
    out = f(torch.zeros((2, K), dtype=torch.bfloat16), torch.zeros((N, K // 2), dtype=torch.uint8),
            torch.zeros((K // 32, N), dtype=torch.uint8), None)
    assert out == "tc" and seen == [True]


def test_hipw4_chunked_body_covers_any_m(libpath, monkeypatch):
    import fp8kv_hipw4 as hw
    import h4mv
    rows = []

    def rec(x, w, st, out=None):
        rows.append((x.shape[0], out.shape[0], x.is_contiguous(), out.is_contiguous()))
        return out
    monkeypatch.setattr(h4mv, "mxfp4_gemv", rec)
    N, K = 16, 64
    out = hw.mxfp4_linear_chunked(torch.zeros((19, K), dtype=torch.bfloat16),
                                  torch.zeros((N, K // 2), dtype=torch.uint8),
                                  torch.zeros((K // 32, N), dtype=torch.uint8))
    assert out.shape == (19, N)
    assert rows == [(8, 8, True, True), (8, 8, True, True), (3, 3, True, True)]


def test_hipw4_chunked_body_takes_wide_gemm(libpath, monkeypatch):
    """M > 8 with scales that pack goes to the wide-batch tensor-core GEMM."""
    import fp8kv_hipw4 as hw
    import h4mv
    packed = torch.zeros(4, dtype=torch.uint8)
    seen = []
    monkeypatch.setattr(hw, "packed_scales_for", lambda s, N, K: packed)
    monkeypatch.setattr(h4mv, "mxfp4_gemm_wide", lambda x, w, p: seen.append((tuple(x.shape), p is packed)) or "wide")
    monkeypatch.setattr(h4mv, "mxfp4_gemv", lambda *a, **k: "slices")
    N, K = 16, 256
    w = torch.zeros((N, K // 2), dtype=torch.uint8)
    s = torch.zeros((K // 32, N), dtype=torch.uint8)
    assert hw.mxfp4_linear_chunked(torch.zeros((19, K), dtype=torch.bfloat16), w, s) == "wide"
    assert seen == [((19, K), True)]


def test_hipw4_defines_op_when_fork_absent():
    env = dict(os.environ, FP8KV_HIPW4="1", FP8KV_OVERRIDE="0", PYTHONPATH=PKG)
    code = ("import torch, fp8kv_hipw4 as hw; "
            "x=torch.empty((3,256),dtype=torch.bfloat16,device='meta'); "
            "w=torch.empty((64,128),dtype=torch.uint8,device='meta'); "
            "s=torch.empty((8,64),dtype=torch.uint8,device='meta'); "
            "y=torch.ops.radiance.mxfp4_linear(x,w,s,w); "
            "print('SHAPE', tuple(y.shape), y.dtype, hw._state['installed'])")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "SHAPE (3, 64) torch.bfloat16 True" in r.stdout
    assert "[hipw4] installed (radiance op defined here)" in r.stderr


def test_profhook_window(tmp_path):
    import fp8kv_profhook as ph
    ph._state.update(step=0, prof=None, done=False)
    out = tmp_path / "prof.txt"
    steps = []
    f = ph.wrap_step(lambda i: steps.append(i) or torch.ones(64).sum(), 2, 3, str(out))
    for i in range(7):
        f(i)
    assert steps == list(range(7))
    assert ph._state["done"] and out.exists()
    assert "steps=3 device_busy_ms=" in out.read_text()


def test_sitecustomize_chain_patches_once():
    """sitecustomize with FP8KV_PREFILL=1: the two modules import each other;
    the forward must be wrapped exactly once, over vLLM's own function."""
    env = dict(os.environ, FP8KV_PREFILL="1", FP8KV_OVERRIDE="1", PYTHONPATH=PKG)
    code = ("from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl as T; "
            "f=T.forward; o=f._b200kv_orig; "
            "print('WRAPPED', hasattr(f,'_b200kv_orig'), hasattr(o,'_b200kv_orig'), "
            "o.__module__)")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "WRAPPED True False vllm.v1.attention.backends.triton_attn" in r.stdout
    assert "[fp8kv-override] installed" in r.stderr
    assert "[fp8kv-prefill] installed" in r.stderr


def test_wide_workspace_is_never_freed_when_outgrown(libpath, monkeypatch):
    """A graph captured with a smaller workspace keeps writing to it, so growing
    the per-stream workspace must keep the old one alive."""
    import h4mv

    class _Stream:
        cuda_stream = 12345

    class _Dev:
        index = 99
    orig = torch.empty
    monkeypatch.setattr(h4mv.torch, "empty", lambda n, dtype=None, device=None: orig(n, dtype=dtype))
    monkeypatch.setattr(h4mv, "_workspaces", {})
    monkeypatch.setattr(h4mv, "_outgrown", [])
    a = h4mv.wide_workspace(64, 256, _Dev(), _Stream())
    b = h4mv.wide_workspace(200, 256, _Dev(), _Stream())
    c = h4mv.wide_workspace(100, 256, _Dev(), _Stream())
    assert b.numel() > a.numel() and c is b
    assert any(t is a for t in h4mv._outgrown)


def test_hipw4_hooks_vllm_quark_w4a16_scheme():
    """With FP8KV_HIPW4=1 the module also hooks vLLM's Quark OCP-MX scheme
    (W4A16 MXFP4 layers: load-time prepack, apply through the op); the hook is
    idempotent and leaves CPU layers to the scheme's own path."""
    env = dict(os.environ, FP8KV_HIPW4="1", FP8KV_OVERRIDE="0", PYTHONPATH=PKG)
    code = ("import torch, fp8kv_hipw4 as hw; "
            "from vllm.model_executor.layers.quantization.quark.schemes.quark_ocp_mx import QuarkOCP_MX as Q; "
            "assert Q._b200kv_hooked and hw.install_quark_hook(); "
            "s = Q({'dtype': 'fp4', 'qscheme': 'per_group', 'group_size': 32}, None); "
            "assert hw._w4a16_mxfp4(s); "
            "l = torch.nn.Module(); "
            "l.weight = torch.nn.Parameter(torch.zeros(64, 128, dtype=torch.uint8), requires_grad=False); "
            "l.weight_scale = torch.nn.Parameter(torch.zeros(64, 8, dtype=torch.uint8), requires_grad=False); "
            "s.process_weights_after_loading(l); "
            "print('CKPT', hasattr(l, '_b200kv_scale_ckpt'))")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "CKPT False" in r.stdout
    assert "[hipw4] quark W4A16 MXFP4 hook installed" in r.stderr


def test_layers_keep_bf16_queries(override):
    """vLLM 0.22 on CUDA would quantise the query to fp8 before an fp8-KV
    backend that reports supports_quant_query_input (true on CUDA, false on
    the reference's ROCm); the installed patch builds every impl with it off,
    so the kernels get bf16 queries, and uninstall restores vLLM's __init__."""
    mod, cls, _ = override
    assert hasattr(cls.__init__, "_b200kv_orig")
    impl = cls(num_heads=4, head_size=128, scale=0.088, num_kv_heads=1, alibi_slopes=None,
               sliding_window=None, kv_cache_dtype="fp8")
    assert impl.supports_quant_query_input is False
    orig = cls.__init__._b200kv_orig
    mod.uninstall()
    assert cls.__init__ is orig


def test_split_hint_dropped_under_graph_capture(override, monkeypatch):
    """Under CUDA-graph capture the host's max_seq_len is the capture batch's,
    and a replay keeps the split count it sizes; the patch passes no hint then,
    so the kernel sizes the split for the block table's full width."""
    mod, cls, calls = override
    q, kv, out, layer = _tensors(2)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    cls.forward(_impl(), layer, q, None, None, kv, _meta(ns=2, maxq=1), out)
    assert calls["decode"][-1][1]["max_seq_len"] == 0
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    cls.forward(_impl(), layer, q, None, None, kv, _meta(ns=2, maxq=1), out)
    assert calls["decode"][-1][1]["max_seq_len"] == 100
