"""The vLLM drop-in layer on the B200: TritonAttentionImpl.forward patched by
fp8kv_override (decode, varlen prefill + decode mix, KV-cache write) over a
vLLM-layout cache [NB, 2, PBLK, HKV, D], and radiance::mxfp4_linear routed
by fp8kv_hipw4, each against the CPU oracle with the kernels' own tolerances
(attention: max abs < 0.05 and rel-to-max < 2e-2; matvec: rel-to-max < 5e-3)."""
import types

import pytest
import torch

import fp8kv_oracle as FO
import mxfp4_oracle as MO

pytestmark = pytest.mark.gpu

HQ, HKV, D, PBLK = 32, 8, 128, 16


def _impl():
    from vllm.v1.kv_cache_interface import KVQuantMode
    return types.SimpleNamespace(
        _kv_quant_mode=KVQuantMode.FP8_PER_TENSOR, head_size=D, num_kv_heads=HKV,
        num_queries_per_kv=HQ // HKV, use_td=False, sliding_window=(-1, -1), sinks=None,
        alibi_slopes=None, logits_soft_cap=0, chunk_lookback=-1,
        attn_type=types.SimpleNamespace(name="DECODER"), fp8_dtype=torch.float8_e4m3fn,
        scale=D ** -0.5, kv_cache_dtype="fp8")


def _vllm_cache(k, v):
    return torch.stack([k.view(torch.uint8), v.view(torch.uint8)], dim=1)


def _check(got, ref):
    got = got.float().cpu()
    err = (got - ref).abs().max().item()
    rel = err / max(ref.abs().max().item(), 1e-30)
    assert err < 0.05 and rel < 2e-2, (err, rel)


@pytest.fixture
def patched(cuda, monkeypatch):
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl
    import fp8kv_override
    fp8kv_override.uninstall()
    monkeypatch.setenv("FP8KV_KVWRITE", "1")
    assert fp8kv_override._install()
    yield fp8kv_override, TritonAttentionImpl
    fp8kv_override.uninstall()
    fp8kv_override._state["prefill"] = False


def test_forward_decode_batch(patched):
    mod, cls = patched
    c = FO.make_decode_case(6, [1, 17, 300, 1024, 2049, 64], seed=11)
    dev = torch.device("cuda", 0)
    kv = _vllm_cache(c["k_cache"], c["v_cache"]).to(dev)
    q = c["q"].to(dev)
    out = torch.full_like(q, float("nan"))
    md = types.SimpleNamespace(num_actual_tokens=6, max_query_len=1, query_start_loc=c["qsl"].to(dev),
                               max_seq_len=2049, seq_lens=c["seq_lens"].to(dev),
                               block_table=c["block_table"].to(dev), use_cascade=False,
                               mm_prefix_range_tensor=None)
    layer = types.SimpleNamespace(_k_scale=torch.tensor([c["k_scale"]], device=dev),
                                  _v_scale=torch.tensor([c["v_scale"]], device=dev))
    before = dict(mod._state["counts"])
    cls.forward(_impl(), layer, q, None, None, kv, md, out)
    torch.cuda.synchronize()
    assert mod._state["counts"]["decode"] == before["decode"] + 1
    assert mod._state["counts"]["fallback"] == before["fallback"]
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


def test_forward_mixed_prefill_decode_and_kv_write(patched):
    """One engine step: new tokens of three sequences (a 130-token chunk on top
    of 170 cached, a 1-token decode, a fresh 5-token prompt) are written to the
    cache by do_kv_cache_update, then attended by forward."""
    mod, cls = patched
    mod.enable_prefill()
    dev = torch.device("cuda", 0)
    qlens, lens = [130, 1, 5], [300, 77, 5]
    g = torch.Generator().manual_seed(5)
    nblk = [(L + PBLK - 1) // PBLK for L in lens]
    nb = sum(nblk) + 4
    kf, vf = torch.randn(nb, PBLK, HKV, D, generator=g), torch.randn(nb, PBLK, HKV, D, generator=g)
    kc, ks = FO.quantize_fp8_per_tensor(kf)
    vc, vs = FO.quantize_fp8_per_tensor(vf)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(3, max(nblk), dtype=torch.int32)
    p = 0
    for s, n in enumerate(nblk):
        bt[s, :n] = perm[p:p + n]
        p += n
    T = sum(qlens)
    cu = torch.tensor([0, 130, 131, 136], dtype=torch.int32)
    key = (torch.randn(T, HKV, D, generator=g) * 0.5).to(torch.bfloat16)
    val = (torch.randn(T, HKV, D, generator=g) * 0.5).to(torch.bfloat16)
    slots = []
    for s in range(3):
        for i in range(qlens[s]):
            pos = lens[s] - qlens[s] + i
            slots.append(int(bt[s, pos // PBLK]) * PBLK + pos % PBLK)
    slots = torch.tensor(slots, dtype=torch.int64)
    q = torch.randn(T, HQ, D, generator=g).to(torch.bfloat16)

    kv = _vllm_cache(kc, vc).to(dev)
    layer = types.SimpleNamespace(_k_scale=torch.tensor([ks], device=dev),
                                  _v_scale=torch.tensor([vs], device=dev))
    before = dict(mod._state["counts"])
    cls.do_kv_cache_update(_impl(), layer, key.to(dev), val.to(dev), kv, slots.to(dev))
    md = types.SimpleNamespace(num_actual_tokens=T, max_query_len=130, query_start_loc=cu.to(dev),
                               max_seq_len=300, seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
                               block_table=bt.to(dev), use_cascade=False, mm_prefix_range_tensor=None)
    out = torch.full((T, HQ, D), float("nan"), dtype=torch.bfloat16, device=dev)
    cls.forward(_impl(), layer, q.to(dev), None, None, kv, md, out)
    torch.cuda.synchronize()
    c = mod._state["counts"]
    assert c["kv_write"] == before.get("kv_write", 0) + 1 and c["prefill"] == before["prefill"] + 1
    assert c["fallback"] == before["fallback"]

    kv_cpu = kv.cpu()
    k_after = kv_cpu[:, 0].view(torch.float8_e4m3fn)
    v_after = kv_cpu[:, 1].view(torch.float8_e4m3fn)
    kq = (key.float() / ks).to(torch.float8_e4m3fn)
    flat = k_after.reshape(-1, HKV, D)
    assert torch.equal(flat[slots].view(torch.uint8), kq.view(torch.uint8))
    ref = FO.prefill_reference(q, k_after, v_after, cu, torch.tensor(lens, dtype=torch.int32), bt,
                               ks, vs, D ** -0.5)
    _check(out, ref)


def test_radiance_op_routes_to_b200_matvec(cuda, monkeypatch):
    monkeypatch.setenv("FP8KV_HIPW4", "1")
    import fp8kv_hipw4 as hw
    assert hw._install()
    N, K = 1024, 2048
    for M in (1, 4, 8, 19):
        W, S, St, X = MO.make_case(N, K, M, seed=M)
        ref = MO.mxfp4_linear_reference(W, S, X)
        fast0, slow0 = hw._state["fast"], hw._state["slow"]
        y = torch.ops.radiance.mxfp4_linear(X.to(cuda), W.to(cuda), S.to(cuda), W.to(cuda))
        torch.cuda.synchronize()
        assert y.shape == (M, N) and y.dtype == torch.bfloat16
        assert MO.rel_to_max_err(y.float().cpu(), ref) < 5e-3, M
        if M <= hw.max_m():
            assert hw._state["fast"] == fast0 + 1
        else:
            assert hw._state["slow"] == slow0 + 1


def test_quark_w4a16_layer_prepacked_at_load_and_graph_capturable(cuda, monkeypatch):
    """vLLM's Quark OCP-MX scheme on a W4A16 MXFP4 layer as the engine loads it
    (weight [N, K/2], scales [N, K/32]): process_weights_after_loading (hooked)
    packs the scale atoms, so a CUDA-graph capture of apply_weights needs no
    lazy repack; results within two bf16 roundings of the oracle (the product
    and the bias add) for M = 1, 4 and a 3-D batch of 12 tokens, bias added."""
    monkeypatch.setenv("FP8KV_HIPW4", "1")
    import fp8kv_hipw4 as hw
    assert hw._install() and hw.install_quark_hook()
    from vllm.model_executor.layers.quantization.quark.schemes.quark_ocp_mx import QuarkOCP_MX
    scheme = QuarkOCP_MX({"dtype": "fp4", "qscheme": "per_group", "group_size": 32}, None)
    N, K = 1024, 2048
    W, S, St, _ = MO.make_case(N, K, 1, seed=3)
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(W.to(cuda), requires_grad=False)
    layer.weight_scale = torch.nn.Parameter(St.to(cuda), requires_grad=False)
    scheme.process_weights_after_loading(layer)
    ckpt = layer._b200kv_scale_ckpt
    assert tuple(ckpt.shape) == (K // 32, N)
    assert ("p", ckpt.data_ptr(), tuple(ckpt.shape), ckpt.device) in hw._repack_cache
    g = torch.Generator().manual_seed(17)
    bias = torch.randn(N, generator=g).to(torch.bfloat16).to(cuda)
    # apply_weights rounds to bf16 twice, the product and then the bias add,
    # each by at most 2^-8 of the value: 1e-2 of the maximum bounds both
    tol = 1e-2
    for shape in ((1, K), (4, K), (3, 4, K)):
        x = torch.randn(*shape, generator=g).to(torch.bfloat16).to(cuda)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                y = scheme.apply_weights(layer, x, bias)
        torch.cuda.current_stream().wait_stream(s)
        graph.replay()
        torch.cuda.synchronize()
        assert tuple(y.shape) == shape[:-1] + (N,)
        ref = MO.mxfp4_linear_reference(W, S, x.reshape(-1, K).cpu()) + bias.float().cpu()
        assert MO.rel_to_max_err(y.reshape(-1, N).float().cpu(), ref) < tol, shape
