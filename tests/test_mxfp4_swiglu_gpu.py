"""gate_up with the SwiGLU epilogue (b200kv_mxfp4_gemm_swiglu for M <= 8,
b200kv_mxfp4_gemm_wide_swiglu for wide batches) on the B200.

The epilogue's contract is bit equality with the unfused path on the same
weights: the plain GEMM of the [gate | up] rows followed by b200kv_swiglu
(bf16(bf16(silu(g)) * u), HF Llama's act_fn(gate) * up rounded as the decoder
rounds it), with the fused kernel given the rows in gate_up_row_order and the
scales packed after that permutation and the same K-split (the order of the
fp32 sum).  Checked over M, over every K-split the M <= 8 kernel can be
forced to (the finishing rank pairs gate and up rows from the partials of all
ranks), and on the wide GEMM, which takes K unsplit, over token tiles and
weight-tile shapes against the plain wide GEMM at K-split 1; the oracle then
bounds the activation itself."""
import pytest
import torch

import mxfp4_oracle as MO

pytestmark = pytest.mark.gpu


def _case(inter, K, M, seed, lo=118, hi=124):
    g = torch.Generator().manual_seed(seed)
    W = torch.randint(0, 256, (2 * inter, K // 2), dtype=torch.uint8, generator=g)
    St = torch.randint(lo, hi, (2 * inter, K // 32), dtype=torch.uint8, generator=g)
    X = torch.randn(M, K, generator=g).to(torch.bfloat16)
    return W, St, X


def _unfused(W, St, X, inter, dev):
    import h4mv
    from _b200kv import check, lib
    N, K = W.shape[0], W.shape[1] * 2
    packed, _ = h4mv.pack_scales(St.to(dev), N, K)
    gu = h4mv.mxfp4_gemm(X.to(dev), W.to(dev), packed)
    act = torch.empty(X.shape[0], inter, dtype=torch.bfloat16, device=dev)
    check(lib.b200kv_swiglu(gu.data_ptr(), act.data_ptr(), X.shape[0], inter,
                            torch.cuda.current_stream(dev).cuda_stream), "b200kv_swiglu")
    return act


def _fused(W, St, X, inter, dev):
    import h4mv
    order = h4mv.gate_up_row_order(inter)
    Wp, Sp = W.index_select(0, order).contiguous(), St.index_select(0, order).contiguous()
    N, K = W.shape[0], W.shape[1] * 2
    packed, _ = h4mv.pack_scales(Sp.to(dev), N, K)
    return h4mv.mxfp4_gemm_swiglu(X.to(dev), Wp.to(dev), packed)


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("inter,K", [(64, 128), (1792, 4096), (448, 1024)])
def test_skinny_equals_gemm_then_swiglu(cuda, inter, K, M):
    W, St, X = _case(inter, K, M, seed=inter + K + M)
    want = _unfused(W, St, X, inter, cuda)
    got = _fused(W, St, X, inter, cuda)
    assert got.shape == (M, inter)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("ks", [1, 2, 3, 4, 8])
def test_skinny_every_k_split(cuda, monkeypatch, ks):
    inter, K, M = 320, 4096, 4
    W, St, X = _case(inter, K, M, seed=ks)
    want = _unfused(W, St, X, inter, cuda)
    monkeypatch.setenv("B200KV_MMA_KSPLIT", str(ks))
    got = _fused(W, St, X, inter, cuda)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("M", [9, 64, 200])
@pytest.mark.parametrize("mt,nt", [(1, 1), (2, 1), (1, 2)])
def test_wide_equals_gemm_then_swiglu(cuda, monkeypatch, M, mt, nt):
    inter, K = 384, 1024
    W, St, X = _case(inter, K, M, seed=M + 10 * mt + 100 * nt)
    # the wide epilogue takes K unsplit: the plain GEMM at K-split 1 sums in the same order
    monkeypatch.setenv("B200KV_GEMM_KSPLIT", "1")
    want = _unfused(W, St, X, inter, cuda)
    monkeypatch.setenv("B200KV_GEMM_MT", str(mt))
    monkeypatch.setenv("B200KV_GEMM_NT", str(nt))
    got = _fused(W, St, X, inter, cuda)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_7b_gate_up_against_oracle(cuda):
    """The 7B gate_up (28672 x 4096) at M = 1 and 8: the activation against the
    oracle's fp32 product with the same SwiGLU rounding, within one bf16
    rounding of the product feeding it plus 1e-3 of the largest output."""
    inter, K = 14336, 4096
    for M in (1, 8):
        W, St, X = _case(inter, K, M, seed=M)
        got = _fused(W, St, X, inter, cuda).float().cpu()
        ref = MO.mxfp4_linear_reference(W, St.t().contiguous(), X.float())
        g = ref[:, :inter].to(torch.bfloat16).float()
        u = ref[:, inter:].to(torch.bfloat16).float()
        want = ((g / (1 + torch.exp(-g))).to(torch.bfloat16).float() * u).to(torch.bfloat16).float()
        err = (got - want).abs().max() / want.abs().max()
        assert float(err) < 1e-2, (M, float(err))


def test_rejects_bad_arguments(cuda):
    import h4mv
    from _b200kv import lib
    # status codes of include/b200kv.h
    B200KV_ERR_INVALID_ARG, B200KV_ERR_UNSUPPORTED, B200KV_ERR_MISALIGNED = 1, 2, 3
    K = 256
    W = torch.zeros(192, K // 2, dtype=torch.uint8, device=cuda)
    packed, _ = h4mv.pack_scales(torch.full((192, K // 32), 127, dtype=torch.uint8, device=cuda), 192, K)
    x = torch.zeros(2, K, dtype=torch.bfloat16, device=cuda)
    out = torch.empty(2, 96, dtype=torch.bfloat16, device=cuda)
    st = torch.cuda.current_stream(cuda).cuda_stream
    # 2 I = 192 is not a whole number of 128-row tiles
    assert lib.b200kv_mxfp4_gemm_swiglu(W.data_ptr(), packed.data_ptr(), x.data_ptr(), out.data_ptr(),
                                        192, K, 2, st) == B200KV_ERR_UNSUPPORTED
    ws = torch.empty(lib.b200kv_mxfp4_gemm_wide_workspace_bytes(16, K), dtype=torch.uint8, device=cuda)
    xw = torch.zeros(16, K, dtype=torch.bfloat16, device=cuda)
    assert lib.b200kv_mxfp4_gemm_wide_swiglu(W.data_ptr(), packed.data_ptr(), xw.data_ptr(), K, ws.data_ptr(),
                                             ws.numel(), out.data_ptr(), 192, K, 16, st) == B200KV_ERR_UNSUPPORTED
    W2 = torch.zeros(256, K // 2, dtype=torch.uint8, device=cuda)
    p2, _ = h4mv.pack_scales(torch.full((256, K // 32), 127, dtype=torch.uint8, device=cuda), 256, K)
    big = torch.empty(16 * 128 + 8, dtype=torch.bfloat16, device=cuda)
    # act must be 16-byte aligned for the wide epilogue's vector stores
    assert lib.b200kv_mxfp4_gemm_wide_swiglu(W2.data_ptr(), p2.data_ptr(), xw.data_ptr(), K, ws.data_ptr(),
                                             ws.numel(), big[1:].data_ptr(), 256, K, 16,
                                             st) == B200KV_ERR_MISALIGNED
    assert lib.b200kv_mxfp4_gemm_swiglu(None, p2.data_ptr(), x.data_ptr(), out.data_ptr(), 256, K, 2,
                                        st) == B200KV_ERR_INVALID_ARG
    with pytest.raises(ValueError):
        h4mv.mxfp4_gemm_swiglu(x, W, packed)


def test_graph_capturable(cuda):
    inter, K, M = 256, 512, 4
    W, St, X = _case(inter, K, M, seed=3)
    import h4mv
    order = h4mv.gate_up_row_order(inter)
    Wp = W.index_select(0, order).contiguous().to(cuda)
    packed, _ = h4mv.pack_scales(St.index_select(0, order).contiguous().to(cuda), 2 * inter, K)
    x = X.to(cuda)
    out = torch.empty(M, inter, dtype=torch.bfloat16, device=cuda)
    h4mv.mxfp4_gemm_swiglu(x, Wp, packed, out=out)
    want = out.clone()
    out.zero_()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(gr):
        h4mv.mxfp4_gemm_swiglu(x, Wp, packed, out=out)
    torch.cuda.current_stream().wait_stream(s)
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
