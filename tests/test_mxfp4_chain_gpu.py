"""Chains of dependent MXFP4 matvecs in one persistent launch
(b200kv_mxfp4_chain) on the B200.

Each op is the product of b200kv_mxfp4_gemm (the reference kernel h4mv_t,
h4mv/h4mv.cu:43-104, restated by oracle/mxfp4_oracle.py), so each op's output
is checked against the fp32 oracle applied to the chain's own input of that
op, within one bf16 rounding (the bound of the single-op tests).  Exactness
through the dependency machinery is checked bit for bit: permutation weights
(each output row copies one input element) carry x through a chain unchanged,
and integer inputs make every partial sum exact, so a stale or early read of
a tile shows up as a wrong value.  Outputs are poisoned with NaN before each
run.  Grid sizes from 2 CTAs upward exercise many-segment reductions."""
import pytest
import torch

import mxfp4_oracle as MO
from mxfp4_terms import integer_case, within_one_rounding

pytestmark = pytest.mark.gpu


def _packed(St, N, K, dev):
    import h4mv
    p, edge = h4mv.pack_scales(St.to(dev), N, K, h4mv.SCALES_TRANSPOSED)
    assert not edge
    return p


def _perm_weights(N, K, seed):
    """Row n holds 1.0 at k = perm[n] (K >= N): out[m, n] = x[m, perm[n]]."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(K, generator=g)[:N]
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n in range(N):
        k = int(perm[n])
        W[n, k // 2] = 2 if k % 2 == 0 else (2 << 4)
    return W, torch.full((N, K // 32), 127, dtype=torch.uint8), perm


@pytest.fixture(params=[0, 2, 5])
def ctas(request, monkeypatch):
    """0 = one CTA per SM; 2 and 5 put several segments on every tile."""
    if request.param:
        monkeypatch.setenv("B200KV_CHAIN_CTAS", str(request.param))
    return request.param


@pytest.mark.parametrize("M", [1, 3, 8])
def test_permutation_chain_exact(cuda, ctas, M):
    """x through four dependent permutation ops comes out bit for bit, every
    intermediate too (each op reads tiles of the previous op's output that
    other CTAs finish)."""
    import h4mv
    dims = [2048, 1536, 1280, 1024, 768]
    x = (torch.randn(M, dims[0], generator=torch.Generator().manual_seed(M)) * 4).to(torch.bfloat16)
    ops, wants, cur = [], [], x.float()
    for j in range(len(dims) - 1):
        K, N = dims[j], dims[j + 1]
        W, St, perm = _perm_weights(N, K, seed=j + 10 * M)
        cur = cur[:, perm]
        wants.append(cur)
        op = {"weight": W.to(cuda), "scales": _packed(St, N, K, cuda),
              "out": torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)}
        if j == 0:
            op["x"] = x.to(cuda)
        else:
            op["x_from"] = j - 1
        ops.append(op)
    chain = h4mv.MXFP4Chain(ops, M, cuda)
    chain.run()
    torch.cuda.synchronize()
    for j, op in enumerate(ops):
        assert torch.equal(op["out"].float().cpu(), wants[j]), j


@pytest.mark.parametrize("N,K,M", [(1, 128, 1), (300, 384, 2), (1000, 3200, 7), (4096, 4096, 8), (129, 14336, 1)])
def test_single_op_integer_exact(cuda, ctas, N, K, M):
    import h4mv
    W, St, X, ref = integer_case(N, K, M, seed=N + K + M)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)
    chain = h4mv.MXFP4Chain([{"weight": W.to(cuda), "scales": _packed(St, N, K, cuda), "x": X.to(cuda),
                              "out": out}], M, cuda)
    chain.run()
    torch.cuda.synchronize()
    assert torch.equal(out.float().cpu(), ref)


@pytest.mark.parametrize("M", [1, 4, 8])
def test_7b_layer_chain_each_op_within_one_rounding(cuda, M):
    """o -> gate_up (SwiGLU) -> down -> qkv at 7B shapes on config-2 data: each
    op against the oracle on the chain's own input of that op."""
    import h4mv
    inter = 14336
    shapes = [(4096, 4096), (2 * inter, 4096), (4096, inter), (6144, 4096)]
    order = h4mv.gate_up_row_order(inter)
    xs = torch.randn(M, 4096, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
    host, ops = [], []
    for j, (N, K) in enumerate(shapes):
        W, S, St, _ = MO.make_case(N, K, M, seed=100 * M + j)
        if j == 1:
            W, St = W[order].contiguous(), St[order].contiguous()
        host.append((W, St))
        width = N // 2 if j == 1 else N
        op = {"weight": W.to(cuda), "scales": _packed(St, N, K, cuda),
              "out": torch.full((M, width), float("nan"), dtype=torch.bfloat16, device=cuda)}
        if j == 0:
            op["x"] = xs.to(cuda)
        else:
            op["x_from"] = j - 1
        if j == 1:
            op["epilogue"] = h4mv.CHAIN_SWIGLU
        ops.append(op)
    h4mv.MXFP4Chain(ops, M, cuda).run()
    torch.cuda.synchronize()
    inp = xs
    for j, (W, St) in enumerate(host):
        got = ops[j]["out"].float().cpu()
        ref = MO.mxfp4_linear_reference(W, St.t().contiguous(), inp)
        if j == 1:  # SwiGLU of the interleaved rows: gate rows then up rows per 128-row tile
            r = ref.view(M, -1, 2, 64)
            g, u = r[:, :, 0].reshape(M, -1), r[:, :, 1].reshape(M, -1)
            g, u = g.to(torch.bfloat16).float(), u.to(torch.bfloat16).float()
            act = (g * torch.sigmoid(g)).to(torch.bfloat16).float() * u
            assert float((got - act).abs().max()) <= 4 * 2.0 ** -8 * float(act.abs().max()), j
        else:
            ok, worst = within_one_rounding(got, ref)
            assert ok, (j, worst)
        inp = ops[j]["out"].cpu()


def test_swiglu_matches_glue_kernel_on_exact_gate_up(cuda, ctas):
    """Integer inputs make gate/up exact, so the fused epilogue equals
    b200kv_swiglu applied to the per-op kernel's gate_up output bit for bit."""
    import h4mv
    from _b200kv import lib
    inter, K, M = 512, 256, 4
    W, St, X, _ = integer_case(2 * inter, K, M, seed=3)
    order = h4mv.gate_up_row_order(inter)
    plain = h4mv.mxfp4_gemm(X.to(cuda), W.to(cuda), _packed(St, 2 * inter, K, cuda))
    act_ref = torch.empty(M, inter, dtype=torch.bfloat16, device=cuda)
    assert lib.b200kv_swiglu(plain.data_ptr(), act_ref.data_ptr(), M, inter,
                             torch.cuda.current_stream().cuda_stream) == 0
    Wi, Sti = W[order].contiguous(), St[order].contiguous()
    out = torch.full((M, inter), float("nan"), dtype=torch.bfloat16, device=cuda)
    h4mv.MXFP4Chain([{"weight": Wi.to(cuda), "scales": _packed(Sti, 2 * inter, K, cuda), "x": X.to(cuda),
                      "out": out, "epilogue": h4mv.CHAIN_SWIGLU}], M, cuda).run()
    torch.cuda.synchronize()
    assert torch.equal(out, act_ref)


def test_repeated_runs_and_graph_replay(cuda):
    """The counters and ready flags persist across launches: new inputs every
    run, eagerly and through CUDA-graph replays, give new exact results."""
    import h4mv
    M, dims = 2, [1024, 768, 512]
    ops, perms = [], []
    x = torch.zeros(M, dims[0], dtype=torch.bfloat16, device=cuda)
    for j in range(2):
        W, St, perm = _perm_weights(dims[j + 1], dims[j], seed=40 + j)
        perms.append(perm)
        op = {"weight": W.to(cuda), "scales": _packed(St, dims[j + 1], dims[j], cuda),
              "out": torch.zeros(M, dims[j + 1], dtype=torch.bfloat16, device=cuda)}
        op.update({"x": x} if j == 0 else {"x_from": 0})
        ops.append(op)
    chain = h4mv.MXFP4Chain(ops, M, cuda)

    def expect(xv):
        return xv.float().cpu()[:, perms[0]][:, perms[1]]
    g = torch.Generator().manual_seed(9)
    for _ in range(3):
        xv = torch.randn(M, dims[0], generator=g).to(torch.bfloat16)
        x.copy_(xv)
        ops[1]["out"].fill_(float("nan"))
        chain.run()
        torch.cuda.synchronize()
        assert torch.equal(ops[1]["out"].float().cpu(), expect(xv))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain.run()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain.run()
    for _ in range(3):
        xv = torch.randn(M, dims[0], generator=g).to(torch.bfloat16)
        x.copy_(xv)
        ops[1]["out"].fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(ops[1]["out"].float().cpu(), expect(xv))


def test_rejects_bad_chains(cuda):
    import ctypes

    import h4mv
    from _b200kv import ChainOp, lib
    W = torch.zeros(256, 128, dtype=torch.uint8, device=cuda)
    P = _packed(torch.full((256, 8), 127, dtype=torch.uint8), 256, 256, cuda)
    x = torch.zeros(1, 256, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(1, 256, dtype=torch.bfloat16, device=cuda)
    base = {"weight": W, "scales": P, "out": out}
    with pytest.raises(ValueError):
        h4mv.MXFP4Chain([dict(base, x_from=0)], 1, cuda)           # x from itself
    with pytest.raises(ValueError):
        h4mv.MXFP4Chain([dict(base, x=x)], 9, cuda)                # M > 8
    with pytest.raises(ValueError):                                  # K of op 1 != N of op 0
        h4mv.MXFP4Chain([dict(base, x=x), {"weight": torch.zeros(256, 64, dtype=torch.uint8, device=cuda),
                                           "scales": P, "out": out, "x_from": 0}], 1, cuda)
    arr = (ChainOp * 1)()
    arr[0].weight, arr[0].packed_scales, arr[0].x, arr[0].x_stride = W.data_ptr(), P.data_ptr(), x.data_ptr(), 256
    arr[0].out, arr[0].out_stride, arr[0].N, arr[0].K, arr[0].x_from, arr[0].epilogue = out.data_ptr(), 256, 256, 256, -1, 0
    need = lib.b200kv_mxfp4_chain_workspace_bytes(arr, 1, 1)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.b200kv_mxfp4_chain(arr, 1, 1, ws.data_ptr(), need - 256, stream) == 4   # workspace too small
    assert lib.b200kv_mxfp4_chain(arr, 1, 1, ws.data_ptr() + 16, need, stream) == 4    # misaligned workspace
    arr[0].K = 200
    assert lib.b200kv_mxfp4_chain(arr, 1, 1, ws.data_ptr(), need, stream) == 2          # K % 128
    assert lib.b200kv_mxfp4_chain(ctypes.cast(None, ctypes.POINTER(ChainOp)), 1, 1, ws.data_ptr(), need,
                                  stream) == 1
