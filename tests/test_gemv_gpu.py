"""MXFP4 W4A16 matvec on the B200 against the CPU oracle (GPU tests).

Known-answer tests restate the reference's probes (h4mv/h4mv_test.py:38-52,
w4-hip-demo/probe_w4hip.py:13-47); full-shape parity uses the reference's
tolerance, max|y - ref| / max|ref| < 5e-3 (h4mv/h4mv_test.py:84), at the 7B
shapes of config 2.
"""
import pytest
import torch

import mxfp4_oracle as MO

pytestmark = pytest.mark.gpu

TOL = 5e-3
SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}


def _run(W, St, X, dev):
    import h4mv
    return h4mv.mxfp4_gemv(X.to(dev), W.to(dev), St.to(dev))


def test_one_hot_probe_all_positions(cuda):
    # h4mv/h4mv_test.py:38-52 through the reference-style raw launch
    import h4mv
    N, K, M = 4, 32, 8
    St = torch.full((N, 1), 127, dtype=torch.uint8, device=cuda)
    for k in range(32):
        W = torch.zeros(N, K // 2, dtype=torch.uint8, device=cuda)
        W[:, k // 2] = 2 if k % 2 == 0 else (2 << 4)
        X = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
        X[:, k] = 1.0
        Y = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
        h4mv.launch(W, St, X, Y, N, K, M)
        torch.cuda.synchronize()
        assert torch.equal(Y.float().cpu(), torch.ones(M, N)), k


def test_every_code_every_position_every_scale(cuda):
    """Row n holds one e2m1 code at one k position; x is all ones, so the output
    is exactly e2m1(code) * scale(s) (kernel scale semantics, h4mv.cu:72)."""
    K = 64
    rows = []
    for code in range(16):
        for pos in range(K):
            rows.append((code, pos))
    N = len(rows)
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n, (code, pos) in enumerate(rows):
        W[n, pos // 2] = code if pos % 2 == 0 else code << 4
    for s in (100, 119, 125, 127, 128, 129, 200, 240):
        St = torch.full((N, K // 32), s, dtype=torch.uint8)
        X = torch.ones(1, K, dtype=torch.bfloat16)
        Y = _run(W, St, X, cuda).float().cpu()[0]
        want = torch.tensor([MO.E2M1_LUT[c] for c, _ in rows]) * float(MO.e8m0_bits(s))
        want = want.to(torch.bfloat16).float()
        assert torch.equal(Y, want), s


def test_edge_scale_codes(cuda):
    """scale byte 0 -> 0 and 255 -> inf, as in the reference kernel."""
    N, K = 8, 64
    W = torch.full((N, K // 2), 0x22, dtype=torch.uint8)   # every weight = 1.0
    X = torch.ones(1, K, dtype=torch.bfloat16)
    St = torch.zeros(N, K // 32, dtype=torch.uint8)
    assert torch.all(_run(W, St, X, cuda).float() == 0)
    St[:, 0] = 255
    St[:, 1] = 127
    Y = _run(W, St, X, cuda).float().cpu()
    assert torch.all(torch.isinf(Y) & (Y > 0))


def test_structured_full_row(cuda):
    # w4-hip-demo/probe_w4hip.py:33-47
    g = torch.Generator().manual_seed(0)
    N, K = 8, 4096
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    S = torch.full((K // 32, N), 127, dtype=torch.uint8)
    X = (torch.arange(K, dtype=torch.float32) % 7 - 3).to(torch.bfloat16).view(1, K)
    ref = MO.mxfp4_linear_reference(W, S, X)
    Y = _run(W, S.t().contiguous(), X, cuda).float().cpu()
    assert torch.equal(Y, ref.to(torch.bfloat16).float())


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("M", [1, 4, 8])
def test_7b_shapes(cuda, name, M):
    N, K = SHAPES[name]
    W, S, St, X = MO.make_case(N, K, M, seed=N + K + M)
    ref = MO.mxfp4_linear_reference(W, S, X)
    Y = _run(W, St, X, cuda).float().cpu()
    err = MO.rel_to_max_err(Y, ref)
    assert err < TOL, err


@pytest.mark.parametrize("M", [1, 2, 3, 5, 6, 7, 8])
@pytest.mark.parametrize("N,K", [(1, 32), (7, 96), (17, 160), (33, 4128), (300, 1056), (1000, 512)])
def test_ragged_shapes(cuda, N, K, M):
    W, S, St, X = MO.make_case(N, K, M, seed=7 * N + K + M)
    ref = MO.mxfp4_linear_reference(W, S, X)
    Y = _run(W, St, X, cuda).float().cpu()
    assert MO.rel_to_max_err(Y, ref) < TOL


@pytest.mark.parametrize("ksplit", ["1", "2", "4"])
@pytest.mark.parametrize("nw,kc,stages", [("4", "16", "2"), ("4", "32", "4"), ("8", "64", "3"),
                                          ("8", "16", "8")])
def test_launch_geometries(cuda, monkeypatch, ksplit, nw, kc, stages):
    monkeypatch.setenv("B200KV_GEMV_KSPLIT", ksplit)
    monkeypatch.setenv("B200KV_GEMV_NW", nw)
    monkeypatch.setenv("B200KV_GEMV_KC", kc)
    monkeypatch.setenv("B200KV_GEMV_STAGES", stages)
    W, S, St, X = MO.make_case(200, 2048, 5, seed=11)
    ref = MO.mxfp4_linear_reference(W, S, X)
    Y = _run(W, St, X, cuda).float().cpu()
    assert MO.rel_to_max_err(Y, ref) < TOL


def test_wide_dynamic_range_activations(cuda):
    """x spanning bf16's range (2^-100 .. 2^100): the dequantised weights are exact
    and products accumulate in fp32, so the error stays at fp32 rounding."""
    g = torch.Generator().manual_seed(3)
    N, K, M = 64, 1024, 3
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    S = torch.randint(119, 126, (K // 32, N), dtype=torch.uint8, generator=g)
    e = torch.randint(-100, 100, (M, K), generator=g).float()
    X = (torch.randn(M, K, generator=g) * torch.exp2(e)).to(torch.bfloat16)
    ref = MO.mxfp4_linear_reference(W, S, X).double()
    Y = _run(W, S.t().contiguous(), X, cuda).double().cpu()
    for m in range(M):  # per activation row: its own magnitude sets the scale
        assert MO.rel_to_max_err(Y[m], ref[m]) < TOL, m


def test_deterministic(cuda):
    W, S, St, X = MO.make_case(4096, 4096, 4, seed=2)
    a = _run(W, St, X, cuda)
    b = _run(W, St, X, cuda)
    assert torch.equal(a, b)


def test_rejects_bad_arguments(cuda):
    import h4mv
    from _b200kv import B200KVError
    W, S, St, X = MO.make_case(16, 64, 9, seed=1)
    with pytest.raises(B200KVError):
        h4mv.mxfp4_gemv(X.to(cuda), W.to(cuda), St.to(cuda))
    Y = torch.empty(9, 16, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(B200KVError):
        h4mv.launch(W.to(cuda), St.to(cuda), X.to(cuda), Y, 16, 64, 9)
