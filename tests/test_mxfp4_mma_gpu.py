"""MXFP4 W4A16 product for M <= 8 on block-scaled tcgen05 MMAs
(b200kv_mxfp4_gemm: kind::mxf8f6f4, e2m1 weights, x as two e4m3 terms) on the
B200 against the CPU oracle (oracle/mxfp4_oracle.py, the reference's dequant +
fp32 matmul, h4mv/h4mv_test.py:19-32).

Every product the kernel forms is the exact dequantised product (x's two
terms are exact for every element within 2^-13 of its block maximum), so the
bound is the fp32 summation order plus the final bf16 rounding: each output
within one bf16 rounding of the fp32 reference plus 1e-6 of the largest
output, far inside the reference's own max|y - ref| / max|ref| < 5e-3
(h4mv_test.py:84).  On integer-valued inputs every partial sum is exact in
fp32 and outputs are compared bit for bit over every K-split, ring shape and
number of issuing warps; the scale packer is checked byte for byte."""
import pytest
import torch

import mxfp4_oracle as MO
from mxfp4_terms import e4m3_terms_reference, integer_case, one_hot_weights, wide_binade_x, within_one_rounding

pytestmark = pytest.mark.gpu

SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}


def _atoms_reference(St, N, K):
    """CPU restatement of the scale-factor atom layout: byte 16*(r%32) + 4*(r/32) + g."""
    ntiles, nsteps = -(-N // 128), K // 128
    out = torch.full((ntiles, nsteps, 512), 127, dtype=torch.uint8)
    b = torch.arange(512)
    dp, jj, kb = b >> 4, (b >> 2) & 3, b & 3
    for t in range(ntiles):
        for s in range(nsteps):
            n = t * 128 + dp + 32 * jj
            g = s * 4 + kb
            ok = n < N
            out[t, s, ok] = St[n[ok], g[ok]]
    return out.flatten()


def _run(W, St, X, dev, layout=0):
    import h4mv
    N, K = W.shape[0], W.shape[1] * 2
    S = St if layout == 0 else St.t().contiguous()
    packed, edge = h4mv.pack_scales(S.to(dev), N, K, layout)
    assert not edge
    return h4mv.mxfp4_gemm(X.to(dev), W.to(dev), packed).float().cpu()


def test_pack_layouts_match_atom_definition(cuda):
    import h4mv
    N, K = 300, 512
    g = torch.Generator().manual_seed(1)
    St = torch.randint(1, 255, (N, K // 32), dtype=torch.uint8, generator=g)
    want = _atoms_reference(St, N, K)
    p0, e0 = h4mv.pack_scales(St.to(cuda), N, K, h4mv.SCALES_TRANSPOSED)
    p1, e1 = h4mv.pack_scales(St.t().contiguous().to(cuda), N, K, h4mv.SCALES_CHECKPOINT)
    assert torch.equal(p0.cpu(), want) and torch.equal(p1.cpu(), want)
    assert not e0 and not e1
    St[7, 3] = 255
    _, e2 = h4mv.pack_scales(St.to(cuda), N, K)
    St[7, 3] = 0
    _, e3 = h4mv.pack_scales(St.to(cuda), N, K)
    assert e2 and e3


def test_one_hot_every_position(cuda):
    """W row n holds code 2 (1.0) at k = n; x = ones: out[n] = 2^(s-127) exactly."""
    N, K = 256, 256
    W = one_hot_weights(N, K)
    St = torch.randint(118, 136, (N, K // 32), dtype=torch.uint8, generator=torch.Generator().manual_seed(2))
    X = torch.ones(1, K, dtype=torch.bfloat16)
    Y = _run(W, St, X, cuda)[0]
    want = torch.tensor([2.0 ** (int(St[n, n // 32]) - 127) for n in range(N)])
    assert torch.equal(Y, want)


def test_every_code_and_scale(cuda):
    K = 256
    rows = [(code, pos) for code in range(16) for pos in range(K)]
    N = len(rows)
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n, (code, pos) in enumerate(rows):
        W[n, pos // 2] = code if pos % 2 == 0 else code << 4
    for s in (100, 119, 125, 127, 128, 129, 200, 240):
        St = torch.full((N, K // 32), s, dtype=torch.uint8)
        Y = _run(W, St, torch.ones(1, K, dtype=torch.bfloat16), cuda)[0]
        want = torch.tensor([MO.E2M1_LUT[c] for c, _ in rows]) * float(MO.e8m0_bits(s))
        assert torch.equal(Y, want.to(torch.bfloat16).float()), s


@pytest.mark.parametrize("M", [1, 3, 8])
def test_one_hot_reproduces_x_exactly(cuda, M):
    """W row n holds 1.0 at k = n: out[m, n] = x[m, n].  Values spanning 13
    binades inside every 32-block come back bit for bit (both terms exact)."""
    K = N = 1024
    X = wide_binade_x(M, K, -12, seed=3 + M)
    Y = _run(one_hot_weights(N, K), torch.full((N, K // 32), 127, dtype=torch.uint8), X, cuda)
    assert torch.equal(Y, X.float())


def test_small_elements_within_bound(cuda):
    """Elements more than 2^-13 below their block maximum may lose low bits:
    the result equals the two-term restatement exactly, and stays within 2^-21
    of the block maximum of x."""
    K = N = 512
    M = 8
    X = wide_binade_x(M, K, -24, seed=4).abs()
    X[:, ::32] = 1.5  # every block maximum at 1.5
    Y = _run(one_hot_weights(N, K), torch.full((N, K // 32), 127, dtype=torch.uint8), X, cuda)
    assert torch.equal(Y, e4m3_terms_reference(X.float()).to(torch.bfloat16).float())
    assert float((Y - X.float()).abs().max()) <= 2.0 ** -21 * 2


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("M", [1, 4, 8])
def test_7b_shapes(cuda, name, M):
    N, K = SHAPES[name]
    W, S, St, X = MO.make_case(N, K, M, seed=M * 7 + len(name))
    ref = MO.mxfp4_linear_reference(W, S, X)
    for layout in (0, 1):
        Y = _run(W, St, X, cuda, layout)
        ok, worst = within_one_rounding(Y, ref)
        assert ok, (name, M, layout, worst)
        assert MO.rel_to_max_err(Y, ref) < 5e-3


@pytest.mark.parametrize("N,K,M", [(1, 128, 1), (200, 512, 3), (129, 2048, 8), (1000, 1280, 5), (300, 384, 2)])
def test_ragged(cuda, N, K, M):
    W, S, St, X = MO.make_case(N, K, M, seed=N + K)
    ref = MO.mxfp4_linear_reference(W, S, X)
    ok, worst = within_one_rounding(_run(W, St, X, cuda), ref)
    assert ok, worst


@pytest.mark.parametrize("issuers", [1, 2, 4])
@pytest.mark.parametrize("ks,bps,stages", [(1, 4, 2), (2, 8, 1), (2, 4, 2), (3, 2, 4), (5, 4, 1), (8, 2, 2), (4, 8, 1)])
def test_plans_bit_exact(cuda, monkeypatch, issuers, ks, bps, stages):
    """Every K-split, boxes per stage, ring depth and issuer count gives the
    exact result on integer inputs (ragged N and a K that leaves partial last
    stages and slices)."""
    monkeypatch.setenv("B200KV_MMA_ISSUERS", str(issuers))
    monkeypatch.setenv("B200KV_MMA_KSPLIT", str(ks))
    monkeypatch.setenv("B200KV_MMA_BPS", str(bps))
    monkeypatch.setenv("B200KV_MMA_STAGES", str(stages))
    W, St, X, ref = integer_case(1000, 3200, 7, seed=issuers * 100 + ks * 10 + bps)
    assert torch.equal(_run(W, St, X, cuda), ref)


def test_matches_cuda_core_kernel(cuda):
    """Both MXFP4 kernels on the same inputs agree to two bf16 roundings of the
    largest output (each rounds its own fp32 sum to bf16)."""
    import h4mv
    N, K, M = 6144, 4096, 4
    W, S, St, X = MO.make_case(N, K, M, seed=11)
    a = h4mv.mxfp4_gemv(X.to(cuda), W.to(cuda), St.to(cuda)).float().cpu()
    b = _run(W, St, X, cuda)
    assert MO.rel_to_max_err(b, a) <= 2 * 2.0 ** -8


def test_rejects_bad_arguments(cuda):
    import h4mv
    from _b200kv import B200KVError
    from _b200kv import lib
    W, S, St, X = MO.make_case(256, 256, 1, seed=0)
    packed, _ = h4mv.pack_scales(St.to(cuda), 256, 256)
    x9 = torch.zeros(9, 256, dtype=torch.bfloat16, device=cuda)
    out = torch.empty(9, 256, dtype=torch.bfloat16, device=cuda)
    Wd = W.to(cuda)
    # the skinny kernel takes M <= 8 (h4mv.mxfp4_gemm sends larger M to the wide one)
    assert lib.b200kv_mxfp4_gemm(Wd.data_ptr(), packed.data_ptr(), x9.data_ptr(), out.data_ptr(), 256, 256, 9,
                                 torch.cuda.current_stream().cuda_stream) == 2
    with pytest.raises(B200KVError):  # K % 128 == 0
        h4mv.mxfp4_gemm(torch.zeros(2, 192, dtype=torch.bfloat16, device=cuda),
                        torch.zeros(256, 96, dtype=torch.uint8, device=cuda), packed)
    with pytest.raises(ValueError):  # the wide one too
        h4mv.mxfp4_gemm(torch.zeros(9, 192, dtype=torch.bfloat16, device=cuda),
                        torch.zeros(256, 96, dtype=torch.uint8, device=cuda), packed)
    with pytest.raises(ValueError):
        h4mv.pack_scales(torch.zeros(256, 3, dtype=torch.uint8, device=cuda), 256, 96)


@pytest.mark.parametrize("N,K,M", [(1024, 512, 1), (512, 1024, 2), (6144, 4096, 1), (4096, 14336, 3),
                                   (28672, 4096, 8), (512, 512, 5)])
def test_exact_against_term_restatement(cuda, N, K, M):
    """With x replaced by its two-term representation the product is exact up
    to fp32 summation order and the final bf16 rounding, also on activations
    spanning many binades within a block."""
    W, S, St, X = MO.make_case(N, K, M, seed=N + K + M)
    X = (X.float() * wide_binade_x(M, K, -16, seed=M).float().abs()).to(torch.bfloat16)
    ref = MO.mxfp4_linear_reference(W, S, e4m3_terms_reference(X.float()))
    ok, worst = within_one_rounding(_run(W, St, X, cuda), ref)
    assert ok, worst
