"""MXFP4 W4A16 product on block-scaled tcgen05 MMAs (b200kv_mxfp4_gemm) on the
B200 against the CPU oracle.  Tolerance: the reference's own bound,
max|y - ref| / max|ref| < 5e-3 (h4mv/h4mv_test.py:84); the scale packer is
checked byte for byte."""
import pytest
import torch

import mxfp4_oracle as MO

pytestmark = pytest.mark.gpu

TOL = 5e-3
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
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n in range(N):
        W[n, n // 2] = 2 if n % 2 == 0 else (2 << 4)
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


_E2M1 = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6], dtype=torch.float64)


TERMS = 6  # e2m1 terms per activation (the kernel's kTerms)


def _terms_reference(x, terms=TERMS):
    """CPU restatement of the kernel's activation split: per 32-block, `terms`
    greedy e2m1 terms, term scale 2^(E-129) for a residual maximum in
    [2^(E-127), 2^(E-126)), round to nearest (ties to the even code), saturate
    at 6."""
    r = x.double().view(x.shape[0], -1, 32).clone()
    total = torch.zeros_like(r)
    for _ in range(terms):
        mx = r.abs().amax(-1, keepdim=True)
        E = torch.floor(torch.log2(mx.clamp(min=1e-300)))
        s = torch.exp2(E - 2)
        a = (r / s).abs().clamp(max=6.0)
        d = (a[..., None] - _E2M1).abs()
        best = d.min(-1, keepdim=True).values
        idx = torch.where(d == best, torch.arange(8), 99).min(-1).values  # lowest code on ties
        tie = (d == best).sum(-1) > 1
        idx = torch.where(tie & (idx % 2 == 1), idx + 1, idx)             # ties to the even code
        q = torch.where(mx > 0, torch.sign(r) * _E2M1[idx] * s, torch.zeros_like(r))
        total += q
        r = r - q
    return total.view_as(x).float()


def test_activation_terms(cuda):
    """x is written as six block-scaled e2m1 terms: w = one-hot 1.0 picks one x
    element per row, so out = that representation of x, bit for bit; on values
    spanning 11 binades inside each 32-block it stays within 5e-4 of the block
    maximum."""
    K = 1024
    N = K
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n in range(N):
        W[n, n // 2] = 2 if n % 2 == 0 else (2 << 4)
    St = torch.full((N, K // 32), 127, dtype=torch.uint8)
    g = torch.Generator().manual_seed(3)
    mant = 1.0 + torch.randint(0, 128, (4, K), generator=g).float() / 128.0
    sign = torch.where(torch.rand(4, K, generator=g) < 0.5, -1.0, 1.0)
    X = (sign * mant * torch.exp2(torch.randint(-10, 1, (4, K), generator=g).float())).to(torch.bfloat16)
    Y = _run(W, St, X, cuda)
    assert torch.equal(Y, _terms_reference(X.float()).to(torch.bfloat16).float())
    x = X.float()
    blockmax = x.abs().view(4, -1, 32).amax(-1, keepdim=True).expand(-1, -1, 32).reshape(4, K)
    assert bool(((Y - x).abs() <= 5e-4 * blockmax).all())


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("M", [1, 4, 8])
def test_7b_shapes(cuda, name, M):
    N, K = SHAPES[name]
    W, S, St, X = MO.make_case(N, K, M, seed=M * 7 + len(name))
    ref = MO.mxfp4_linear_reference(W, S, X)
    for layout in (0, 1):
        Y = _run(W, St, X, cuda, layout)
        assert MO.rel_to_max_err(Y, ref) < TOL, (name, M, layout)


@pytest.mark.parametrize("N,K,M", [(1, 256, 1), (200, 512, 3), (129, 2048, 8), (1000, 1280, 5)])
def test_ragged(cuda, N, K, M):
    W, S, St, X = MO.make_case(N, K, M, seed=N + K)
    ref = MO.mxfp4_linear_reference(W, S, X)
    Y = _run(W, St, X, cuda)
    assert MO.rel_to_max_err(Y, ref) < TOL


@pytest.mark.parametrize("ks", [1, 2, 3, 5, 8])
def test_k_split_geometries(cuda, monkeypatch, ks):
    monkeypatch.setenv("B200KV_MMA_KSPLIT", str(ks))
    N, K, M = 1024, 4096, 2
    W, S, St, X = MO.make_case(N, K, M, seed=ks)
    ref = MO.mxfp4_linear_reference(W, S, X)
    assert MO.rel_to_max_err(_run(W, St, X, cuda), ref) < TOL


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
    with pytest.raises(B200KVError):  # the skinny kernel needs K % 256 == 0
        h4mv.mxfp4_gemm(torch.zeros(2, 384, dtype=torch.bfloat16, device=cuda),
                        torch.zeros(256, 192, dtype=torch.uint8, device=cuda), packed)
    with pytest.raises(ValueError):  # the wide one K % 128 == 0
        h4mv.mxfp4_gemm(torch.zeros(9, 192, dtype=torch.bfloat16, device=cuda),
                        torch.zeros(256, 96, dtype=torch.uint8, device=cuda), packed)
    with pytest.raises(ValueError):
        h4mv.pack_scales(torch.zeros(256, 3, dtype=torch.uint8, device=cuda), 256, 96)


@pytest.mark.parametrize("N,K,M", [(1024, 512, 1), (512, 1024, 2), (2048, 512, 1), (6144, 4096, 1),
                                   (4096, 14336, 3), (28672, 4096, 8), (512, 512, 5)])
def test_exact_against_term_restatement(cuda, N, K, M):
    """With x replaced by its six-term representation the product is exact up
    to fp32 summation order and the final bf16 rounding: every output within
    one bf16 rounding (plus 1e-6 of the maximum) of the fp32 reference."""
    W, S, St, X = MO.make_case(N, K, M, seed=N + K + M)
    g = torch.Generator().manual_seed(M)
    X = (X.float() * (1 + 3 * torch.rand(X.shape, generator=g))).to(torch.bfloat16)  # wider blocks
    ref = MO.mxfp4_linear_reference(W, S, _terms_reference(X.float()))
    Y = _run(W, St, X, cuda)
    tol = ref.abs() * 2.0 ** -8 + 1e-6 * ref.abs().max()
    assert bool(((Y - ref).abs() <= tol).all()), float(((Y - ref).abs() - tol).max())
