"""MXFP4 W4A16 GEMM for wide batches (b200kv_mxfp4_gemm_wide: block-scaled
tcgen05 kind::mxf8f6f4, e2m1 weights, x as two e4m3 terms) on the B200 against
the CPU oracle (oracle/mxfp4_oracle.py, the reference's dequant + fp32 matmul,
h4mv/h4mv_test.py:19-32).

Every product the kernel forms is the exact dequantised product, so the bound
is the fp32 summation order plus the final bf16 rounding: each output within
one bf16 rounding of the fp32 reference plus 1e-6 of the largest output (far
inside the reference's own max|y - ref| / max|ref| < 5e-3, h4mv_test.py:84).
On integer-valued inputs every partial sum is exact in fp32 and the outputs
are compared bit for bit, for every tile shape and K-split of the kernel."""
import pytest
import torch

import mxfp4_oracle as MO
from mxfp4_terms import e4m3_terms_reference as _e4m3_terms_reference
from mxfp4_terms import integer_case as _integer_case
from mxfp4_terms import within_one_rounding as _within_one_rounding

pytestmark = pytest.mark.gpu

SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}


def _packed(St, N, K, dev):
    import h4mv
    packed, edge = h4mv.pack_scales(St.to(dev), N, K, h4mv.SCALES_TRANSPOSED)
    assert not edge
    return packed


def _run(W, St, X, dev, **kw):
    import h4mv
    N, K = W.shape[0], W.shape[1] * 2
    return h4mv.mxfp4_gemm_wide(X.to(dev), W.to(dev), _packed(St, N, K, dev), **kw).float().cpu()


def test_one_hot_reproduces_x_exactly(cuda):
    """W row n holds 1.0 at k = n: out[m, n] = x[m, n].  Values spanning 13
    binades inside every 32-block come back bit for bit (both terms exact)."""
    K = N = 1024
    M = 70
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n in range(N):
        W[n, n // 2] = 2 if n % 2 == 0 else (2 << 4)
    St = torch.full((N, K // 32), 127, dtype=torch.uint8)
    g = torch.Generator().manual_seed(3)
    mant = 1.0 + torch.randint(0, 128, (M, K), generator=g).float() / 128.0
    sign = torch.where(torch.rand(M, K, generator=g) < 0.5, -1.0, 1.0)
    X = (sign * mant * torch.exp2(torch.randint(-12, 1, (M, K), generator=g).float())).to(torch.bfloat16)
    Y = _run(W, St, X, cuda)
    assert torch.equal(Y, X.float())


def test_small_elements_within_bound(cuda):
    """Elements more than 2^-13 below their block maximum may lose low bits:
    the result equals the two-term restatement exactly, and stays within
    2^-21 of the block maximum of x."""
    K = N = 512
    M = 64
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n in range(N):
        W[n, n // 2] = 2 if n % 2 == 0 else (2 << 4)
    St = torch.full((N, K // 32), 127, dtype=torch.uint8)
    g = torch.Generator().manual_seed(4)
    mant = 1.0 + torch.randint(0, 128, (M, K), generator=g).float() / 128.0
    X = (mant * torch.exp2(torch.randint(-24, 1, (M, K), generator=g).float())).to(torch.bfloat16)
    X[:, ::32] = 1.5  # every block maximum at 1.5
    Y = _run(W, St, X, cuda)
    assert torch.equal(Y, _e4m3_terms_reference(X.float()).to(torch.bfloat16).float())
    assert float((Y - X.float()).abs().max()) <= 2.0 ** -21 * 2


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("M", [16, 64])
def test_7b_shapes(cuda, name, M):
    N, K = SHAPES[name]
    W, S, St, X = MO.make_case(N, K, M, seed=M * 13 + len(name))
    ref = MO.mxfp4_linear_reference(W, S, X)
    Y = _run(W, St, X, cuda)
    ok, worst = _within_one_rounding(Y, ref)
    assert ok, (name, M, worst)
    assert MO.rel_to_max_err(Y, ref) < 5e-3


@pytest.mark.parametrize("N,K,M", [(1, 128, 1), (200, 384, 9), (129, 2048, 65), (1000, 1280, 130),
                                   (4096, 4096, 256)])
def test_ragged(cuda, N, K, M):
    W, S, St, X = MO.make_case(N, K, M, seed=N + K + M)
    ref = MO.mxfp4_linear_reference(W, S, X)
    ok, worst = _within_one_rounding(_run(W, St, X, cuda), ref)
    assert ok, worst


@pytest.mark.parametrize("kb", [1, 2])
@pytest.mark.parametrize("M", [130, 100, 40])
@pytest.mark.parametrize("mt,nt,ks", [(1, 1, 1), (1, 1, 3), (2, 1, 5), (1, 2, 2), (2, 1, 8), (1, 1, 7),
                                      (1, 2, 1)])
def test_tile_shapes_and_k_splits_bit_exact(cuda, monkeypatch, mt, nt, ks, M, kb):
    """Three token-tile counts (3, 2, 1) with ragged last tiles; one or two
    128-k steps per ring stage (16 steps over ks slices leave partial last
    stages)."""
    monkeypatch.setenv("B200KV_GEMM_MT", str(mt))
    monkeypatch.setenv("B200KV_GEMM_NT", str(nt))
    monkeypatch.setenv("B200KV_GEMM_KSPLIT", str(ks))
    monkeypatch.setenv("B200KV_GEMM_KB", str(kb))
    W, St, X, ref = _integer_case(1000, 2048, M, seed=mt * 100 + nt * 10 + ks + M)
    Y = _run(W, St, X, cuda)
    assert torch.equal(Y, ref)


def test_strided_x_and_explicit_workspace(cuda):
    """x as a column slice of a wider buffer (row stride > K), workspace passed in."""
    from _b200kv import lib
    W, St, X, ref = _integer_case(384, 1024, 100, seed=7)
    wide = torch.zeros(100, 1024 + 256, dtype=torch.bfloat16)
    wide[:, 128:128 + 1024] = X
    xd = wide.to(cuda)[:, 128:128 + 1024]
    ws = torch.empty(lib.b200kv_mxfp4_gemm_wide_workspace_bytes(100, 1024), dtype=torch.uint8, device=cuda)
    import h4mv
    Y = h4mv.mxfp4_gemm_wide(xd, W.to(cuda), _packed(St, 384, 1024, cuda), workspace=ws).float().cpu()
    assert torch.equal(Y, ref)


def test_dispatch_from_mxfp4_gemm(cuda):
    """h4mv.mxfp4_gemm takes M > 8 to the wide kernel."""
    import h4mv
    W, St, X, ref = _integer_case(256, 512, 40, seed=8)
    Y = h4mv.mxfp4_gemm(X.to(cuda), W.to(cuda), _packed(St, 256, 512, cuda)).float().cpu()
    assert torch.equal(Y, ref)


def test_matches_skinny_kernel_where_both_apply(cuda):
    """At M = 8 both tensor-core kernels (the same two-term activation split,
    different summation orders) agree to two bf16 roundings of the largest
    output."""
    import h4mv
    N, K, M = 4096, 4096, 8
    W, S, St, X = MO.make_case(N, K, M, seed=12)
    p = _packed(St, N, K, cuda)
    a = h4mv.mxfp4_gemm(X.to(cuda), W.to(cuda), p).float().cpu()
    b = h4mv.mxfp4_gemm_wide(X.to(cuda), W.to(cuda), p).float().cpu()
    assert MO.rel_to_max_err(b, a) <= 2 * 2.0 ** -8


def test_rejects_bad_arguments(cuda):
    import h4mv
    from _b200kv import B200KVError
    W, S, St, X = MO.make_case(256, 256, 16, seed=0)
    p = _packed(St, 256, 256, cuda)
    small = torch.empty(16, dtype=torch.uint8, device=cuda)
    with pytest.raises(B200KVError):
        h4mv.mxfp4_gemm_wide(X.to(cuda), W.to(cuda), p, workspace=small)
    with pytest.raises(ValueError):
        h4mv.wide_workspace(16, 96, cuda, torch.cuda.current_stream())


@pytest.mark.parametrize("N,offset", [(1000, 0), (1001, 0), (1000, 3)])
def test_unsplit_output_stores(cuda, monkeypatch, N, offset):
    """Without a K-split the tile leaves through 16-byte stores when N % 8 == 0
    and the output is 16-byte aligned, else element by element; an output
    view at an odd element offset takes the second path."""
    import h4mv
    monkeypatch.setenv("B200KV_GEMM_KSPLIT", "1")
    W, St, X, ref = _integer_case(N, 1024, 70, seed=N + offset)
    buf = torch.full((70 * N + offset,), float("nan"), dtype=torch.bfloat16, device=cuda)
    out = buf[offset:].view(70, N)
    h4mv.mxfp4_gemm_wide(X.to(cuda), W.to(cuda), _packed(St, N, 1024, cuda), out=out)
    assert torch.equal(out.float().cpu(), ref)
    assert bool(buf[:offset].isnan().all())


@pytest.mark.parametrize("n256", ["0", "1"])
@pytest.mark.parametrize("M", [100, 128, 300])
def test_two_token_tiles_one_or_two_mmas(cuda, monkeypatch, n256, M):
    """With two token tiles per CTA the kernel issues one N = 256 MMA (scale
    atoms of the two tiles side by side in tensor memory) or two of N = 128;
    both bit-exact on integer inputs, ragged last token tile included."""
    monkeypatch.setenv("B200KV_GEMM_NT", "2")
    monkeypatch.setenv("B200KV_GEMM_N256", n256)
    W, St, X, ref = _integer_case(640, 2048, M, seed=M + int(n256))
    assert torch.equal(_run(W, St, X, cuda), ref)
