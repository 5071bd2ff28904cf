"""The qkv projection with the rotary embedding and the fp8 KV-cache write as
its epilogue (b200kv_mxfp4_gemm_rope_kv) on the B200.

Its contract is bit equality with the unfused path: b200kv_mxfp4_gemm into the
qkv buffer, then b200kv_rope_kv_write (HF Llama neox rotary in fp32 from the
bf16 products, q written back in place, k rotated and v quantised into the
paged cache).  Checked over M, over head counts of one GPU and of
tensor-parallel shards, over every K-split the skinny kernel can be forced to
(the finishing rank pairs dims r and r + 64 from the partials of every rank),
with a skipped slot (-1) and positions past the table clamped."""
import pytest
import torch

pytestmark = pytest.mark.gpu

D, BS = 128, 16


def _case(hq, hkv, K, M, seed):
    g = torch.Generator().manual_seed(seed)
    N = (hq + 2 * hkv) * D
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    St = torch.randint(118, 124, (N, K // 32), dtype=torch.uint8, generator=g)
    X = torch.randn(M, K, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 5000, (M,), generator=g).to(torch.int32)
    pos[0] = 4095
    slots = torch.randperm(8 * BS, generator=g)[:M].to(torch.int64)
    if M > 1:
        slots[1] = -1
    return W, St, X, pos, slots


def _run(W, St, X, pos, slots, hq, hkv, dev, fused):
    import decoder
    import h4mv
    from _b200kv import KV_FP8_E4M3, check, lib
    N, K, M = W.shape[0], W.shape[1] * 2, X.shape[0]
    packed, _ = h4mv.pack_scales(St.to(dev), N, K)
    Wd, Xd = W.to(dev), X.to(dev)
    table = decoder.rope_table(4096, D, 1e6).to(dev)
    pos_d, slots_d = pos.to(dev), slots.to(dev)
    kc = torch.zeros(8, BS, hkv, D, dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    ks = torch.full((1,), 1 / 24, device=dev)
    vs = torch.full((1,), 1 / 40, device=dev)
    qkv = torch.zeros(M, N, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    if fused:
        check(lib.b200kv_mxfp4_gemm_rope_kv(Wd.data_ptr(), packed.data_ptr(), Xd.data_ptr(), qkv.data_ptr(),
                                            N, K, M, pos_d.data_ptr(), table.data_ptr(), 4096,
                                            slots_d.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                            *kc.stride()[:3], *vc.stride()[:3], ks.data_ptr(), vs.data_ptr(),
                                            hq, hkv, BS, KV_FP8_E4M3, st), "b200kv_mxfp4_gemm_rope_kv")
    else:
        h4mv.mxfp4_gemm(Xd, Wd, packed, out=qkv)
        check(lib.b200kv_rope_kv_write(qkv.data_ptr(), qkv.stride(0), pos_d.data_ptr(), table.data_ptr(), 4096,
                                       slots_d.data_ptr(), kc.data_ptr(), vc.data_ptr(), *kc.stride()[:3],
                                       *vc.stride()[:3], ks.data_ptr(), vs.data_ptr(), M, hq, hkv, D, BS,
                                       KV_FP8_E4M3, st), "b200kv_rope_kv_write")
    torch.cuda.synchronize()
    return qkv[:, :hq * D].cpu(), kc.cpu(), vc.cpu()


def _check(hq, hkv, K, M, seed, dev):
    case = _case(hq, hkv, K, M, seed)
    qa, ka, va = _run(*case, hq, hkv, dev, fused=False)
    qb, kb, vb = _run(*case, hq, hkv, dev, fused=True)
    assert torch.equal(qa.view(torch.int16), qb.view(torch.int16))
    assert torch.equal(ka, kb) and torch.equal(va, vb)
    assert int(kb.count_nonzero()) > 0 and int(vb.count_nonzero()) > 0


@pytest.mark.parametrize("M", [1, 2, 5, 8])
@pytest.mark.parametrize("hq,hkv,K", [(32, 8, 4096), (4, 1, 4096), (8, 2, 1024)])
def test_equals_gemm_then_rope_kv_write(cuda, hq, hkv, K, M):
    _check(hq, hkv, K, M, seed=hq + K + M, dev=cuda)


@pytest.mark.parametrize("ks", ["1", "2", "4"])
def test_every_k_split(cuda, monkeypatch, ks):
    monkeypatch.setenv("B200KV_MMA_KSPLIT", ks)
    _check(8, 2, 4096, 3, seed=7, dev=cuda)


def test_argument_errors(cuda):
    """N must be (hq + 2 hkv) * 128; fp8 caches only; M <= 8."""
    from _b200kv import KV_BF16, KV_FP8_E4M3, lib
    A = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda).data_ptr()
    st = torch.cuda.current_stream(cuda).cuda_stream
    base = dict(N=6 * D, K=256, M=1, hq=4, hkv=1, kv=KV_FP8_E4M3)

    def call(**kw):
        a = {**base, **kw}
        return lib.b200kv_mxfp4_gemm_rope_kv(A, A, A, A, a["N"], a["K"], a["M"], A, A, 4096, A, A, A,
                                             4096, 256, 128, 4096, 256, 128, A, A, a["hq"], a["hkv"], BS,
                                             a["kv"], st)
    assert call(N=5 * D) == 2            # not (hq + 2 hkv) heads of 128
    assert call(kv=KV_BF16) == 2         # bf16 cache: the unfused path
    assert call(M=9) == 2                # M <= 8
    assert call(hq=0) == 1
