"""fp8-KV causal prefill attention (tcgen05) on the B200 against the CPU
oracle and against the REFERENCE's own Triton kernel outputs (fixtures run on
CPU by the Triton interpreter).  Tolerance: the reference's own bound, max abs
< 0.05 (vllm-fp8kv/prefill_test.py:49), and rel-to-max < 2e-2."""
import math

import pytest
import torch

import fp8kv_oracle as FO
from test_oracle_pins import CASES, PRE, _bf16, golden_prefill_inputs

pytestmark = pytest.mark.gpu

ATOL = 0.05
RTOL = 2e-2
HQ, HKV, D, PBLK = 32, 8, 128, 16


def _check(got, ref):
    got = got.float().cpu()
    err = (got - ref).abs().max().item()
    rel = err / max(ref.abs().max().item(), 1e-30)
    assert err < ATOL and rel < RTOL, (err, rel)


@pytest.mark.parametrize("name", PRE)
def test_golden_reference_kernel_cases(cuda, name):
    import fp8kv_prefill
    a = golden_prefill_inputs(CASES[name])
    q = a["q"].to(cuda)
    out = torch.zeros_like(q)
    fp8kv_prefill.run(q, a["k_cache"].to(cuda), a["v_cache"].to(cuda), out,
                      a["block_table"].to(cuda), a["k_scale"], a["v_scale"], a["sm_scale"],
                      a["q0"], a["qlen"])
    _check(out, _bf16(CASES[name]["out"]).float())
    cu = torch.tensor([0, a["qlen"]], dtype=torch.int32)
    lens = torch.tensor([a["q0"] + a["qlen"]], dtype=torch.int32)
    ref = FO.prefill_reference(a["q"], a["k_cache"], a["v_cache"], cu, lens, a["block_table"],
                               a["k_scale"], a["v_scale"], a["sm_scale"])
    _check(out, ref)


def _ref_cache(ctx, seed, hkv=HKV, pblk=PBLK, permute=True):
    """Reference test data (prefill_test.py:13-21): (randn * 2) cast to fp8."""
    g = torch.Generator().manual_seed(seed)
    nb = math.ceil(ctx / pblk) + 3
    k = (torch.randn(nb, pblk, hkv, D, generator=g) * 2).to(torch.float8_e4m3fn)
    v = (torch.randn(nb, pblk, hkv, D, generator=g) * 2).to(torch.float8_e4m3fn)
    bt = (torch.randperm(nb, generator=g) if permute else torch.arange(nb)).to(torch.int32).view(1, nb)
    return k, v, bt, g


# prefill_test.py:95-98
@pytest.mark.parametrize("ctx,q0,qlen,ks,vs", [(2048, 0, 2048, 1.0, 1.0), (2898, 2048, 850, 1.0, 1.0),
                                              (4096, 3840, 256, 1.0, 1.0), (2048, 0, 2048, 0.5, 2.0)])
def test_reference_test_cases(cuda, ctx, q0, qlen, ks, vs):
    import fp8kv_prefill
    k, v, bt, g = _ref_cache(ctx, seed=q0 + qlen)
    q = torch.randn(qlen, HQ, D, generator=g).to(torch.bfloat16)
    out = torch.zeros(qlen, HQ, D, dtype=torch.bfloat16, device=cuda)
    fp8kv_prefill.run(q.to(cuda), k.to(cuda), v.to(cuda), out, bt.to(cuda),
                      torch.tensor([ks], device=cuda), torch.tensor([vs], device=cuda), D ** -0.5,
                      q0, qlen)
    ref = FO.prefill_reference(q, k, v, torch.tensor([0, qlen], dtype=torch.int32),
                               torch.tensor([ctx], dtype=torch.int32), bt, ks, vs, D ** -0.5)
    _check(out, ref)


def test_config3_varlen_through_kv_write(cuda):
    """Config 3: 4 sequences {512, 1024, 1536, 2048} packed with cu_seqlens; bf16
    K/V ~ N(0,1) written into the fp8 paged cache by the KV-write kernel with
    per-tensor amax/448 scales, then attended causally."""
    import fp8kv_prefill
    import kv_cache
    lens = [512, 1024, 1536, 2048]
    T = sum(lens)
    g = torch.Generator().manual_seed(3)
    q = torch.randn(T, HQ, D, generator=g).to(torch.bfloat16)
    key = torch.randn(T, HKV, D, generator=g).to(torch.bfloat16)
    val = torch.randn(T, HKV, D, generator=g).to(torch.bfloat16)
    nblk = [L // PBLK for L in lens]
    nb = sum(nblk) + 8
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(4, max(nblk), dtype=torch.int32)
    slots = torch.empty(T, dtype=torch.int64)
    pos = off = 0
    for s, L in enumerate(lens):
        bt[s, :nblk[s]] = perm[pos:pos + nblk[s]]
        pos += nblk[s]
        t = torch.arange(L)
        slots[off:off + L] = bt[s, t // PBLK].long() * PBLK + t % PBLK
        off += L
    ks = key.float().abs().max().item() / 448.0
    vs = val.float().abs().max().item() / 448.0
    kc = torch.zeros(nb, PBLK, HKV, D, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    kv_cache.reshape_and_cache_flash(key.to(cuda), val.to(cuda), kc, vc, slots.to(cuda), "fp8", ks, vs)
    cu = torch.tensor([0, 512, 1536, 3072, 5120], dtype=torch.int32)
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    out = torch.zeros(T, HQ, D, dtype=torch.bfloat16, device=cuda)
    fp8kv_prefill.prefill_attention(q.to(cuda), kc, vc, out, cu.to(cuda), seq_lens.to(cuda),
                                    bt.to(cuda), ks, vs, D ** -0.5, max_qlen=2048)
    ref = FO.prefill_reference(q, kc.cpu(), vc.cpu(), cu, seq_lens, bt, ks, vs, D ** -0.5)
    _check(out, ref)


@pytest.mark.parametrize("gqa", [1, 2, 8])
def test_gqa_variants_with_continuation(cuda, gqa):
    import fp8kv_prefill
    hkv = 2
    hq = hkv * gqa
    lens_q, lens_kv = [70, 1, 200], [70, 33, 450]   # second and third are continuations
    T = sum(lens_q)
    g = torch.Generator().manual_seed(gqa)
    nblk = [math.ceil(L / PBLK) for L in lens_kv]
    nb = sum(nblk) + 2
    k = (torch.randn(nb, PBLK, hkv, D, generator=g) * 2).to(torch.float8_e4m3fn)
    v = (torch.randn(nb, PBLK, hkv, D, generator=g) * 2).to(torch.float8_e4m3fn)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(3, max(nblk), dtype=torch.int32)
    pos = 0
    for s in range(3):
        bt[s, :nblk[s]] = perm[pos:pos + nblk[s]]
        pos += nblk[s]
    q = torch.randn(T, hq, D, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0, 70, 71, 271], dtype=torch.int32)
    lens = torch.tensor(lens_kv, dtype=torch.int32)
    out = torch.zeros(T, hq, D, dtype=torch.bfloat16, device=cuda)
    fp8kv_prefill.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), out, cu.to(cuda),
                                    lens.to(cuda), bt.to(cuda), 0.7, 1.3, D ** -0.5, max_qlen=200)
    ref = FO.prefill_reference(q, k, v, cu, lens, bt, 0.7, 1.3, D ** -0.5)
    _check(out, ref)


def test_bf16_cache(cuda):
    import fp8kv_prefill
    g = torch.Generator().manual_seed(9)
    nb, ctx = 20, 300
    k = torch.randn(nb, PBLK, HKV, D, generator=g).to(torch.bfloat16)
    v = torch.randn(nb, PBLK, HKV, D, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g).to(torch.int32).view(1, nb)
    q = torch.randn(ctx, HQ, D, generator=g).to(torch.bfloat16)
    out = torch.zeros(ctx, HQ, D, dtype=torch.bfloat16, device=cuda)
    fp8kv_prefill.run(q.to(cuda), k.to(cuda), v.to(cuda), out, bt.to(cuda), 1.0, 1.0, D ** -0.5, 0, ctx)
    ref = FO.prefill_reference(q, k, v, torch.tensor([0, ctx], dtype=torch.int32),
                               torch.tensor([ctx], dtype=torch.int32), bt, 1.0, 1.0, D ** -0.5)
    _check(out, ref)


def _paged_case(lens_q, lens_kv, pblk, seed, hkv=HKV, hq=HQ, unused_bt=0):
    g = torch.Generator().manual_seed(seed)
    nblk = [math.ceil(L / pblk) for L in lens_kv]
    nb = sum(nblk) + 3
    k = (torch.randn(nb, pblk, hkv, D, generator=g) * 2).to(torch.float8_e4m3fn)
    v = (torch.randn(nb, pblk, hkv, D, generator=g) * 2).to(torch.float8_e4m3fn)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.full((len(lens_kv), max(nblk) + 2), unused_bt, dtype=torch.int32)
    pos = 0
    for s, n in enumerate(nblk):
        bt[s, :n] = perm[pos:pos + n]
        pos += n
    T = sum(lens_q)
    q = torch.randn(T, hq, D, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0] + torch.tensor(lens_q).cumsum(0).tolist(), dtype=torch.int32)
    return q, k, v, bt, cu, torch.tensor(lens_kv, dtype=torch.int32)


@pytest.mark.parametrize("pblk", [16, 32, 64, 128])
def test_block_sizes(cuda, pblk):
    """Every block size the TMA page gather takes (one load per page and head)."""
    import fp8kv_prefill
    lens_q, lens_kv = [300, 1, 129], [300, 200, 400]
    q, k, v, bt, cu, lens = _paged_case(lens_q, lens_kv, pblk, seed=pblk)
    out = torch.zeros_like(q, device=cuda)
    fp8kv_prefill.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), out, cu.to(cuda),
                                    lens.to(cuda), bt.to(cuda), 0.8, 1.1, D ** -0.5, max_qlen=300)
    _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 0.8, 1.1, D ** -0.5))


def test_non_finite_bytes_past_the_sequence(cuda):
    """Cache slots past seq_len hold NaN codes and the unused block-table entries
    point outside the cache: neither may reach the output."""
    import fp8kv_prefill
    lens_q, lens_kv = [37, 90], [37, 250]
    q, k, v, bt, cu, lens = _paged_case(lens_q, lens_kv, PBLK, seed=77, unused_bt=1 << 30)
    kb, vb = k.view(torch.uint8), v.view(torch.uint8)
    for s, L in enumerate(lens_kv):
        last = int(bt[s, (L - 1) // PBLK])
        kb[last, L % PBLK or PBLK:] = 0x7F
        vb[last, L % PBLK or PBLK:] = 0x7F
    out = torch.zeros_like(q, device=cuda)
    fp8kv_prefill.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), out, cu.to(cuda),
                                    lens.to(cuda), bt.to(cuda), 1.0, 1.0, D ** -0.5, max_qlen=90)
    assert torch.isfinite(out.float()).all()
    _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 1.0, 1.0, D ** -0.5))


def test_large_dynamic_range_rows(cuda):
    """Query rows spanning 2^-20 .. 2^20 and a peaked softmax: the split
    e4m3 terms of q and p keep the reference's bf16 precision."""
    import fp8kv_prefill
    lens_q, lens_kv = [256], [700]
    q, k, v, bt, cu, lens = _paged_case(lens_q, lens_kv, PBLK, seed=5)
    g = torch.Generator().manual_seed(6)
    scale = torch.exp2(torch.randint(-20, 21, (q.shape[0], q.shape[1], 1), generator=g).float())
    q = (q.float() * scale * 0.05).to(torch.bfloat16)
    q[::7] = (q[::7].float() * 0 + torch.randn(q[::7].shape, generator=g) * 3).to(torch.bfloat16)
    out = torch.zeros_like(q, device=cuda)
    fp8kv_prefill.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), out, cu.to(cuda),
                                    lens.to(cuda), bt.to(cuda), 1.0, 1.0, D ** -0.5, max_qlen=256)
    _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 1.0, 1.0, D ** -0.5))
