"""Paged-KV decode attention on the B200 against the CPU oracle and against the
REFERENCE's own Triton kernels (fixtures run on CPU by the Triton interpreter).

Tolerances: the reference's own bound, max abs < 0.05
(vllm-fp8kv/fp8kv_v3.py:168), and max|out - ref| / max|ref| < 2e-2 (the
north-star's fp32-accumulate bound) against the fp32 oracle.
"""
import math

import pytest
import torch

import fp8kv_oracle as FO
from test_oracle_pins import CASES, DEC, golden_decode_inputs, _bf16

pytestmark = pytest.mark.gpu

ATOL = 0.05
RTOL = 2e-2


def _to(case, dev):
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in case.items()}


def _check(got, ref, rows=None):
    got = got.float().cpu()
    if rows is not None:
        got, ref = got[rows], ref[rows]
    err = (got - ref).abs().max().item()
    rel = err / max(ref.abs().max().item(), 1e-30)
    assert err < ATOL and rel < RTOL, (err, rel)
    return err


def _run_v3(c, dev, **kw):
    import fp8kv_v3
    g = _to(c, dev)
    ns = g["block_table"].shape[0]
    out = torch.full((ns, g["q"].shape[1], g["q"].shape[2]), float("nan"),
                     dtype=torch.bfloat16, device=dev)
    fp8kv_v3.run(g["q"], g["k_cache"], g["v_cache"], out, g["qsl"], g["seq_lens"],
                 g["block_table"], g["k_scale"], g["v_scale"], g["sm_scale"], **kw)
    return out


@pytest.mark.parametrize("name", DEC)
def test_golden_reference_kernel_cases(cuda, name):
    import fp8kv_kernel
    import fp8kv_v3
    a = golden_decode_inputs(CASES[name])
    g = _to(a, cuda)
    T = g["q"].shape[0]
    out = torch.zeros(T, g["q"].shape[1], 128, dtype=torch.bfloat16, device=cuda)
    ks = torch.tensor([a["k_scale"]], device=cuda)
    vs = torch.tensor([a["v_scale"]], device=cuda)
    if a["out_by_qsl"]:
        fp8kv_kernel.run(g["q"], g["k_cache"], g["v_cache"], out, g["qsl"], g["seq_lens"],
                         g["block_table"], ks, vs, a["sm_scale"])
        rows = a["qsl"][:-1].long()
    else:
        fp8kv_v3.run(g["q"], g["k_cache"], g["v_cache"], out, g["qsl"], g["seq_lens"],
                     g["block_table"], ks, vs, a["sm_scale"], nsplit=a["nsplit"])
        rows = torch.arange(a["seq_lens"].numel())
    ref_kernel = _bf16(CASES[name]["out"]).float()
    _check(out, ref_kernel, rows)   # against the reference's own kernel output
    ref = FO.decode_reference(a["q"], a["k_cache"], a["v_cache"], a["qsl"], a["seq_lens"],
                              a["block_table"], a["k_scale"], a["v_scale"], a["sm_scale"],
                              out_by_qsl=a["out_by_qsl"], out_rows=T)
    _check(out, ref, rows)


@pytest.mark.parametrize("batch", [1, 4, 8])
def test_config1_ctx4096(cuda, batch):
    c = FO.make_decode_case(batch, [4096] * batch, seed=batch)
    out = _run_v3(c, cuda)
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


LENS = [1, 2, 15, 16, 17, 63, 64, 65, 255, 256, 257, 511, 1000, 2049]


@pytest.mark.parametrize("gqa", [1, 2, 4, 8])
def test_ragged_lengths_all_gqa(cuda, gqa):
    hkv = 2
    c = FO.make_decode_case(len(LENS), LENS, hq=hkv * gqa, hkv=hkv, seed=10 + gqa)
    out = _run_v3(c, cuda)
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


@pytest.mark.parametrize("nsplit", [1, 2, 3, 8, 16])
def test_explicit_split_counts(cuda, nsplit):
    c = FO.make_decode_case(3, [3000, 17, 1500], seed=20)
    out = _run_v3(c, cuda, nsplit=nsplit)
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


def test_bf16_kv_cache(cuda):
    import fp8kv_kernel
    c = FO.make_decode_case(4, [100, 4096, 1, 777], kv_dtype=torch.bfloat16, seed=30)
    g = _to(c, cuda)
    out = torch.zeros(4, 32, 128, dtype=torch.bfloat16, device=cuda)
    one = torch.ones(1, device=cuda)
    fp8kv_kernel.run(g["q"], g["k_cache"], g["v_cache"], out, g["qsl"], g["seq_lens"],
                     g["block_table"], one, one, c["sm_scale"])
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], 1.0, 1.0, c["sm_scale"], out_by_qsl=True)
    _check(out, ref)


def test_scale_folding(cuda):
    # fp8kv_v3.py:169-177: cache = (randn * 2) cast straight to fp8, then ks = 0.5, vs = 2.0
    c = FO.make_decode_case(2, [4096, 300], seed=40)
    g = torch.Generator().manual_seed(41)
    c["k_cache"] = (torch.randn(c["k_cache"].shape, generator=g) * 2).to(torch.float8_e4m3fn)
    c["v_cache"] = (torch.randn(c["v_cache"].shape, generator=g) * 2).to(torch.float8_e4m3fn)
    c["k_scale"], c["v_scale"] = 0.5, 2.0
    out = _run_v3(c, cuda)
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], 0.5, 2.0, c["sm_scale"])
    _check(out, ref)


def test_zero_length_sequence_gives_zeros(cuda):
    c = FO.make_decode_case(3, [10, 0, 20], seed=50)
    out = _run_v3(c, cuda)
    assert torch.all(out[1] == 0)
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref, torch.tensor([0, 2]))


def test_vllm_interleaved_cache_layout(cuda):
    """vLLM 0.22 TritonAttention cache: [NB, 2, PBLK, HKV, D], K/V via unbind(1),
    so the K and V views are non-contiguous with block stride 2*PBLK*HKV*D."""
    c = FO.make_decode_case(2, [700, 4096], seed=60)
    nb = c["k_cache"].shape[0]
    kv = torch.stack([c["k_cache"].view(torch.uint8), c["v_cache"].view(torch.uint8)], 1)
    kv = kv.view(torch.float8_e4m3fn).to(cuda)
    k, v = kv.unbind(1)
    assert not k.is_contiguous()
    g = _to(c, cuda)
    import fp8kv_v3
    out = torch.zeros(2, 32, 128, dtype=torch.bfloat16, device=cuda)
    fp8kv_v3.run(g["q"], k, v, out, g["qsl"], g["seq_lens"], g["block_table"],
                 c["k_scale"], c["v_scale"], c["sm_scale"])
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


def test_block_table_index_probe(cuda):
    """One-hot V at a single logical token behind a permuted table, with K
    making that token dominate: the output must equal that V row exactly."""
    for target in (0, 15, 16, 1000, 4095):
        c = FO.make_decode_case(1, [4096], hq=4, hkv=1, seed=70)
        k = torch.zeros_like(c["k_cache"].float())
        v = torch.zeros_like(k)
        pblk = k.shape[1]
        blk = int(c["block_table"][0, target // pblk])
        slot = target % pblk
        k[blk, slot, 0, :] = 8.0
        v[blk, slot, 0, :] = torch.linspace(-4, 4, 128)
        c["k_cache"] = k.to(torch.float8_e4m3fn)
        c["v_cache"] = v.to(torch.float8_e4m3fn)
        c["q"] = torch.full_like(c["q"].float(), 8.0).to(torch.bfloat16)
        c["k_scale"] = c["v_scale"] = 1.0
        out = _run_v3(c, cuda).float().cpu()
        want = v[blk, slot, 0].to(torch.float8_e4m3fn).float().to(torch.bfloat16).float()
        assert torch.equal(out[0, 0], want), target


@pytest.mark.parametrize("hint", [0, 32768])
def test_long_context_32k(cuda, hint):
    c = FO.make_decode_case(2, [32768, 20000], hq=8, hkv=2, seed=80)
    out = _run_v3(c, cuda, max_seq_len=hint)
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


def test_determinism(cuda):
    import _b200kv
    c = FO.make_decode_case(4, [4096, 33, 2000, 4096], seed=90)
    a = _run_v3(c, cuda)
    b = _run_v3(c, cuda)
    assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert _b200kv.device_status() == 0


def test_cuda_graph_capture(cuda):
    import fp8kv_v3
    c = FO.make_decode_case(2, [4096, 123], seed=95)
    g = _to(c, cuda)
    ks = torch.tensor([c["k_scale"]], device=cuda)
    vs = torch.tensor([c["v_scale"]], device=cuda)
    out = torch.zeros(2, 32, 128, dtype=torch.bfloat16, device=cuda)
    args = (g["q"], g["k_cache"], g["v_cache"], out, g["qsl"], g["seq_lens"], g["block_table"],
            ks, vs, c["sm_scale"])
    fp8kv_v3.run(*args)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            fp8kv_v3.run(*args)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    ref = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                              c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
    _check(out, ref)


# ---- the two page-load paths: TMA page tiles (fp8, block 16/32/64/128, pool
# size known) and the per-row asynchronous-copy gather (everything else, or
# B200KV_DECODE_TMA=0) -------------------------------------------------------
def _oracle(c):
    return FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                               c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])


@pytest.mark.parametrize("path", ["tma", "gather"])
@pytest.mark.parametrize("pblk", [16, 32, 64, 128, 48])
def test_block_sizes_both_paths(cuda, monkeypatch, path, pblk):
    if path == "gather":
        monkeypatch.setenv("B200KV_DECODE_TMA", "0")
    lens = [1, 47, 129, 1000, 4096, 2500]
    c = FO.make_decode_case(len(lens), lens, pblk=pblk, seed=100 + pblk)
    _check(_run_v3(c, cuda), _oracle(c))


def test_paths_agree_bit_for_bit(cuda, monkeypatch):
    """Both paths take the same per-token products in the same order (the TMA
    path only permutes MMA rows), so their outputs are identical."""
    lens = [4096, 33, 2000, 700, 1, 4096, 3333, 129]
    c = FO.make_decode_case(len(lens), lens, seed=110)
    a = _run_v3(c, cuda)
    monkeypatch.setenv("B200KV_DECODE_TMA", "0")
    b = _run_v3(c, cuda)
    assert torch.equal(a, b)


@pytest.mark.parametrize("pblk", [16, 64])
def test_nan_codes_past_the_sequence(cuda, pblk):
    """Slots of the last page past seq_len, and every unused pool block, hold
    0x7F (an fp8 NaN): they must not reach the output."""
    lens = [5, 100, 1023, 4095]
    c = FO.make_decode_case(len(lens), lens, pblk=pblk, seed=120)
    kc = c["k_cache"].view(torch.uint8).clone()
    vc = c["v_cache"].view(torch.uint8).clone()
    used = torch.zeros(kc.shape[0], pblk, dtype=torch.bool)
    for s, L in enumerate(lens):
        for t in range(L):
            used[int(c["block_table"][s, t // pblk]), t % pblk] = True
    kc[~used] = 0x7F
    vc[~used] = 0x7F
    c["k_cache"], c["v_cache"] = kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn)
    out = _run_v3(c, cuda)
    assert torch.isfinite(out.float()).all()
    _check(out, _oracle(c))


@pytest.mark.parametrize("ring", ["64", "128", "128w8"])
@pytest.mark.parametrize("pblk", [16, 32, 64])
def test_ring_shapes(cuda, monkeypatch, ring, pblk):
    """Every ring shape of the TMA kernel (128-token stages with four or eight
    compute warps, 64-token stages with four) over ragged lengths, partial
    stages and one- and many-stage shares."""
    monkeypatch.setenv("B200KV_DECODE_RING", ring)
    lens = [1, 47, 63, 64, 65, 129, 1000, 4096]
    c = FO.make_decode_case(len(lens), lens, pblk=pblk, seed=130 + pblk)
    _check(_run_v3(c, cuda), _oracle(c))
    for nsplit in (1, 16):
        c1 = FO.make_decode_case(1, [4096], seed=140 + nsplit)
        _check(_run_v3(c1, cuda, nsplit=nsplit), _oracle(c1))

