"""Config 5 (the serving shape) on sampled sequences against the CPU oracle
(oracle/fp8kv_oracle.py: the reference's prefill / decode attention): a mixed
batch of decode rows at long contexts (up to 32k, as config 5 draws them) and
new prefills over one fragmented fp8 pool, run the two ways the serving step
runs it -- one varlen call for the whole batch (what the vLLM forward patch
does) and the decode kernel for the decode rows plus the varlen kernel for the
prefills.  Tolerance as the other attention tests: max abs error < 0.05 and
< 2e-2 of the largest output."""
import math

import pytest
import torch

import fp8kv_oracle as FO

pytestmark = pytest.mark.gpu

HQ, HKV, D, PBLK = 32, 8, 128, 16
ATOL, RTOL = 0.05, 2e-2


def _check(got, ref):
    got = got.float().cpu()
    err = (got - ref).abs().max().item()
    rel = err / max(ref.abs().max().item(), 1e-30)
    assert err < ATOL and rel < RTOL, (err, rel)


def _serving_case(ctx, prefills, seed, prefill_ctx=()):
    """Decode rows at contexts `ctx` (one new token each), new prefills of
    lengths `prefills` and continued prefills (kv length, query rows) in
    `prefill_ctx`, pages of every sequence drawn from one permutation."""
    g = torch.Generator().manual_seed(seed)
    seq = [c + 1 for c in ctx] + list(prefills) + [L for L, _ in prefill_ctx]
    qlens = [1] * len(ctx) + list(prefills) + [ql for _, ql in prefill_ctx]
    nblk = [math.ceil(L / PBLK) for L in seq]
    nb = sum(nblk) + 5
    k = (torch.randn(nb, PBLK, HKV, D, generator=g) * 2).to(torch.float8_e4m3fn)
    v = (torch.randn(nb, PBLK, HKV, D, generator=g) * 2).to(torch.float8_e4m3fn)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(len(seq), max(nblk), dtype=torch.int32)
    pos = 0
    for s, n in enumerate(nblk):
        bt[s, :n] = perm[pos:pos + n]
        pos += n
    T = sum(qlens)
    q = torch.randn(T, HQ, D, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32)
    return q, k, v, bt, cu, torch.tensor(seq, dtype=torch.int32)


CTX = [30001, 2048, 17000, 32768, 5000]
PRE = [384, 129]


def test_mixed_batch_one_varlen_call(cuda):
    import fp8kv_prefill
    q, k, v, bt, cu, lens = _serving_case(CTX, PRE, seed=1)
    out = torch.zeros_like(q, device=cuda)
    fp8kv_prefill.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), out, cu.to(cuda), lens.to(cuda),
                                    bt.to(cuda), 0.9, 1.2, D ** -0.5, max_qlen=max(PRE))
    _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 0.9, 1.2, D ** -0.5))


def test_split_decode_rows_and_prefills(cuda):
    """Decode kernel on the decode rows, varlen kernel on the prefills (views
    into the same q / out / block table, as the serving step slices them)."""
    import _decode
    import fp8kv_prefill
    q, k, v, bt, cu, lens = _serving_case(CTX, PRE, seed=2)
    nd = len(CTX)
    qd, kd, vd, btd, lensd = q.to(cuda), k.to(cuda), v.to(cuda), bt.to(cuda), lens.to(cuda)
    out = torch.zeros_like(qd)
    qsl = torch.arange(nd + 1, dtype=torch.int32, device=cuda)
    _decode.decode_attention(qd, kd, vd, out, qsl, lensd[:nd], btd[:nd], 0.9, 1.2, D ** -0.5,
                             out_by_qsl=True, max_seq_len_hint=max(CTX) + 1)
    cu_pre = (cu[nd:] - nd).to(cuda)
    fp8kv_prefill.prefill_attention(qd[nd:], kd, vd, out[nd:], cu_pre, lensd[nd:], btd[nd:], 0.9, 1.2,
                                    D ** -0.5, max_qlen=max(PRE))
    _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 0.9, 1.2, D ** -0.5))


def test_device_split_entry(cuda):
    """b200kv_attn_varlen_mixed (the forward patch's path for mixed batches):
    one-token sequences on the decode kernel, the rest on the varlen kernel,
    chosen on the device; within tolerance of the oracle and bit for bit equal
    to the two separate calls of the split arrangement."""
    import _decode
    import fp8kv_prefill
    q, k, v, bt, cu, lens = _serving_case(CTX, PRE, seed=3)
    qd, kd, vd, btd, lensd, cud = q.to(cuda), k.to(cuda), v.to(cuda), bt.to(cuda), lens.to(cuda), cu.to(cuda)
    out = torch.full_like(qd, float("nan"))
    fp8kv_prefill.mixed_attention(qd, kd, vd, out, cud, lensd, btd, 0.9, 1.2, D ** -0.5,
                                  max_qlen=max(PRE), max_seq_len=max(CTX) + 1)
    _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 0.9, 1.2, D ** -0.5))
    nd = len(CTX)
    ref = torch.zeros_like(qd)
    qsl = torch.arange(nd + 1, dtype=torch.int32, device=cuda)
    _decode.decode_attention(qd, kd, vd, ref, qsl, lensd[:nd], btd[:nd], 0.9, 1.2, D ** -0.5,
                             out_by_qsl=True, max_seq_len_hint=max(CTX) + 1)
    fp8kv_prefill.prefill_attention(qd[nd:], kd, vd, ref[nd:], (cud[nd:] - nd).contiguous(), lensd[nd:],
                                    btd[nd:], 0.9, 1.2, D ** -0.5, max_qlen=max(PRE))
    assert torch.equal(out, ref)


def test_device_split_all_decode_and_all_prefill(cuda):
    """Batches with only one-token sequences, or none, through the same entry."""
    import fp8kv_prefill
    for ctx, pre in (([3000, 100, 7000], []), ([], [200, 33, 512])):
        q, k, v, bt, cu, lens = _serving_case(ctx, pre, seed=4 + len(ctx))
        out = torch.full_like(q, float("nan"), device=cuda)
        fp8kv_prefill.mixed_attention(q.to(cuda), k.to(cuda), v.to(cuda), out, cu.to(cuda), lens.to(cuda),
                                      bt.to(cuda), 1.0, 1.0, D ** -0.5, max_qlen=max(pre, default=1),
                                      max_seq_len=int(lens.max()))
        _check(out, FO.prefill_reference(q, k, v, cu, lens, bt, 1.0, 1.0, D ** -0.5))


def _prefill_raw(cuda, q, k, v, out, cu, lens, bt, num_tokens, max_qlen):
    """b200kv_prefill_attn's varlen form with an explicit num_tokens (0 = the
    dense grid of num_seqs x max_qlen's tile pairs)."""
    from _b200kv import KV_FP8_E4M3, check, lib
    ks = torch.tensor([0.9], device=cuda)
    vs = torch.tensor([1.2], device=cuda)
    check(lib.b200kv_prefill_attn(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        v.stride(0), v.stride(1), v.stride(2), out.data_ptr(), out.stride(0), out.stride(1), cu.data_ptr(),
        lens.data_ptr(), bt.data_ptr(), bt.stride(0), ks.data_ptr(), vs.data_ptr(), D ** -0.5,
        bt.shape[0], max_qlen, 0, 0, q.shape[1], k.shape[2], q.shape[2], k.shape[1], k.shape[0], KV_FP8_E4M3,
        num_tokens, torch.cuda.current_stream(cuda).cuda_stream), "b200kv_prefill_attn")
    return out


@pytest.mark.parametrize("qlens", [[1, 700, 1, 1, 65, 64, 63, 1, 2], [5] * 40 + [300], [1] * 37 + [129, 1, 2]])
def test_compact_grid_equals_dense_grid(cuda, qlens):
    """With the batch's token count the varlen kernel's grid enumerates the
    batch's (sequence, tile pair) items instead of num_seqs x the longest
    sequence's pairs: every item is computed as before, so the outputs are
    bit for bit those of the dense grid (ragged, one-token and more than 32
    sequences, so the item scan crosses its chunks of 32)."""
    ctx = [q + 37 * (i % 5) for i, q in enumerate(qlens)]
    q, k, v, bt, cu, lens = _serving_case([], [], seed=7, prefill_ctx=list(zip(ctx, qlens)))
    qd, kd, vd, btd, lensd, cud = q.to(cuda), k.to(cuda), v.to(cuda), bt.to(cuda), lens.to(cuda), cu.to(cuda)
    dense = _prefill_raw(cuda, qd, kd, vd, torch.full_like(qd, float("nan")), cud, lensd, btd, 0, max(qlens))
    compact = _prefill_raw(cuda, qd, kd, vd, torch.full_like(qd, float("nan")), cud, lensd, btd, q.shape[0],
                           max(qlens))
    assert torch.equal(dense, compact)
    _check(compact, FO.prefill_reference(q, k, v, cu, lens, bt, 0.9, 1.2, D ** -0.5))
