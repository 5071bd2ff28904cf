"""ORACLE -- test infrastructure, not product code.

CPU restatement of the reference's attention checkers and of the fp8 e4m3
codec.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs may import this module, and only as the checker or the
timed CPU baseline; the product path (libb200kv.so) never calls it.

Follows:
  * vllm-fp8kv/fp8kv_v3.py:161-167, :171-176   decode reference: dequantise the
      cache (k.float() * k_scale), GQA einsum, fp32 softmax, einsum with V
      (generalised here to per-sequence lengths and a block table)
  * vllm-fp8kv/fp8kv_kernel.py:109-122          same, output row = qsl[s]
  * vllm-fp8kv/prefill_test.py:23-38            prefill reference: causal mask
      `kv position > q0 + row` masked per head (generalised to varlen cu_seqlens
      and per-sequence block tables)
  * fp8 e4m3fn decode from bit fields (OCP 8-bit float spec: bias 7, no inf,
      S.1111.111 = NaN), checked exhaustively against torch.float8_e4m3fn.
Pinned against the reference's own Triton kernels executed on CPU by the
Triton interpreter (tests/golden/gen_golden.py -> tests/golden/*.npz).
"""
import math

import numpy as np
import torch


def e4m3_decode_bits(code):
    """fp8 e4m3fn code (0..255) -> float from the bit fields."""
    code = int(code)
    s, e, m = code >> 7, (code >> 3) & 0xF, code & 7
    if e == 0xF and m == 7:
        return float("nan")
    if e == 0:
        mag = m / 8.0 * 2.0 ** -6
    else:
        mag = (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return -mag if s else mag


def e4m3_table():
    return np.array([e4m3_decode_bits(c) for c in range(256)], dtype=np.float32)


def gather_kv(cache, block_table_row, length):
    """cache [NB, PBLK, HKV, D] -> fp32 [length, HKV, D] in logical token order."""
    pblk = cache.shape[1]
    nblk = (length + pblk - 1) // pblk
    blocks = block_table_row[:nblk].long()
    return cache[blocks].float().reshape(nblk * pblk, cache.shape[2], cache.shape[3])[:length]


def decode_reference(q, k_cache, v_cache, qsl, seq_lens, block_table, k_scale, v_scale,
                     sm_scale, out_by_qsl=False, out_rows=None):
    """fp32 decode attention on CPU.

    q [T, HQ, D] (any float dtype), caches [NB, PBLK, HKV, D] (fp8 or bf16);
    returns fp32 [R, HQ, D] with R = out_rows or (T if out_by_qsl else NS).
    fp8 caches are dequantised with the per-tensor scales (fp8kv_v3.py:171);
    bf16 caches ignore the scales (fp8kv_kernel.py K_FP8=False).
    """
    q = q.cpu()
    k_cache = k_cache.cpu()
    v_cache = v_cache.cpu()
    qsl = qsl.cpu()
    seq_lens = seq_lens.cpu()
    block_table = block_table.cpu()
    fp8 = k_cache.dtype == torch.float8_e4m3fn
    ks = float(k_scale) if fp8 else 1.0
    vs = float(v_scale) if fp8 else 1.0
    ns = block_table.shape[0]
    hq, d = q.shape[1], q.shape[2]
    hkv = k_cache.shape[2]
    gqa = hq // hkv
    if out_rows is None:
        out_rows = q.shape[0] if out_by_qsl else ns
    out = torch.zeros(out_rows, hq, d, dtype=torch.float32)
    for s in range(ns):
        L = int(seq_lens[s])
        row = int(qsl[s]) if out_by_qsl else s
        if L <= 0:
            continue
        kd = gather_kv(k_cache, block_table[s], L) * ks
        vd = gather_kv(v_cache, block_table[s], L) * vs
        qh = q[int(qsl[s])].float().view(hkv, gqa, d)
        for g in range(gqa):
            sc = torch.einsum("hd,nhd->hn", qh[:, g], kd) * sm_scale
            out[row, g::gqa] = torch.einsum("hn,nhd->hd", torch.softmax(sc, -1), vd)
    return out


def prefill_reference(q, k_cache, v_cache, cu_seqlens_q, seq_lens, block_table, k_scale,
                      v_scale, sm_scale):
    """fp32 causal prefill on CPU (prefill_test.py:23-38, varlen).

    Sequence s owns query rows cu[s]..cu[s+1]-1 whose positions are
    q0 + i with q0 = seq_lens[s] - qlen_s; key j is visible iff j <= q0 + i.
    """
    q = q.cpu()
    k_cache = k_cache.cpu()
    v_cache = v_cache.cpu()
    cu = cu_seqlens_q.cpu()
    seq_lens = seq_lens.cpu()
    block_table = block_table.cpu()
    fp8 = k_cache.dtype == torch.float8_e4m3fn
    ks = float(k_scale) if fp8 else 1.0
    vs = float(v_scale) if fp8 else 1.0
    hq, d = q.shape[1], q.shape[2]
    hkv = k_cache.shape[2]
    gqa = hq // hkv
    out = torch.zeros(q.shape[0], hq, d, dtype=torch.float32)
    for s in range(block_table.shape[0]):
        a, b = int(cu[s]), int(cu[s + 1])
        qlen = b - a
        if qlen <= 0:
            continue
        L = int(seq_lens[s])
        q0 = L - qlen
        kd = gather_kv(k_cache, block_table[s], L) * ks
        vd = gather_kv(v_cache, block_table[s], L) * vs
        qf = q[a:b].float()
        rows = torch.arange(qlen) + q0
        mask = torch.arange(L)[None, :] > rows[:, None]
        for h in range(hq):
            kh = h // gqa
            sc = torch.einsum("md,nd->mn", qf[:, h], kd[:, kh]) * sm_scale
            sc = sc.masked_fill(mask, float("-inf"))
            out[a:b, h] = torch.einsum("mn,nd->md", torch.softmax(sc, -1), vd[:, kh])
    return out


def quantize_fp8_per_tensor(x):
    """Per-tensor e4m3 quantisation used by the synthetic configs:
    s = amax / 448, fp8 = (x / s).to(float8_e4m3fn).  Returns (fp8, s)."""
    amax = x.abs().max().float().clamp_min(1e-12)
    s = (amax / 448.0).item()
    return (x.float() / s).to(torch.float8_e4m3fn), s


def make_decode_case(num_seqs, ctx_lens, hq=32, hkv=8, d=128, pblk=16, seed=0,
                     kv_dtype=torch.float8_e4m3fn, pool_extra=8):
    """Config-1 style synthetic decode inputs (CPU tensors).

    K/V ~ N(0,1) quantised per tensor (amax/448); each sequence gets a random
    permutation of pool blocks; q ~ N(0,1) bf16; one query token per sequence.
    Returns dict with q, k_cache, v_cache, qsl, seq_lens, block_table, k_scale,
    v_scale, sm_scale.
    """
    g = torch.Generator().manual_seed(seed)
    ctx_lens = list(ctx_lens)
    blocks_per = [max(1, math.ceil(L / pblk)) for L in ctx_lens]
    maxblk = max(blocks_per)
    nb = sum(blocks_per) + pool_extra
    kf = torch.randn(nb, pblk, hkv, d, generator=g)
    vf = torch.randn(nb, pblk, hkv, d, generator=g)
    if kv_dtype == torch.float8_e4m3fn:
        kc, ks = quantize_fp8_per_tensor(kf)
        vc, vs = quantize_fp8_per_tensor(vf)
    else:
        kc, ks = kf.to(kv_dtype), 1.0
        vc, vs = vf.to(kv_dtype), 1.0
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(num_seqs, maxblk, dtype=torch.int32)
    pos = 0
    for s in range(num_seqs):
        bt[s, :blocks_per[s]] = perm[pos:pos + blocks_per[s]]
        pos += blocks_per[s]
    q = torch.randn(num_seqs, hq, d, generator=g).to(torch.bfloat16)
    return dict(q=q, k_cache=kc, v_cache=vc,
                qsl=torch.arange(num_seqs + 1, dtype=torch.int32),
                seq_lens=torch.tensor(ctx_lens, dtype=torch.int32),
                block_table=bt, k_scale=ks, v_scale=vs, sm_scale=d ** -0.5)
