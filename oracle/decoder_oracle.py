"""ORACLE -- test infrastructure, not product code.

CPU restatement, in fp32 with the model dtype's (bf16) rounding points, of one
decode step of the 7B-class decoder the reference serves (HF Llama layout:
RMSNorm, fused qkv, neox rotary embedding, GQA attention over the paged fp8
cache, o, residual, RMSNorm, SwiGLU MLP, residual; final RMSNorm and a bf16
lm_head).  The hot-path pieces are the other oracles' (mxfp4_oracle's
dequant + fp32 matmul, fp8kv_oracle's decode attention, the KV write's
(x / scale).to(float8_e4m3fn)); the glue follows HF's formulas:
  * RMSNorm: y = w * bf16(h32 * rsqrt(mean(h32^2) + eps))
  * rotary:  theta^(-2i/d) frequencies, (x1, x2) -> (x1 c - x2 s, x2 c + x1 s)
             on the two halves of each head (rotate_half), fp32, one rounding
  * SwiGLU:  bf16(bf16(silu(g)) * u)
  * residual: h = bf16(h + delta)
  * KV write: e4m3(x / scale) saturated at +-448
Only tests/ and bench.py's CPU legs may import this module.
"""
import torch

import fp8kv_oracle as FO
import mxfp4_oracle as MO


def rope_table(max_pos, head_dim, theta):
    """fp32 [max_pos, head_dim]: cos of the head_dim/2 frequencies, then sin
    (angles in float64, rounded once)."""
    inv = theta ** (-torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], 1).float()


def rmsnorm(h, w, eps):
    h32 = h.float()
    r = torch.rsqrt(h32.pow(2).mean(-1, keepdim=True) + eps)
    return ((h32 * r).to(torch.bfloat16).float() * w.float()).to(torch.bfloat16)


def rope(x, pos, table):
    """x bf16 [..., heads, d] of one token at position pos."""
    d = x.shape[-1]
    half = d // 2
    c, s = table[pos, :half], table[pos, half:]
    x32 = x.float()
    x1, x2 = x32[..., :half], x32[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(torch.bfloat16)


def swiglu(gu, inter):
    g, u = gu[..., :inter].float(), gu[..., inter:].float()
    s = (g * torch.sigmoid(g)).to(torch.bfloat16).float()
    return (s * u).to(torch.bfloat16)


def fp8_saturate(x):
    """e4m3 with saturation at +-448 (the KV write's satfinite convert; a
    plain torch cast would turn out-of-range values into NaN)."""
    return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


def linear(x, W, S):
    """MXFP4 linear: W [N, K/2] packed, S [K/32, N] e8m0 -> bf16 [M, N]."""
    return MO.mxfp4_linear_reference(W, S, x).to(torch.bfloat16)


def linear_rowpar(x, W, S, tp):
    """Row-parallel MXFP4 linear over tp ranks, as tensor parallelism computes
    it: each rank's K slice gives an fp32 partial rounded to bf16, the partials
    are summed in rank order in fp32 and rounded to bf16 (the allreduce)."""
    if tp == 1:
        return linear(x, W, S)
    K = x.shape[1]
    k = K // tp
    acc = None
    for r in range(tp):
        part = MO.mxfp4_linear_reference(W[:, r * k // 2:(r + 1) * k // 2],
                                         S[r * k // 32:(r + 1) * k // 32], x[:, r * k:(r + 1) * k])
        part = part.to(torch.bfloat16).float()
        acc = part if acc is None else acc + part
    return acc.to(torch.bfloat16)


def decode_step(cfg, weights, caches, tokens, positions, block_table, table, tp=1):
    """One decode step for B sequences; caches (per layer dict k, v, ks, vs) are
    updated in place with the new tokens' K/V.  tp > 1 rounds the row-parallel
    o and down partials as tensor parallelism does.  Returns fp32 logits [B, V]."""
    B = tokens.shape[0]
    H, hq, hkv, d, inter = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.inter
    bs = cfg.block_size
    h = weights["embed"][tokens.long()].clone()
    for li, lw in enumerate(weights["layers"]):
        x = rmsnorm(h, lw["in_norm"], cfg.eps)
        qkv = linear(x, *lw["qkv"]).view(B, hq + 2 * hkv, d)
        c = caches[li]
        q = torch.empty(B, hq, d, dtype=torch.bfloat16)
        for b in range(B):
            p = int(positions[b])
            q[b] = rope(qkv[b, :hq], p, table)
            k = rope(qkv[b, hq:hq + hkv], p, table)
            v = qkv[b, hq + hkv:]
            blk, off = int(block_table[b, p // bs]), p % bs
            c["k"][blk, off] = fp8_saturate(k.float() / c["ks"])
            c["v"][blk, off] = fp8_saturate(v.float() / c["vs"])
        seq_lens = (positions + 1).to(torch.int32)
        qsl = torch.arange(B + 1, dtype=torch.int32)
        attn = FO.decode_reference(q, c["k"], c["v"], qsl, seq_lens, block_table, c["ks"], c["vs"],
                                   d ** -0.5).to(torch.bfloat16)
        o = linear_rowpar(attn.reshape(B, hq * d), *lw["o"], tp)
        h = (h.float() + o.float()).to(torch.bfloat16)
        x = rmsnorm(h, lw["post_norm"], cfg.eps)
        act = swiglu(linear(x, *lw["gate_up"]), inter)
        dn = linear_rowpar(act, *lw["down"], tp)
        h = (h.float() + dn.float()).to(torch.bfloat16)
    x = rmsnorm(h, weights["final_norm"], cfg.eps)
    return x.float() @ weights["lm_head"].float().t()
