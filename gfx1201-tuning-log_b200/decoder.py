"""The 7B-class MXFP4 decoder of the reference's benchmarks (config 4), decode
loop on b200kv's kernels.

HF Llama layout: per layer RMSNorm -> fused qkv (MXFP4) -> rotary embedding +
paged fp8 KV write -> decode attention -> o (MXFP4) -> residual + RMSNorm ->
gate_up (MXFP4) -> SwiGLU -> down (MXFP4) -> residual; final RMSNorm, bf16
lm_head, greedy argmax.  Random-init weights (config 2's MXFP4 distribution:
codes uniform over the 16 values, e8m0 scales uniform in 2^-8..2^-2), bf16
embeddings and lm_head.  Tensor parallel over `tp` ranks as in tp.py, the
lm_head vocab-parallel with a (max, index) gather for the argmax.

A decode step reads tokens, positions and the block tables from device
tensors and advances them on the device, so it can be captured once in a CUDA
graph and replayed token after token.  prefill() runs a prompt through the
same layers with the wide MXFP4 GEMM, the fused RoPE + KV write and the varlen
causal prefill kernel, so the decode loop continues from a cache the prefill
wrote.
"""
from dataclasses import dataclass

import torch

import fp8kv_prefill
import fp8kv_v3
import h4mv
from _b200kv import KV_BF16, KV_FP8_E4M3, check, lib


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 14336
    vocab: int = 128256
    rope_theta: float = 1e6
    eps: float = 1e-5
    block_size: int = 16


SEVEN_B = DecoderConfig()


def rope_table(max_pos, head_dim, theta):
    """fp32 [max_pos, head_dim]: cos of the head_dim/2 rotary frequencies
    theta^(-2i/head_dim), then their sin; angles in float64, rounded once."""
    inv = theta ** (-torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], 1).float()


CONFIG2_SCALES = (119, 126)  # e8m0 bytes drawn from [lo, hi): 2^-8 .. 2^-2


def _mxfp4(g, n, k, device, scales):
    W = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=g)
    St = torch.randint(scales[0], scales[1], (n, k // 32), dtype=torch.uint8, device=device, generator=g)
    return W, St


def random_layer(cfg, li, seed, device="cpu", scales=CONFIG2_SCALES):
    """Full (unsharded) weights of layer li: MXFP4 (W [N, K/2], St [N, K/32])
    for qkv ([q | k | v] rows), o, gate_up ([gate | up] rows), down; bf16 norms.
    Every rank draws the same layer from the same seed and keeps its shard."""
    g = torch.Generator(device=device).manual_seed(seed * 1000 + li)
    H, d = cfg.hidden, cfg.head_dim
    nqkv = (cfg.heads + 2 * cfg.kv_heads) * d
    lay = {"qkv": _mxfp4(g, nqkv, H, device, scales), "o": _mxfp4(g, H, cfg.heads * d, device, scales),
           "gate_up": _mxfp4(g, 2 * cfg.inter, H, device, scales),
           "down": _mxfp4(g, H, cfg.inter, device, scales)}
    for name in ("in_norm", "post_norm"):
        lay[name] = (1.0 + 0.1 * torch.randn(H, device=device, generator=g)).to(torch.bfloat16)
    return lay


def random_head(cfg, seed, device="cpu"):
    """bf16 embeddings, lm_head ~ N(0, 1) * 0.02 and 1.0 scale, final norm."""
    g = torch.Generator(device=device).manual_seed(seed * 1000 + 999)
    emb = (torch.randn(cfg.vocab, cfg.hidden, device=device, generator=g)).to(torch.bfloat16)
    head = (0.02 * torch.randn(cfg.vocab, cfg.hidden, device=device, generator=g)).to(torch.bfloat16)
    fnorm = (1.0 + 0.1 * torch.randn(cfg.hidden, device=device, generator=g)).to(torch.bfloat16)
    return {"embed": emb, "lm_head": head, "final_norm": fnorm}


def shard_layer(lay, cfg, rank, tp):
    """This rank's shard of a full layer (tp.py's layout)."""
    import tp as tpm
    if tp == 1:
        return dict(lay)
    inter = cfg.inter
    gu_rows = torch.cat([torch.arange(rank * inter // tp, (rank + 1) * inter // tp),
                         inter + torch.arange(rank * inter // tp, (rank + 1) * inter // tp)])
    W, St = lay["gate_up"]
    gu_rows = gu_rows.to(W.device)
    return {
        "qkv": tpm.qkv_shard(*lay["qkv"], cfg.heads, cfg.kv_heads, cfg.head_dim, rank, tp),
        "o": tpm.row_shard(*lay["o"], rank, tp),
        "gate_up": (W.index_select(0, gu_rows).contiguous(), St.index_select(0, gu_rows).contiguous()),
        "down": tpm.row_shard(*lay["down"], rank, tp),
        "in_norm": lay["in_norm"], "post_norm": lay["post_norm"],
    }


def _linear(W, St, device, kernel="auto"):
    """Weights on the device with their scales in the layout of the faster
    kernel: tensor-core atoms when K % 128 == 0 and no edge byte, else (or
    with kernel="mma.sync") the transposed scales of the mma.sync kernel."""
    W = W.to(device).contiguous()
    St = St.to(device).contiguous()
    N, K = W.shape[0], W.shape[1] * 2
    if K % 128 == 0 and kernel == "auto":
        packed, edge = h4mv.pack_scales(St, N, K)
        if not edge:
            return ("tc", W, packed)
    return ("mv", W, St)


def _gate_up_linear(W, St, inter, device, kernel="auto", fuse=True):
    """gate_up ([gate | up] rows, `inter` each) prepared for the GEMM with the
    SwiGLU epilogue when the tensor-core kernels take it: rows (and their
    scales) permuted once to h4mv.gate_up_row_order, kind "tcsw".  Otherwise
    the plain layout, and the SwiGLU runs as its own kernel."""
    if fuse and kernel == "auto" and inter % 64 == 0 and W.shape[0] == 2 * inter:
        order = h4mv.gate_up_row_order(inter, W.device)
        lin = _linear(W.index_select(0, order), St.index_select(0, order), device, kernel)
        if lin[0] == "tc":
            return ("tcsw",) + lin[1:]
    return _linear(W, St, device, kernel)


def _gate_up(x, lin, gu, act, inter, stream):
    """act = SwiGLU(x @ gate_up^T): one launch on "tcsw" weights, else the
    product into gu and the SwiGLU kernel."""
    if lin[0] == "tcsw":
        return h4mv.mxfp4_gemm_swiglu(x, lin[1], lin[2], out=act)
    _gemm(x, lin, gu)
    check(lib.b200kv_swiglu(gu.data_ptr(), act.data_ptr(), x.shape[0], inter, stream), "b200kv_swiglu")
    return act


def _gemm(x, lin, out):
    kind, W, S = lin
    if kind == "tc":  # M > 8 goes to the wide-batch GEMM
        return h4mv.mxfp4_gemm(x, W, S, out=out)
    for m0 in range(0, x.shape[0], h4mv.MAX_M):  # the mma.sync matvec, 8 rows at a time
        h4mv.mxfp4_gemv(x[m0:m0 + h4mv.MAX_M], W, S, out=out[m0:m0 + h4mv.MAX_M])
    return out


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


class MXFP4Decoder:
    """Decode loop of `batch` sequences with room for `max_ctx` tokens each.

    tp/rank/allreduce: this rank's part of a tensor-parallel group (allreduce
    sums a bf16 tensor in place over the group, e.g. tp.PeerAllreduce;
    gather(out, inp) all-gathers a float32 tensor, for the argmax).  Weights are
    drawn on `gen_device` (CPU in tests, so the oracle sees the same numbers).
    fuse_swiglu: gate_up runs with the SwiGLU epilogue (rows permuted at load
    time) wherever the tensor-core kernels take the weights.  fuse_allreduce:
    under tensor parallelism with a tp.PeerAllreduce, the decode step's o and
    down products run with the allreduce in their epilogue (one launch each,
    bit for bit the product followed by the allreduce); off by default, as it
    measured slower than the product followed by the one-shot allreduce.
    fuse_rope: the decode step's qkv product runs with the rotary embedding and
    the fp8 KV write in its epilogue (one launch, bit for bit the product
    followed by b200kv_rope_kv_write) wherever the tensor-core kernel takes it."""

    def __init__(self, cfg, device, batch, max_ctx, seed=0, tp=1, rank=0, allreduce=None,
                 gather=None, kv_scale=1.0 / 8, gen_device=None, layers=None, mxfp4_kernel="auto",
                 scales=CONFIG2_SCALES, fuse_swiglu=True, fuse_allreduce=False, fuse_rope=True):
        self.cfg, self.dev, self.B, self.tp, self.rank = cfg, device, batch, tp, rank
        self.allreduce = allreduce if allreduce is not None else (lambda t: t)
        self._fused_ar = fuse_allreduce and tp > 1 and hasattr(allreduce, "gemm")
        self._fuse_rope = fuse_rope
        self.gather = gather
        if cfg.heads % tp or cfg.kv_heads % tp or cfg.inter % tp or cfg.vocab % tp:
            raise ValueError("model does not divide over tp")
        self.hq, self.hkv = cfg.heads // tp, cfg.kv_heads // tp
        gdev = gen_device if gen_device is not None else device
        d, bs = cfg.head_dim, cfg.block_size
        nlayers = cfg.layers if layers is None else layers
        self.layers = []
        for li in range(nlayers):
            sh = shard_layer(random_layer(cfg, li, seed, gdev, scales), cfg, rank, tp)
            lin = lambda name: _linear(*sh[name], device, mxfp4_kernel)  # noqa: E731
            gate_up = _gate_up_linear(*sh["gate_up"], cfg.inter // tp, device, mxfp4_kernel, fuse_swiglu)
            self.layers.append({
                "qkv": lin("qkv"), "o": lin("o"), "gate_up": gate_up, "down": lin("down"),
                "in_norm": sh["in_norm"].to(device), "post_norm": sh["post_norm"].to(device)})
        head = random_head(cfg, seed, gdev)
        vl = cfg.vocab // tp
        self.embed = head["embed"].to(device)
        self.lm_head = head["lm_head"][rank * vl:(rank + 1) * vl].to(device).contiguous()
        self.final_norm = head["final_norm"].to(device)
        del head
        # paged fp8 KV: sequence b owns blocks [b * maxblk, (b + 1) * maxblk)
        self.maxblk = -(-max_ctx // bs)
        nb = batch * self.maxblk
        self.block_table = torch.arange(nb, dtype=torch.int32, device=device).view(batch, self.maxblk)
        self.kv = []
        for _ in range(nlayers):
            self.kv.append({
                "k": torch.zeros(nb, bs, self.hkv, d, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn),
                "v": torch.zeros(nb, bs, self.hkv, d, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn),
                "ks": torch.full((1,), kv_scale, dtype=torch.float32, device=device),
                "vs": torch.full((1,), kv_scale, dtype=torch.float32, device=device)})
        self.rope = rope_table(max_ctx, d, cfg.rope_theta).to(device)
        self.max_ctx = max_ctx
        # per-step state (device): next input tokens and their positions
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=device)
        self.positions = torch.zeros(batch, dtype=torch.int32, device=device)
        H, nqkv = cfg.hidden, (self.hq + 2 * self.hkv) * d
        z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16, device=device)  # noqa: E731
        self.buf = {"h": z(batch, H), "x": z(batch, H), "qkv": z(batch, nqkv), "attn": z(batch, self.hq, d),
                    "o": z(batch, H), "gu": z(batch, 2 * cfg.inter // tp), "act": z(batch, cfg.inter // tp),
                    "dn": z(batch, H)}
        self.qsl = torch.arange(batch + 1, dtype=torch.int32, device=device)
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=device)
        self.slots = torch.zeros(batch, dtype=torch.int64, device=device)
        self.logits = torch.zeros(batch, vl, dtype=torch.float32, device=device)
        self._top_val = torch.zeros(batch, dtype=torch.float32, device=device)
        self._top_idx = torch.zeros(batch, dtype=torch.int64, device=device)

    # ---- glue kernels ---------------------------------------------------------
    def _rmsnorm(self, delta, w):
        b = self.buf
        check(lib.b200kv_rmsnorm_residual(b["h"].data_ptr(), delta.data_ptr() if delta is not None else None,
                                          w.data_ptr(), b["x"].data_ptr(), self.B, self.cfg.hidden,
                                          float(self.cfg.eps), _stream(b["h"])), "b200kv_rmsnorm_residual")

    def _rope_kv(self, kv):
        b, k, v = self.buf, kv["k"], kv["v"]
        check(lib.b200kv_rope_kv_write(
            b["qkv"].data_ptr(), b["qkv"].stride(0), self.positions.data_ptr(), self.rope.data_ptr(),
            self.max_ctx, self.slots.data_ptr(), k.data_ptr(), v.data_ptr(),
            k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1), v.stride(2),
            kv["ks"].data_ptr(), kv["vs"].data_ptr(), self.B, self.hq, self.hkv, self.cfg.head_dim,
            self.cfg.block_size, KV_FP8_E4M3 if k.dtype == torch.float8_e4m3fn else KV_BF16,
            _stream(b["qkv"])), "b200kv_rope_kv_write")

    def _qkv_rope_kv(self, x, lin, kv):
        """qkv = x @ W^T, RoPE on q and k, k and v into the cache: one launch
        (b200kv_mxfp4_gemm_rope_kv) on tensor-core weights at M <= 8 with an fp8
        cache and head_dim 128, else the product and the glue kernel."""
        b, k, v = self.buf, kv["k"], kv["v"]
        if (self._fuse_rope and lin[0] == "tc" and x.shape[0] <= h4mv.MAX_M and x.is_contiguous()
                and k.dtype == torch.float8_e4m3fn and self.cfg.head_dim == 128):
            W, S = lin[1], lin[2]
            check(lib.b200kv_mxfp4_gemm_rope_kv(
                W.data_ptr(), S.data_ptr(), x.data_ptr(), b["qkv"].data_ptr(), W.shape[0], W.shape[1] * 2,
                x.shape[0], self.positions.data_ptr(), self.rope.data_ptr(), self.max_ctx,
                self.slots.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                v.stride(0), v.stride(1), v.stride(2), kv["ks"].data_ptr(), kv["vs"].data_ptr(), self.hq,
                self.hkv, self.cfg.block_size, KV_FP8_E4M3, _stream(x)), "b200kv_mxfp4_gemm_rope_kv")
            return
        _gemm(x, lin, b["qkv"])
        self._rope_kv(kv)

    def _row_parallel(self, x, lin, out):
        """out = the allreduced row-parallel product x @ W^T (o, down)."""
        if self._fused_ar and lin[0] == "tc" and x.shape[0] <= h4mv.MAX_M:
            return self.allreduce.gemm(x, lin[1], lin[2], out)
        _gemm(x, lin, out)
        self.allreduce(out)
        return out

    # ---- prompt ----------------------------------------------------------------
    def prefill(self, prompts, allreduce=None):
        """Run prompts (device int64 [B, P], every sequence P tokens, P <
        max_ctx) through the model from position 0: per layer the qkv, o,
        gate_up and down products at M = B * P (wide MXFP4 GEMM), RoPE + fp8 KV
        write of every prompt token, and varlen causal prefill attention.
        Writes this rank's logits of each sequence's last prompt token, sets
        tokens to the greedy next token and positions to P, and returns the
        tokens.  allreduce sums the row-parallel partials of all B * P rows
        (default: the decode allreduce)."""
        cfg, d, bs, B = self.cfg, self.cfg.head_dim, self.cfg.block_size, self.B
        P = prompts.shape[1]
        if prompts.shape[0] != B or P >= self.max_ctx:
            raise ValueError(f"prompts must be [{B}, P] with P < {self.max_ctx}")
        T, H, dev = B * P, cfg.hidden, self.dev
        red = allreduce if allreduce is not None else self.allreduce
        pos = torch.arange(P, dtype=torch.int32, device=dev).repeat(B)
        seq = torch.arange(B, device=dev).repeat_interleave(P)
        slots = self.block_table[seq, (pos // bs).long()].long() * bs + (pos % bs).long()
        cu = torch.arange(0, T + 1, P, dtype=torch.int32, device=dev)
        lens = torch.full((B,), P, dtype=torch.int32, device=dev)
        z = lambda *s: torch.empty(*s, dtype=torch.bfloat16, device=dev)  # noqa: E731
        h = torch.index_select(self.embed, 0, prompts.reshape(-1))
        x, o, dn = z(T, H), z(T, H), z(T, H)
        qkv = z(T, (self.hq + 2 * self.hkv) * d)
        attn = z(T, self.hq, d)
        gu, act = z(T, 2 * cfg.inter // self.tp), z(T, cfg.inter // self.tp)
        st = _stream(h)

        def norm(delta, w):
            check(lib.b200kv_rmsnorm_residual(h.data_ptr(), delta.data_ptr() if delta is not None else None,
                                              w.data_ptr(), x.data_ptr(), T, H, float(cfg.eps), st),
                  "b200kv_rmsnorm_residual")
        norm(None, self.layers[0]["in_norm"] if self.layers else self.final_norm)
        for li, lay in enumerate(self.layers):
            kv = self.kv[li]
            k, v = kv["k"], kv["v"]
            _gemm(x, lay["qkv"], qkv)
            check(lib.b200kv_rope_kv_write(
                qkv.data_ptr(), qkv.stride(0), pos.data_ptr(), self.rope.data_ptr(), self.max_ctx,
                slots.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                v.stride(0), v.stride(1), v.stride(2), kv["ks"].data_ptr(), kv["vs"].data_ptr(), T, self.hq,
                self.hkv, d, bs, KV_FP8_E4M3 if k.dtype == torch.float8_e4m3fn else KV_BF16, st),
                "b200kv_rope_kv_write")
            q = qkv[:, :self.hq * d].unflatten(1, (self.hq, d))
            fp8kv_prefill.prefill_attention(q, k, v, attn, cu, lens, self.block_table, kv["ks"], kv["vs"],
                                            d ** -0.5, max_qlen=P)
            _gemm(attn.view(T, self.hq * d), lay["o"], o)
            red(o)
            norm(o, lay["post_norm"])
            _gate_up(x, lay["gate_up"], gu, act, cfg.inter // self.tp, st)
            _gemm(act, lay["down"], dn)
            red(dn)
            norm(dn, self.layers[li + 1]["in_norm"] if li + 1 < len(self.layers) else self.final_norm)
        last = x.view(B, P, H)[:, P - 1].contiguous()
        self.logits.copy_(torch.mm(last, self.lm_head.t(), out_dtype=torch.float32))
        self.tokens.copy_(self._argmax())
        self.positions.fill_(P)
        return self.tokens

    def _argmax(self):
        """Greedy token per sequence from this rank's logits (vocab-parallel
        under tensor parallelism: local (max, index), then a gather)."""
        # at tp 1 the greedy tokens go straight to self.tokens (the next step's input)
        val, idx = self._top_val, (self.tokens if self.tp == 1 else self._top_idx)
        lg = self.logits
        check(lib.b200kv_argmax_rows(lg.data_ptr(), lg.stride(0), lg.shape[0], lg.shape[1], val.data_ptr(),
                                     idx.data_ptr(), _stream(lg)), "b200kv_argmax_rows")
        if self.tp > 1:
            B, vl = self.B, self.cfg.vocab // self.tp
            mine = torch.stack([val, (idx + self.rank * vl).float()], 1)  # exact below 2^24
            allv = torch.empty(self.tp, B, 2, dtype=torch.float32, device=self.dev)
            self.gather(allv, mine)
            best = allv[:, :, 0].argmax(0)  # first maximum = lowest vocab index on ties
            idx = allv[:, :, 1].gather(0, best.unsqueeze(0)).squeeze(0).long()
        return idx

    # ---- one decode step --------------------------------------------------------
    def step(self):
        """Embed self.tokens at self.positions, run the layers, write this
        rank's logits and return the greedy next tokens (device int64 [B]);
        tokens and positions advance in place."""
        cfg, b, B, d, bs = self.cfg, self.buf, self.B, self.cfg.head_dim, self.cfg.block_size
        # sequence lengths, KV slots and the embedding lookup: one launch
        check(lib.b200kv_decode_step_prep(self.positions.data_ptr(), self.tokens.data_ptr(), self.embed.data_ptr(),
                                          cfg.hidden, self.embed.shape[0], self.block_table.data_ptr(),
                                          self.block_table.stride(0), self.block_table.shape[1], bs, B,
                                          self.seq_lens.data_ptr(), self.slots.data_ptr(), b["h"].data_ptr(),
                                          _stream(b["h"])), "b200kv_decode_step_prep")
        self._rmsnorm(None, self.layers[0]["in_norm"] if self.layers else self.final_norm)
        for li, lay in enumerate(self.layers):
            kv = self.kv[li]
            self._qkv_rope_kv(b["x"], lay["qkv"], kv)
            q = b["qkv"][:, :self.hq * d].unflatten(1, (self.hq, d))
            fp8kv_v3.run(q, kv["k"], kv["v"], b["attn"], self.qsl, self.seq_lens, self.block_table,
                         kv["ks"], kv["vs"], d ** -0.5, max_seq_len=self.max_ctx)
            self._row_parallel(b["attn"].view(B, self.hq * d), lay["o"], b["o"])
            self._rmsnorm(b["o"], lay["post_norm"])
            _gate_up(b["x"], lay["gate_up"], b["gu"], b["act"], cfg.inter // self.tp, _stream(b["x"]))
            self._row_parallel(b["act"], lay["down"], b["dn"])
            nxt = self.layers[li + 1]["in_norm"] if li + 1 < len(self.layers) else self.final_norm
            self._rmsnorm(b["dn"], nxt)
        # bf16 lm_head on cuBLAS (a plain library GEMM), fp32 logits
        self.logits.copy_(torch.mm(b["x"], self.lm_head.t(), out_dtype=torch.float32))
        self.tokens.copy_(self._argmax())
        self.positions.add_(1)
        return self.tokens
