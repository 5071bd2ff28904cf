#!/usr/bin/env python
"""Hot-path benchmark on B200: one 7B-class decode step's attention + MXFP4
linears (BASELINE metric "decode-attn & MXFP4 GEMV HBM GB/s; 7B decode tok/s
at bs 1/4/8, 1-8 GPU").

A step = 32 layers x [ qkv GEMV (M=B) -> paged fp8 decode attention over
B sequences of 4096 tokens (q read straight out of the qkv output) -> o_proj
GEMV -> gate_up GEMV ; down GEMV (M=B, K=14336) ], every layer with its own
weights and KV pool (3.9 GB at B=1, far above the 126 MB L2, so no flush is
needed between steps).  value = algorithmic HBM bytes of the step / device time.
The same line carries the step's parts at B = 1, 4 and 8, the 7B decoder's
tok/s at B = 1, 4 and 8 (config 4), config 2 at M = 64, config 3 (prefill)
and config 5 (serving), each with its CPU baseline where the metric has one.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]

N > 1 runs under torchrun with tensor parallelism over the N GPUs (attention
by kv head, qkv/gate_up column-parallel, o/down row-parallel + allreduce;
--parallel replicas runs N independent copies instead); the reported time is
the max over ranks.  `--impl reference` times the reference's own CPU path
for this work (the PyTorch dequant + attention / dequant + matmul checker
restated in oracle/) on the host's cores, on a bounded sample (one layer per
step).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gfx1201-tuning-log_b200")
ORACLE = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

import torch  # noqa: E402

METRIC = "decode-attn & MXFP4 GEMV HBM GB/s; 7B decode tok/s at bs 1/4/8, 1–8 GPU"
SHAPES = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336))
HQ, HKV, D, PBLK = 32, 8, 128, 16


def gemv_bytes(N, K, M):
    """Algorithmic bytes of one MXFP4 matvec: W + scales + x + out."""
    return N * K // 2 + N * K // 32 + 2 * M * K + 2 * M * N


def decode_bytes(B, ctx, tp=1):
    """Algorithmic bytes of one decode-attention call (one rank's kv heads under
    tensor parallelism): fp8 K+V, q, out, block table, lens."""
    return B * (2 * ctx * (HKV // tp) * D + (HQ // tp) * D * 2 * 2 + (ctx // PBLK) * 4 + 8)


def layer_bytes(B, ctx):
    return sum(gemv_bytes(N, K, B) for _, N, K in SHAPES) + decode_bytes(B, ctx)


def rank_shapes(tp):
    """(name, N, K) of one rank's MXFP4 linears under tensor parallelism over tp
    ranks: qkv and gate_up column-parallel (N / tp), o and down row-parallel
    (K / tp, followed by an allreduce of the [B, 4096] partials)."""
    return tuple((name, N // tp if name in ("qkv", "gate_up") else N,
                  K if name in ("qkv", "gate_up") else K // tp) for name, N, K in SHAPES)


def workload_config(args):
    return {"workload": f"7B decode-step hot path: {args.layers} layers x [MXFP4 GEMV "
                        f"qkv/o/gate_up/down at M={args.batch} + fp8 paged decode attention "
                        f"{args.batch} seq x {args.ctx} ctx, GQA 32/8, D 128, block 16]",
            "batch": args.batch, "ctx": args.ctx, "layers": args.layers,
            "mxfp4_kernel": ("block-scaled tcgen05 (kind::mxf8f6f4: e2m1 weights, x as two exact e4m3 "
                             "terms), scales packed at load" if args.gemv == "tc" else "CUDA-core mma.sync"),
            "l2": "inputs larger than L2 (distinct weights/KV per layer), no flush",
            "parallelism": (f"tp{args.tp}: attention by kv head, qkv/gate_up column-parallel, "
                            + ("o/down row-parallel with the allreduce in their epilogue (peer memory)"
                               if args.allreduce == "fused" else
                               f"o/down row-parallel + {args.allreduce} allreduce (in the CUDA graph)")
                            if args.tp > 1 else f"replicas x{args.gpus}")}


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
            return
        t0 = time.time()  # the timed region starts once the sampler answers
        while not self.lines and self.proc.poll() is None and time.time() - t0 < 10:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
def build_weights(args, dev):
    """Random-init MXFP4 weights of `layers` layers (this rank's shards), scales
    packed at load; shared by every batch size."""
    tp = args.tp
    g = torch.Generator(device=dev).manual_seed(1234 + args.rank)
    weights = []
    for _ in range(args.layers):
        lay = {}
        for name, N, K in rank_shapes(tp):
            W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g)
            St = torch.randint(119, 126, (N, K // 32), dtype=torch.uint8, device=dev, generator=g)
            if args.gemv == "tc":  # load-time repack of the scales into tensor-core atoms
                import h4mv
                packed, edge = h4mv.pack_scales(St, N, K)
                assert not edge
                lay[name] = (W, packed)
            else:
                lay[name] = (W, St)
        weights.append(lay)
    return weights


def build_model(args, dev, weights, B):
    """Per-layer fp8 KV pools for B sequences of args.ctx tokens (random
    permuted block tables, per-tensor amax/448 scales), the layers' inputs, and
    the step's output buffers.  Returns (layers, bufs); layers[i] holds the
    weights of layer i too."""
    ctx, tp = args.ctx, args.tp
    hkv = HKV // tp  # this rank's kv heads
    g = torch.Generator(device=dev).manual_seed(4321 + 17 * B + args.rank)
    layers = []
    nblk = ctx // PBLK
    for w in weights:
        lay = dict(w)
        nb = B * nblk
        kf = torch.randn(nb, PBLK, hkv, D, device=dev, generator=g)
        ks = kf.abs().max() / 448.0
        lay["k"] = (kf / ks).to(torch.float8_e4m3fn)
        del kf
        vf = torch.randn(nb, PBLK, hkv, D, device=dev, generator=g)
        vs = vf.abs().max() / 448.0
        lay["v"] = (vf / vs).to(torch.float8_e4m3fn)
        del vf
        lay["ks"] = ks.reshape(1).float()
        lay["vs"] = vs.reshape(1).float()
        lay["bt"] = torch.randperm(nb, device=dev, generator=g).to(torch.int32).view(B, nblk)
        lay["x"] = torch.randn(B, 4096, device=dev, generator=g).to(torch.bfloat16)
        lay["act"] = torch.randn(B, 14336 // tp, device=dev, generator=g).to(torch.bfloat16)
        layers.append(lay)
    bufs = {
        "B": B,
        "qkv": torch.empty(B, 6144 // tp, dtype=torch.bfloat16, device=dev),
        "attn": torch.empty(B, HQ // tp, D, dtype=torch.bfloat16, device=dev),
        "o": torch.empty(B, 4096, dtype=torch.bfloat16, device=dev),
        "gate_up": torch.empty(B, 28672 // tp, dtype=torch.bfloat16, device=dev),
        "down": torch.empty(B, 4096, dtype=torch.bfloat16, device=dev),
        "qsl": torch.arange(B + 1, dtype=torch.int32, device=dev),
        "slens": torch.full((B,), ctx, dtype=torch.int32, device=dev),
    }
    return layers, bufs


def run_step(layers, bufs, args, which=("gemv", "attn", "comm")):
    """One hot-path step through the public API (h4mv.mxfp4_gemm or
    h4mv.mxfp4_gemv, fp8kv_v3.run); under tensor parallelism the o and down
    partials are summed over the ranks (tp.allreduce_)."""
    import fp8kv_v3
    import h4mv
    import tp
    B = bufs["B"]
    hq = HQ // args.tp
    sm = D ** -0.5
    gemv = h4mv.mxfp4_gemm if args.gemv == "tc" else h4mv.mxfp4_gemv
    do_g, do_a, do_c = "gemv" in which, "attn" in which, "comm" in which and args.tp > 1
    # o and down with the allreduce in their epilogue: the GEMV part carries it
    fused = args.tp > 1 and args.allreduce == "fused"
    if fused:
        do_c = False

    def row_parallel(x, lin, out):
        if fused:
            args.allreduce_fn.gemm(x, *lin, out=out)
        else:
            gemv(x, *lin, out=out)
    for lay in layers:
        if do_g:
            gemv(lay["x"], *lay["qkv"], out=bufs["qkv"])
        if do_a:
            q = bufs["qkv"][:, :hq * D].unflatten(1, (hq, D))
            fp8kv_v3.run(q, lay["k"], lay["v"], bufs["attn"], bufs["qsl"], bufs["slens"], lay["bt"],
                         lay["ks"], lay["vs"], sm, max_seq_len=args.ctx)
        if do_g:
            row_parallel(bufs["attn"].view(B, hq * D), lay["o"], bufs["o"])
        if do_c:
            args.allreduce_fn(bufs["o"])
        if do_g:
            gemv(bufs["o"], *lay["gate_up"], out=bufs["gate_up"])
            row_parallel(lay["act"], lay["down"], bufs["down"])
        if do_c:
            args.allreduce_fn(bufs["down"])


def capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


def time_graph(graph, steps, warmup, barrier=None):
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    return e0.elapsed_time(e1) / steps


PREFILL_LENS = (512, 1024, 1536, 2048)


def prefill_flops(lens, hq=HQ, d=D):
    """Causal attention FLOPs: 4 * D * HQ * sum L(L+1)/2 (QK^T and PV)."""
    return 4 * d * hq * sum(L * (L + 1) // 2 for L in lens)


def prefill_part(dev, steps, warmup, barrier=None):
    """Config 3: four sequences {512, 1024, 1536, 2048} packed with cu_seqlens,
    bf16 K/V ~ N(0,1) written into a paged fp8 pool (block 16, random block
    permutation, per-tensor amax/448 scales) by the KV-write kernel, then one
    varlen causal prefill call.  Returns (us per call, FLOPs per call)."""
    import fp8kv_prefill
    import kv_cache
    lens = PREFILL_LENS
    T = sum(lens)
    g = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn(T, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    key = torch.randn(T, HKV, D, device=dev, generator=g).to(torch.bfloat16)
    val = torch.randn(T, HKV, D, device=dev, generator=g).to(torch.bfloat16)
    nblk = [L // PBLK for L in lens]
    nb = sum(nblk)
    perm = torch.randperm(nb, device=dev, generator=g).to(torch.int32)
    bt = torch.zeros(len(lens), max(nblk), dtype=torch.int32, device=dev)
    slots, pos = [], 0
    for s, L in enumerate(lens):
        bt[s, :nblk[s]] = perm[pos:pos + nblk[s]]
        pos += nblk[s]
        t = torch.arange(L, device=dev)
        slots.append(bt[s, t // PBLK].long() * PBLK + t % PBLK)
    slots = torch.cat(slots)
    ks = (key.float().abs().max() / 448.0).reshape(1)
    vs = (val.float().abs().max() / 448.0).reshape(1)
    kc = torch.zeros(nb, PBLK, HKV, D, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    kv_cache.reshape_and_cache_flash(key, val, kc, vc, slots, "fp8", ks, vs)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=dev)
    seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    out = torch.empty(T, HQ, D, dtype=torch.bfloat16, device=dev)
    reps = 10

    def call():
        for _ in range(reps):
            fp8kv_prefill.prefill_attention(q, kc, vc, out, cu, seq_lens, bt, ks, vs, D ** -0.5,
                                            max_qlen=max(lens))
    graph = capture(call)
    ms = time_graph(graph, max(steps // 2, 3), warmup, barrier) / reps
    del graph
    return ms * 1e3, prefill_flops(lens)


WIDE_M = 64


def wide_gemm_part(dev, steps, warmup, barrier=None, tp=1, layers=3):
    """Config 2 at M = WIDE_M: this rank's four 7B MXFP4 projections (config-2
    weights: codes uniform, scales 2^-8..2^-2, packed once) on the wide-batch
    tensor-core GEMM, `layers` distinct weight sets cycled so the weights stream
    from HBM (3 layers = 327 MB at tp 1 against the 126 MB L2).  Returns (us per
    layer of four GEMMs, algorithmic bytes per layer, FLOPs per layer)."""
    import h4mv
    shapes = rank_shapes(tp)
    g = torch.Generator(device=dev).manual_seed(5)
    sets = []
    for _ in range(layers):
        for _, N, K in shapes:
            W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g)
            S = torch.randint(119, 126, (K // 32, N), dtype=torch.uint8, device=dev, generator=g)
            P, _ = h4mv.pack_scales(S, N, K, h4mv.SCALES_CHECKPOINT)
            x = torch.randn(WIDE_M, K, device=dev, generator=g).to(torch.bfloat16)
            sets.append((x, W, P, torch.empty(WIDE_M, N, dtype=torch.bfloat16, device=dev)))

    def call():
        for x, W, P, out in sets:
            h4mv.mxfp4_gemm_wide(x, W, P, out=out)
    graph = capture(call)
    ms = time_graph(graph, max(steps // 2, 3), warmup, barrier) / layers
    del graph
    nbytes = sum(gemv_bytes(N, K, WIDE_M) for _, N, K in shapes)
    flops = sum(2 * WIDE_M * N * K for _, N, K in shapes)
    return ms * 1e3, nbytes, flops


SERVE_DECODES, SERVE_PREFILLS, SERVE_PREFILL_LEN, SERVE_CTX = 60, 4, 2048, (2048, 32768)


def serving_part(args, dev, barrier, layers=32, steps=2):
    """Config 5, the serving shape on the 7B model: 64 sequences per step, 60
    decoding (contexts ~U[2k, 32k], seeded) and 4 new 2048-token prefills, over
    one fp8 paged pool per layer with a fragmented random block table (every
    sequence's pages drawn from one random permutation).  A step is `layers` x
    [qkv GEMM (M = 8252 tokens) -> KV write of the 8252 new tokens ->
    attention -> o GEMM -> gate_up GEMM -> down GEMM] on this rank's shards
    (tensor parallel: kv-head attention, NCCL allreduce of the o and down
    outputs); the pages already in the pool are synthetic fp8, the prompt KV a
    real engine would have written.  Attention runs two ways: "mixed", one
    varlen call for the whole batch (decode tokens as one-token prefills, what
    the vLLM forward patch does), and "split", the decode kernel for the 60
    decode rows plus the varlen kernel for the 4 prefills.  Eager launches,
    CUDA events, max over ranks.  Returns a dict for the bench line."""
    import _decode
    import fp8kv_prefill
    import h4mv
    import kv_cache
    tp = args.tp
    hq, hkv, inter = HQ // tp, HKV // tp, 14336 // tp
    gc = torch.Generator().manual_seed(21)
    ctx = torch.randint(SERVE_CTX[0], SERVE_CTX[1] + 1, (SERVE_DECODES,), generator=gc).tolist()
    seq = [c + 1 for c in ctx] + [SERVE_PREFILL_LEN] * SERVE_PREFILLS
    qlens = [1] * SERVE_DECODES + [SERVE_PREFILL_LEN] * SERVE_PREFILLS
    T, NS = sum(qlens), len(seq)
    nblk = [-(-L // PBLK) for L in seq]
    NB = sum(nblk)
    perm = torch.randperm(NB, generator=gc).to(torch.int32)
    bt = torch.zeros(NS, max(nblk), dtype=torch.int32)
    slots, pos = [], 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
        first = seq[i] - qlens[i]  # position of the step's first new token
        t = torch.arange(first, seq[i])
        slots.append(bt[i, t // PBLK].long() * PBLK + t % PBLK)
    slots = torch.cat(slots).to(dev)
    bt = bt.to(dev)
    seq_lens = torch.tensor(seq, dtype=torch.int32, device=dev)
    cu = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    qsl_dec = torch.arange(SERVE_DECODES + 1, dtype=torch.int32, device=dev)
    cu_pre = (cu[SERVE_DECODES:] - SERVE_DECODES).contiguous()
    ks = torch.full((1,), 1 / 16, device=dev)
    g = torch.Generator(device=dev).manual_seed(22)
    lays = []
    for _ in range(layers):
        lay = {}
        for name, N, K in rank_shapes(tp):
            W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g)
            S = torch.randint(119, 126, (K // 32, N), dtype=torch.uint8, device=dev, generator=g)
            lay[name] = (W, h4mv.pack_scales(S, N, K, h4mv.SCALES_CHECKPOINT)[0])
        for name in ("k", "v"):  # synthetic prompt KV (codes 0..125: finite, up to 416/16)
            pool = torch.empty(NB, PBLK, hkv, D, dtype=torch.uint8, device=dev)
            lay[name] = pool.random_(0, 126, generator=g).view(torch.float8_e4m3fn)
        lays.append(lay)
    x = torch.randn(T, 4096, device=dev, generator=g).to(torch.bfloat16)
    qkv = torch.empty(T, (hq + 2 * hkv) * D, dtype=torch.bfloat16, device=dev)
    attn = torch.empty(T, hq, D, dtype=torch.bfloat16, device=dev)
    o = torch.empty(T, 4096, dtype=torch.bfloat16, device=dev)
    act = torch.empty(T, inter, dtype=torch.bfloat16, device=dev)
    dn = torch.empty(T, 4096, dtype=torch.bfloat16, device=dev)
    q = qkv[:, :hq * D].view(T, hq, D)
    kn = qkv[:, hq * D:(hq + hkv) * D].view(T, hkv, D)
    vn = qkv[:, (hq + hkv) * D:].view(T, hkv, D)
    sm = D ** -0.5
    allreduce = None
    if tp > 1:
        import torch.distributed as dist
        allreduce = dist.all_reduce

    def attention(L, mode):
        if mode == "mixed":  # the forward patch's path: split on the device by query count
            fp8kv_prefill.mixed_attention(q, L["k"], L["v"], attn, cu, seq_lens, bt, ks, ks, sm,
                                          max_qlen=SERVE_PREFILL_LEN, max_seq_len=SERVE_CTX[1] + 1)
        elif mode == "one_call":
            fp8kv_prefill.prefill_attention(q, L["k"], L["v"], attn, cu, seq_lens, bt, ks, ks, sm,
                                            max_qlen=SERVE_PREFILL_LEN)
        else:
            _decode.decode_attention(q, L["k"], L["v"], attn, qsl_dec, seq_lens[:SERVE_DECODES],
                                     bt[:SERVE_DECODES], ks, ks, sm, out_by_qsl=True,
                                     max_seq_len_hint=SERVE_CTX[1] + 1)
            fp8kv_prefill.prefill_attention(q[SERVE_DECODES:], L["k"], L["v"], attn[SERVE_DECODES:], cu_pre,
                                            seq_lens[SERVE_DECODES:], bt[SERVE_DECODES:], ks, ks, sm,
                                            max_qlen=SERVE_PREFILL_LEN)

    def step(mode, part="all"):
        for L in lays:
            if part in ("all", "gemm"):
                h4mv.mxfp4_gemm_wide(x, *L["qkv"], out=qkv)
            if part in ("all", "attn"):
                kv_cache.reshape_and_cache_flash(kn, vn, L["k"], L["v"], slots, "fp8", ks, ks)
                attention(L, mode)
            if part in ("all", "gemm"):
                h4mv.mxfp4_gemm_wide(attn.view(T, hq * D), *L["o"], out=o)
                if allreduce:
                    allreduce(o)
                h4mv.mxfp4_gemm_swiglu(o, *L["gate_up"], out=act)  # gate_up with the SwiGLU epilogue
                h4mv.mxfp4_gemm_wide(act, *L["down"], out=dn)
                if allreduce:
                    allreduce(dn)

    def timed(mode, part):
        step(mode, part)
        torch.cuda.synchronize()
        if barrier:
            barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step(mode, part)
        e1.record()
        torch.cuda.synchronize()
        if barrier:
            barrier()
        return e0.elapsed_time(e1) / steps

    res = {"mixed": timed("mixed", "all"), "split": timed("split", "all"),
           "attn_mixed": timed("mixed", "attn"), "attn_split": timed("split", "attn"),
           "attn_one_call": timed("one_call", "attn"),
           "gemm": timed("split", "gemm")}
    kv_bytes = layers * sum(c + 1 for c in ctx) * hkv * D * 2
    pre_flops = layers * 4 * D * hq * SERVE_PREFILLS * SERVE_PREFILL_LEN * (SERVE_PREFILL_LEN + 1) // 2
    gemm_flops = layers * sum(2 * T * N * K for _, N, K in rank_shapes(tp))
    del lays
    torch.cuda.empty_cache()
    return res, T, kv_bytes, pre_flops, gemm_flops


DECODE_PROMPT, DECODE_TOKENS = 4096, 256


def decode_7b_part(args, dev, barrier, allreduce, B):
    """Config 4: the full 7B MXFP4 decoder (decoder.py): a DECODE_PROMPT-token
    random-id prompt per sequence through MXFP4Decoder.prefill (wide MXFP4
    GEMMs, RoPE + fp8 KV write, varlen causal prefill attention; eager, timed:
    the time to the first token), then greedy decode steps at batch B reading
    the cache the prefill wrote, one CUDA-graph replay per token.  Returns
    (ms per token step, tokens/s, ms of the prefill)."""
    import decoder
    cfg = decoder.SEVEN_B
    gather = None
    big_allreduce = None
    if args.tp > 1:
        import torch.distributed as dist

        def gather(out, inp):
            dist.all_gather_into_tensor(out.view(-1), inp.contiguous().view(-1))

        def big_allreduce(t):  # the prompt's [B x 4096, 4096] partials: NCCL
            dist.all_reduce(t)
    dec = decoder.MXFP4Decoder(cfg, dev, B, DECODE_PROMPT + DECODE_TOKENS + 16, seed=7, tp=args.tp,
                               rank=args.rank, allreduce=allreduce, gather=gather,
                               fuse_allreduce=args.allreduce == "fused")
    g = torch.Generator(device=dev).manual_seed(11)  # the same prompts on every rank
    prompts = torch.randint(0, cfg.vocab, (B, DECODE_PROMPT), device=dev, generator=g)
    dec.prefill(prompts[:, :64].contiguous(), allreduce=big_allreduce)  # warm-up (kernels, workspaces)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    dec.prefill(prompts, allreduce=big_allreduce)
    e1.record()
    torch.cuda.synchronize()
    ms_prefill = e0.elapsed_time(e1)
    dec.step()
    dec.step()
    graph = capture(dec.step)
    steps = min(DECODE_TOKENS - 3, args.steps)
    ms = time_graph(graph, steps, 1, barrier)
    del graph, dec
    torch.cuda.empty_cache()
    return ms, B / (ms * 1e-3), ms_prefill


BATCH_SWEEP = (1, 4, 8)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


TRAFFIC_PROFILE = os.path.join(ROOT, "profiles", "mxfp4_mma_7b_m1.md")


def profile_traffic():
    """Average DRAM bytes per launch of the four 7B shapes at M = 1 from the
    `dram_bytes_per_launch:` line of the committed ncu summary (None when the
    summary has no such line)."""
    try:
        with open(TRAFFIC_PROFILE) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    vals = [float(t.split("=")[1]) for t in line.split(":", 1)[1].split()]
                    return sum(vals) / len(vals), f"{os.path.relpath(TRAFFIC_PROFILE, ROOT)} (ncu, four shapes)"
    except (OSError, ValueError, IndexError):
        pass
    return None, None


def max_over_ranks(x, dist_on, dev):
    if not dist_on:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


# ---------------------------------------------------------------------------
def cpu_layer_sample(args, seed=0):
    """One layer of the hot path on the host through the oracle (reference
    PyTorch path).  Returns (seconds, bytes)."""
    sys.path.insert(0, ORACLE)
    import fp8kv_oracle as FO
    import mxfp4_oracle as MO
    torch.set_num_threads(os.cpu_count())
    B = args.batch
    cases = [MO.make_case(N, K, B, seed=seed + i) for i, (_, N, K) in enumerate(SHAPES)]
    dc = FO.make_decode_case(B, [args.ctx] * B, seed=seed)
    t0 = time.perf_counter()
    for W, S, St, X in cases:
        MO.mxfp4_linear_reference(W, S, X)
    FO.decode_reference(dc["q"], dc["k_cache"], dc["v_cache"], dc["qsl"], dc["seq_lens"],
                        dc["block_table"], dc["k_scale"], dc["v_scale"], dc["sm_scale"])
    return time.perf_counter() - t0, layer_bytes(B, args.ctx)


def cpu_prefill_baseline():
    """Config 3 on the host: the oracle's causal prefill (prefill_test.py:23-38,
    per sequence) on the 512- and 1024-token sequences of config 3 (a bounded
    sample), scaled to the whole call by FLOPs.  Returns the cpu_baseline dict."""
    sys.path.insert(0, ORACLE)
    import fp8kv_oracle as FO
    torch.set_num_threads(os.cpu_count())
    lens = PREFILL_LENS[:2]
    g = torch.Generator().manual_seed(3)
    T = sum(lens)
    nblk = [L // PBLK for L in lens]
    nb = sum(nblk)
    q = torch.randn(T, HQ, D, generator=g).to(torch.bfloat16)
    kc = (torch.randn(nb, PBLK, HKV, D, generator=g) * 8).to(torch.float8_e4m3fn)
    vc = (torch.randn(nb, PBLK, HKV, D, generator=g) * 8).to(torch.float8_e4m3fn)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(len(lens), max(nblk), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32)
    t0 = time.perf_counter()
    FO.prefill_reference(q, kc, vc, cu, sl, bt, 1 / 16, 1 / 16, D ** -0.5)
    t = time.perf_counter() - t0
    tflops = prefill_flops(lens) / t / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "us_per_call_extrapolated": prefill_flops(PREFILL_LENS) / (tflops * 1e12) * 1e6,
            "sample": f"oracle causal prefill of the {list(lens)}-token sequences of config 3 "
                      f"({prefill_flops(lens) / 1e9:.1f} GFLOP, {t:.2f} s), scaled to the call by FLOPs"}


_CPU_CACHE = {}


def cpu_decoder_baseline(B):
    """Config 4 on the host: one oracle decoder step (oracle/decoder_oracle.py,
    HF Llama semantics) of a 2-layer model of the 7B widths at batch B over
    4096-token fp8 caches, and its final norm + 128256-row lm_head alone; a
    32-layer step is extrapolated from the per-layer time.  Returns the
    cpu_baseline dict (tok/s)."""
    sys.path.insert(0, ORACLE)
    import dataclasses

    import decoder
    import decoder_oracle as DO
    torch.set_num_threads(os.cpu_count())
    cfg = decoder.SEVEN_B
    ctx = DECODE_PROMPT
    table = DO.rope_table(ctx + 8, cfg.head_dim, cfg.rope_theta)
    if "head" not in _CPU_CACHE:  # 2 x 0.5 G bf16 values, drawn once
        _CPU_CACHE["head"] = decoder.random_head(cfg, 7)
    head = _CPU_CACHE["head"]
    if "layers" not in _CPU_CACHE:
        _CPU_CACHE["layers"] = []
        for li in range(2):
            lay = decoder.random_layer(cfg, li, 7)
            _CPU_CACHE["layers"].append({k: ((v[0], v[1].t().contiguous()) if isinstance(v, tuple) else v)
                                         for k, v in lay.items()})
    nblk = -(-(ctx + 1) // cfg.block_size)
    g = torch.Generator().manual_seed(5)
    caches = []
    for _ in range(2):
        k = (torch.randn(B * nblk, cfg.block_size, cfg.kv_heads, cfg.head_dim, generator=g) * 4)
        v = (torch.randn(B * nblk, cfg.block_size, cfg.kv_heads, cfg.head_dim, generator=g) * 4)
        caches.append({"k": k.to(torch.float8_e4m3fn), "v": v.to(torch.float8_e4m3fn), "ks": 0.05, "vs": 0.05})
    bt = torch.arange(B * nblk, dtype=torch.int32).view(B, nblk)
    tokens = torch.randint(0, cfg.vocab, (B,), generator=g)
    positions = torch.full((B,), ctx, dtype=torch.int32)
    w = {"embed": head["embed"], "lm_head": head["lm_head"], "final_norm": head["final_norm"],
         "layers": _CPU_CACHE["layers"]}
    t2 = t_head = 1e30
    for _ in range(2):  # the first call pays first-touch costs
        t0 = time.perf_counter()
        DO.decode_step(dataclasses.replace(cfg, layers=2), w, caches, tokens, positions, bt, table)
        t2 = min(t2, time.perf_counter() - t0)
        t0 = time.perf_counter()
        x = DO.rmsnorm(head["embed"][tokens.long()], head["final_norm"], cfg.eps)
        x.float() @ head["lm_head"].float().t()
        t_head = min(t_head, time.perf_counter() - t0)
    per_layer = max((t2 - t_head) / 2, 1e-9)
    step = cfg.layers * per_layer + t_head
    return {"value": B / step, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle decoder step at batch {B} of a 2-layer model of the 7B widths ({t2:.2f} s) "
                      f"and its final norm + lm_head alone ({t_head:.2f} s), extrapolated to {cfg.layers} "
                      f"layers: {step:.1f} s per token step"}


def cpu_serving_baseline():
    """Config 5 on the host, subsampled: one layer of the oracle at 7B widths
    for 64 of the step's 8252 tokens through the four MXFP4 projections, the
    decode attention of 4 of its 60 sequences (contexts drawn as config 5
    draws them) and the causal prefill of one 2048-token sequence; the 32-layer
    step is extrapolated linearly (tokens for the projections, sequences for
    attention).  Returns the cpu_baseline dict (tok/s)."""
    sys.path.insert(0, ORACLE)
    import fp8kv_oracle as FO
    import mxfp4_oracle as MO
    torch.set_num_threads(os.cpu_count())
    T = SERVE_DECODES + SERVE_PREFILLS * SERVE_PREFILL_LEN
    tok = 64
    gc = torch.Generator().manual_seed(21)
    ctx = torch.randint(SERVE_CTX[0], SERVE_CTX[1] + 1, (SERVE_DECODES,), generator=gc).tolist()
    t0 = time.perf_counter()
    for i, (_, N, K) in enumerate(SHAPES):
        W, S, St, X = MO.make_case(N, K, tok, seed=i)
        MO.mxfp4_linear_reference(W, S, X)
    t_gemm = time.perf_counter() - t0
    dc = FO.make_decode_case(4, [c + 1 for c in ctx[:4]], seed=2)
    t0 = time.perf_counter()
    FO.decode_reference(dc["q"], dc["k_cache"], dc["v_cache"], dc["qsl"], dc["seq_lens"], dc["block_table"],
                        dc["k_scale"], dc["v_scale"], dc["sm_scale"])
    t_dec = time.perf_counter() - t0
    L = SERVE_PREFILL_LEN
    nb = L // PBLK
    g = torch.Generator().manual_seed(3)
    q = torch.randn(L, HQ, D, generator=g).to(torch.bfloat16)
    kc = (torch.randn(nb, PBLK, HKV, D, generator=g) * 8).to(torch.float8_e4m3fn)
    t0 = time.perf_counter()
    FO.prefill_reference(q, kc, kc, torch.tensor([0, L], dtype=torch.int32), torch.tensor([L], dtype=torch.int32),
                         torch.arange(nb, dtype=torch.int32).view(1, nb), 1 / 16, 1 / 16, D ** -0.5)
    t_pre = time.perf_counter() - t0
    step = 32 * (t_gemm * T / tok + t_dec * SERVE_DECODES / 4 + t_pre * SERVE_PREFILLS)
    return {"value": T / step, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"1 layer: projections for {tok} of {T} tokens ({t_gemm:.2f} s), decode attention of 4 "
                      f"of {SERVE_DECODES} sequences ({t_dec:.2f} s), one {L}-token prefill ({t_pre:.2f} s); "
                      f"extrapolated to 32 layers x the whole batch: {step:.0f} s per step"}


def cpu_baseline(args, reps=3):
    cpu_layer_sample(args, seed=99)  # warm
    times = []
    for r in range(reps):
        t, nbytes = cpu_layer_sample(args, seed=r)
        times.append(t)
    t = statistics.median(times)
    return {"value": nbytes / t / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"1 of {args.layers} layers (4 MXFP4 GEMVs at M={args.batch} + decode attention "
                      f"{args.batch}x{args.ctx}), torch fp32 oracle, median of {reps}, "
                      f"{t * 1e3:.0f} ms/layer"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_layer_sample(args, seed=1000)
    times, nbytes = [], 0
    for i in range(args.steps):
        t, nbytes = cpu_layer_sample(args, seed=i)
        times.append(t)
    t = sum(times) / len(times)
    val = nbytes / t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "e2m1/e4m3 operands, f32 accumulate", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": "each step = 1 layer of the hot path through the torch fp32 "
                                       "oracle (reference PyTorch dequant+attention / dequant+matmul)"},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def run_mxfp4_m1(args):
    """The four 7B MXFP4 projections at M = 1 through h4mv.mxfp4_gemm, --warmup
    then --steps rounds of four launches (each on its own weights): the case the
    committed ncu summary of the dominant kernel captures."""
    import h4mv
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234)
    cases = []
    for _, N, K in SHAPES:
        W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g)
        St = torch.randint(119, 126, (N, K // 32), dtype=torch.uint8, device=dev, generator=g)
        P, _ = h4mv.pack_scales(St, N, K)
        x = torch.randn(1, K, device=dev, generator=g).to(torch.bfloat16)
        cases.append((x, W, P, torch.empty(1, N, dtype=torch.bfloat16, device=dev)))
    for _ in range(args.warmup + args.steps):
        for x, W, P, out in cases:
            h4mv.mxfp4_gemm(x, W, P, out=out)
    torch.cuda.synchronize()
    print(json.dumps({"part": "mxfp4_m1", "launches": 4 * (args.warmup + args.steps)}))


def run_decode_attn(args):
    """Decode attention alone, 32 layers' pools at --batch sequences of --ctx
    tokens with --kv-heads kv heads (8: one GPU; 1, 2, 4: the tensor-parallel
    shards of the 7B model on one GPU): --warmup then --steps graph replays of
    the 32 launches, timed with CUDA events (the case the committed ncu
    summaries of decode_tma_kernel capture)."""
    import fp8kv_v3
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, hkv = args.batch, args.kv_heads
    hq = hkv * (HQ // HKV)
    g = torch.Generator(device=dev).manual_seed(4321 + B)
    nblk = args.ctx // PBLK
    lays = []
    for _ in range(args.layers):
        nb = B * nblk
        kv = [(4 * torch.randn(nb, PBLK, hkv, D, device=dev, generator=g)).to(torch.float8_e4m3fn)
              for _ in range(2)]
        bt = torch.randperm(nb, device=dev, generator=g).to(torch.int32).view(B, nblk)
        lays.append((kv[0], kv[1], bt))
    q = torch.randn(B, hq, D, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(B, hq, D, dtype=torch.bfloat16, device=dev)
    qsl = torch.arange(B + 1, dtype=torch.int32, device=dev)
    slens = torch.full((B,), args.ctx, dtype=torch.int32, device=dev)
    sc = torch.full((1,), 1 / 16, device=dev)

    def run():
        for k, v, bt in lays:
            fp8kv_v3.run(q, k, v, out, qsl, slens, bt, sc, sc, D ** -0.5, max_seq_len=args.ctx)
    graph = capture(run)
    ms = time_graph(graph, args.steps, args.warmup)
    byts = args.layers * B * (2 * args.ctx * hkv * D + 2 * hq * D * 2)
    print(json.dumps({"part": "decode_attn", "batch": B, "kv_heads": hkv, "ctx": args.ctx,
                      "us_per_call": ms * 1e3 / args.layers, "gbs": byts / (ms * 1e-3) / 1e9}))


def run_decode_7b(args):
    """The 7B decoder's token step alone (decoder.py, one GPU, --batch
    sequences at position --ctx of an fp8 cache; no prompt pass): --warmup
    then --steps graph replays, for an ncu launch list of the step."""
    import decoder
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dec = decoder.MXFP4Decoder(decoder.SEVEN_B, dev, args.batch, args.ctx + args.steps + args.warmup + 8, seed=7)
    dec.positions.fill_(args.ctx)
    dec.step()
    dec.step()
    graph = capture(dec.step)
    ms = time_graph(graph, args.steps, args.warmup)
    print(json.dumps({"part": "decode_7b", "batch": args.batch, "ctx": args.ctx, "ms_per_token_step": ms,
                      "tok_s": args.batch / (ms * 1e-3)}))


def run_prefill(args):
    """Config 3 alone (prefill_part: four sequences of 512-2048 tokens, one
    varlen causal call per replay), for an ncu capture of prefill_fp8_kernel."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    us, flops = prefill_part(dev, args.steps, args.warmup)
    print(json.dumps({"part": "prefill", "us_per_call": us, "tflops": flops / (us * 1e-6) / 1e12}))


def run_b200(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    args.rank = rank
    dist_on = world > 1
    args.tp = world if dist_on and args.parallel == "tp" else 1
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    barrier = None
    if dist_on:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        barrier = dist.barrier

    weights = build_weights(args, dev)
    layers, bufs = build_model(args, dev, weights, args.batch)
    comm = None
    if args.tp > 1:
        import tp
        if args.allreduce in ("peer", "fused"):
            comm = tp.PeerAllreduce()
            args.allreduce_fn = comm
        else:
            args.allreduce_fn = tp.allreduce_
    # the model's algorithmic bytes per step (one GPU's worth under tp: the
    # shards partition it; replicas each stream a full copy)
    step_bytes = args.layers * layer_bytes(args.batch, args.ctx)
    launches_per_step = args.layers * 5

    g_step = capture(lambda: run_step(layers, bufs, args))
    g_gemv = capture(lambda: run_step(layers, bufs, args, which=("gemv",)))
    g_attn = capture(lambda: run_step(layers, bufs, args, which=("attn",)))
    g_comm = (capture(lambda: run_step(layers, bufs, args, which=("comm",)))
              if args.tp > 1 and args.allreduce != "fused" else None)

    # ---- timed region: whole steps (graph replay), clocks sampled meanwhile --
    clocks = ClockSampler(local)
    clocks.start()
    ms = time_graph(g_step, args.steps, args.warmup, barrier)
    clk = clocks.stop()
    ms = max_over_ranks(ms, dist_on, dev)

    if args.part == "step":
        if rank == 0:
            print(json.dumps({"part": "step", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup}))
        del g_step, g_gemv, g_attn, g_comm
        if dist_on:
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier()
            if comm is not None:
                comm.close()
            dist.destroy_process_group()
        return None

    # ---- per-kernel breakdown (same graphs, kernel class alone) ------------
    ms_gemv = max_over_ranks(time_graph(g_gemv, args.steps, 2, barrier), dist_on, dev)
    ms_attn = max_over_ranks(time_graph(g_attn, args.steps, 2, barrier), dist_on, dev)
    ms_comm = (max_over_ranks(time_graph(g_comm, args.steps, 2, barrier), dist_on, dev)
               if g_comm is not None else None)
    # ---- the step's parts at B = 1, 4, 8 (north_star's "at batch 1-8") ----
    hbm_peak_sweep = _peaks().get("hbm_gbs", 6650.0)
    sweep = {}
    for Bs in BATCH_SWEEP:
        if Bs == args.batch:
            lay_s, buf_s, gg, ga = layers, bufs, g_gemv, g_attn
        else:
            lay_s, buf_s = build_model(args, dev, weights, Bs)
            gg = capture(lambda: run_step(lay_s, buf_s, args, which=("gemv",)))
            ga = capture(lambda: run_step(lay_s, buf_s, args, which=("attn",)))
        ms_g = max_over_ranks(time_graph(gg, args.steps, 2, barrier), dist_on, dev)
        ms_a = max_over_ranks(time_graph(ga, args.steps, 2, barrier), dist_on, dev)
        gb = args.layers * sum(gemv_bytes(N, K, Bs) for _, N, K in rank_shapes(args.tp))
        ab = args.layers * decode_bytes(Bs, args.ctx, args.tp)
        sweep[Bs] = {
            "mxfp4_gemv": {"us_per_step": ms_g * 1e3, "launches_per_step": 4 * args.layers,
                           "gbs": gb / (ms_g * 1e-3) / 1e9, "hbm_frac": gb / (ms_g * 1e-3) / 1e9 / hbm_peak_sweep},
            "decode_attn": {"us_per_step": ms_a * 1e3, "launches_per_step": args.layers,
                            "gbs": ab / (ms_a * 1e-3) / 1e9, "hbm_frac": ab / (ms_a * 1e-3) / 1e9 / hbm_peak_sweep}}
        if Bs != args.batch:
            del gg, ga, lay_s, buf_s
            torch.cuda.empty_cache()
    us_pre, flops_pre = prefill_part(dev, args.steps, 2, barrier)
    us_pre = max_over_ranks(us_pre, dist_on, dev)
    us_wide, bytes_wide, flops_wide = wide_gemm_part(dev, args.steps, 2, barrier, args.tp)
    us_wide = max_over_ranks(us_wide, dist_on, dev)
    dec7, pre7 = {}, {}
    for Bs in BATCH_SWEEP:
        ms_b, _, ms_p = decode_7b_part(args, dev, barrier, args.allreduce_fn if args.tp > 1 else None, Bs)
        dec7[Bs] = max_over_ranks(ms_b, dist_on, dev)
        pre7[Bs] = max_over_ranks(ms_p, dist_on, dev)
    ms_tok = dec7[args.batch] if args.batch in dec7 else None
    serve = None
    if args.serving == "on":
        res, serve_tokens, serve_kv, serve_pre, serve_gemm = serving_part(args, dev, barrier)
        serve = {k: max_over_ranks(v, dist_on, dev) for k, v in res.items()}
    # one rank's bytes (the per-GPU roofline)
    gemv_bytes_step = args.layers * sum(gemv_bytes(N, K, args.batch) for _, N, K in rank_shapes(args.tp))
    attn_bytes_step = args.layers * decode_bytes(args.batch, args.ctx, args.tp)

    # ---- e2e through the public API with host buffers ----------------------
    B = args.batch
    h_x = torch.randn(args.layers, B, 4096).to(torch.bfloat16).pin_memory()
    h_act = torch.randn(args.layers, B, 14336 // args.tp).to(torch.bfloat16).pin_memory()
    d_x = torch.stack([lay["x"] for lay in layers])  # staging views refreshed per step
    d_act = torch.stack([lay["act"] for lay in layers])
    for i, lay in enumerate(layers):
        lay["x"] = d_x[i]
        lay["act"] = d_act[i]
    g_e2e = capture(lambda: run_step(layers, bufs, args))
    h_out = torch.empty(B, 4096, dtype=torch.bfloat16).pin_memory()
    h_attn = torch.empty(B, HQ // args.tp, D, dtype=torch.bfloat16).pin_memory()
    h2d = h_x.numel() * 2 + h_act.numel() * 2
    d2h = h_out.numel() * 2 + h_attn.numel() * 2

    def e2e_step():
        d_x.copy_(h_x, non_blocking=True)
        d_act.copy_(h_act, non_blocking=True)
        g_e2e.replay()
        h_out.copy_(bufs["down"], non_blocking=True)
        h_attn.copy_(bufs["attn"], non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / args.steps, dist_on, dev)

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    gemv_gbs = gemv_bytes_step / (ms_gemv * 1e-3) / 1e9
    n_gemv = args.layers * 4

    # DRAM bytes per launch of the dominant kernel (dram__bytes_read.sum +
    # dram__bytes_write.sum) from the committed ncu summary of the four 7B
    # shapes at M = 1, averaged over the four launches of a layer
    traffic, traffic_src = None, None
    if args.gemv == "tc" and args.batch == 1 and args.tp == 1:
        traffic, traffic_src = profile_traffic()

    result = None
    if rank == 0:
        cpu = cpu_baseline(args) if world == 1 else None
        cpu_pre = cpu_prefill_baseline() if world == 1 else None
        cpu_dec = {b: cpu_decoder_baseline(b) for b in BATCH_SWEEP} if world == 1 else {}
        cpu_srv = cpu_serving_baseline() if world == 1 and serve is not None else None
        copies = world // args.tp  # full model copies streamed per step
        value = copies * step_bytes / (ms * 1e-3) / 1e9
        result = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if args.tp > 1 else "weak",
            "vs_baseline": None,
            "dtype": "e2m1/e4m3 operands, f32 accumulate",
            "data": "synthetic", "config": workload_config(args),
            "tok_s_hot_path_only": copies * args.batch / (ms * 1e-3),
            "parts": {
                "mxfp4_gemv": {"us_per_step": ms_gemv * 1e3, "launches_per_step": n_gemv,
                               "gbs": gemv_gbs, "kernel": args.gemv},
                "decode_attn": {"us_per_step": ms_attn * 1e3, "launches_per_step": args.layers,
                                "gbs": attn_bytes_step / (ms_attn * 1e-3) / 1e9},
                "prefill_attn": {"workload": "config 3: varlen causal prefill, 4 seqs "
                                             f"{list(PREFILL_LENS)}, GQA 32/8, D 128, fp8 paged KV",
                                 "us_per_call": us_pre, "gflop_per_call": flops_pre / 1e9,
                                 "tflops": flops_pre / (us_pre * 1e-6) / 1e12,
                                 "bound": "tensor", "peak_tflops": peaks.get("bf16_tflops", 1590.0),
                                 "frac": flops_pre / (us_pre * 1e-6) / 1e12
                                 / peaks.get("bf16_tflops", 1590.0),
                                 "cpu_baseline": cpu_pre,
                                 "note": "timed outside the decode step (not part of value); "
                                         "each rank runs the full call"},
                "mxfp4_gemm_m64": {"workload": f"config 2 at M = {WIDE_M}: qkv, o, gate_up, down "
                                               "(this rank's shards) on the wide-batch GEMM "
                                               "(tcgen05 kind::mxf8f6f4, x as two exact e4m3 terms)",
                                   "us_per_layer": us_wide,
                                   "gbs": bytes_wide / (us_wide * 1e-6) / 1e9,
                                   "hbm_frac": bytes_wide / (us_wide * 1e-6) / 1e9 / hbm_peak,
                                   "tflops": flops_wide / (us_wide * 1e-6) / 1e12,
                                   "tensor_frac": flops_wide / (us_wide * 1e-6) / 1e12
                                   / peaks.get("bf16_tflops", 1590.0),
                                   "note": "timed outside the decode step (not part of value); "
                                           "tflops counts 2 M N K (the tensor core runs two e4m3 "
                                           "terms at twice the bf16 rate, so bf16 peak is the bound)"},
                "decode_7b": {"workload": f"config 4: full 7B MXFP4 decoder (RMSNorm, qkv, RoPE + fp8 "
                                          f"KV write, decode attention, o, SwiGLU MLP, bf16 lm_head "
                                          f"128256, greedy argmax), batch 1/4/8, a random-id "
                                          f"{DECODE_PROMPT}-token prompt per sequence prefilled by the model "
                                          f"(prefill_ms: wide MXFP4 GEMMs, RoPE + fp8 KV write, varlen causal "
                                          f"prefill attention), then decode tokens {DECODE_PROMPT}+ reading "
                                          f"that cache, one CUDA-graph replay per token",
                              "by_batch": {str(b): {"ms_per_token_step": dec7[b],
                                                    "tok_s": copies * b / (dec7[b] * 1e-3),
                                                    "prefill_ms": pre7[b],
                                                    "prefill_tok_s": copies * b * DECODE_PROMPT / (pre7[b] * 1e-3),
                                                    "cpu_baseline": cpu_dec.get(b)}
                                           for b in BATCH_SWEEP},
                              "ms_per_token_step": ms_tok,
                              "tok_s": copies * args.batch / (ms_tok * 1e-3) if ms_tok else None,
                              "note": "timed outside the hot-path step (not part of value)"},
                "batch_sweep": {"workload": "the step's two kernel classes alone (same graphs as value) at "
                                            "B = 1, 4, 8: MXFP4 GEMV at M = B (qkv, o, gate_up, down x "
                                            f"{args.layers} layers) and decode attention over B x {args.ctx} "
                                            "tokens", "by_batch": {str(b): v for b, v in sweep.items()},
                                "peak_gbs": hbm_peak},
            },
            "roofline": {"bound": "hbm",
                         "kernel": "mxfp4_mma_kernel" if args.gemv == "tc" else "mxfp4_gemv_kernel",
                         "achieved": gemv_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gemv_gbs / hbm_peak, "peak_source": peak_src,
                         "bytes_per_launch_avg": gemv_bytes_step / n_gemv,
                         "us_per_launch_avg": ms_gemv * 1e3 / n_gemv,
                         "traffic": traffic,
                         "traffic_source": traffic_src},
            "cpu_baseline": cpu,
            "e2e": {"value": copies * step_bytes / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "pinned host activations -> H2D, then one CUDA-graph replay of the step's "
                            f"public-API calls (h4mv.{'mxfp4_gemm' if args.gemv == 'tc' else 'mxfp4_gemv'}, "
                            "fp8kv_v3.run) captured once, as a graph-replayed engine runs them (their Python "
                            "dispatch is outside the timed region), D2H of outputs"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if serve is not None:
            result["parts"]["serving_5"] = {
                "workload": f"config 5: 7B, {SERVE_DECODES} decodes (ctx ~U[{SERVE_CTX[0]}, {SERVE_CTX[1]}], seeded) "
                            f"+ {SERVE_PREFILLS} new {SERVE_PREFILL_LEN}-token prefills per step = {serve_tokens} "
                            "tokens; fragmented random block table over one fp8 pool per layer (synthetic "
                            "prompt pages); 32 layers x [qkv, KV write, attention, o, gate_up, down] on the "
                            "wide MXFP4 GEMM; NCCL allreduce under tensor parallelism",
                "tokens_per_step": serve_tokens,
                "ms_per_step_mixed": serve["mixed"], "ms_per_step_split": serve["split"],
                "tok_s_mixed": copies * serve_tokens / (serve["mixed"] * 1e-3),
                "tok_s_split": copies * serve_tokens / (serve["split"] * 1e-3),
                "attention_ms_mixed": serve["attn_mixed"], "attention_ms_split": serve["attn_split"],
                "attention_ms_one_call": serve["attn_one_call"],
                "gemm_ms": serve["gemm"],
                "gemm_tflops": serve_gemm / (serve["gemm"] * 1e-3) / 1e12,
                "decode_kv_gb_per_step": serve_kv / 1e9, "prefill_gflop_per_step": serve_pre / 1e9,
                "cpu_baseline": cpu_srv,
                "note": "mixed = b200kv_attn_varlen_mixed, what the vLLM forward patch calls (decode "
                        "rows to the decode kernel, prefills to the varlen kernel, split on the device); "
                        "split = the same two kernels as two calls on host-known row ranges; one_call = "
                        "the varlen kernel for the whole batch; "
                        "attention_ms includes the KV write; gate_up runs with the SwiGLU epilogue "
                        "(b200kv_mxfp4_gemm_wide_swiglu); per rank under tensor parallelism"}
        if ms_comm is not None:
            result["parts"]["allreduce"] = {
                "us_per_step": ms_comm * 1e3, "calls_per_step": 2 * args.layers,
                "us_per_call": ms_comm * 1e3 / (2 * args.layers),
                "bytes_per_call": args.batch * 4096 * 2,
                "impl": ("b200kv one-shot peer-memory allreduce (NVLink stores + flags)"
                         if args.allreduce == "peer" else "NCCL all_reduce (torch.distributed)")}
            result["parts"]["mxfp4_gemv"]["note"] = "one rank's shards; gbs is per GPU"
            result["parts"]["decode_attn"]["note"] = "one rank's kv heads; gbs is per GPU"
        print(json.dumps(result), flush=True)
    del g_step, g_gemv, g_attn, g_e2e, g_comm  # graphs holding NCCL calls go first
    if dist_on:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
    return result


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 300 graph replays, ~0.6 s of clocks samples; "
                         "10 one-layer host samples for --impl reference)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--parallel", choices=("tp", "replicas"), default="tp",
                    help="N > 1: tensor parallelism over the N GPUs (default) or N full replicas")
    ap.add_argument("--allreduce", choices=("peer", "fused", "nccl"), default="peer",
                    help="tensor-parallel allreduce: b200kv's one-shot peer-memory kernel after the o/down "
                         "GEMV (default), in the GEMV's epilogue over peer memory, or NCCL")
    ap.add_argument("--serving", choices=("on", "off"), default="on",
                    help="time the config-5 serving step (about 70 GB of KV pool per GPU at tp 1)")
    ap.add_argument("--gemv", choices=("tc", "cuda-core"), default="tc",
                    help="MXFP4 kernel: block-scaled tensor cores (packed scales) or CUDA-core mma.sync")
    ap.add_argument("--part", choices=("all", "step", "mxfp4_m1", "decode_attn", "decode_7b", "prefill"),
                    default="all",
                    help="all: the full line; step: the headline step only (for an ncu launch list); "
                         "mxfp4_m1: the four 7B MXFP4 launches at M = 1, --steps times (for an ncu capture); "
                         "decode_attn: 32 decode-attention launches at --batch / --kv-heads; "
                         "decode_7b: the 7B decoder's token step at --batch; prefill: config 3 alone")
    ap.add_argument("--kv-heads", type=int, default=HKV,
                    help="--part decode_attn: kv heads per GPU (1, 2, 4: the 7B model's TP8/4/2 shards)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 300 if args.impl == "b200" else 10
    world = int(os.environ.get("WORLD_SIZE", "1"))
    args.tp = world if world > 1 and args.parallel == "tp" else 1
    args.warmup = max(args.warmup, 3) if args.impl == "b200" else args.warmup
    args.rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args)
    elif args.part == "mxfp4_m1":
        run_mxfp4_m1(args)
    elif args.part == "decode_attn":
        run_decode_attn(args)
    elif args.part == "decode_7b":
        run_decode_7b(args)
    elif args.part == "prefill":
        run_prefill(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
