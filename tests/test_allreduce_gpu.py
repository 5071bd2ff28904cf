"""The tensor-parallel one-shot allreduce (b200kv_allreduce_oneshot) and the
GEMV with the allreduce in its epilogue (b200kv_mxfp4_gemm_allreduce) on two
B200s: two processes, one per GPU, exchange their IPC handles over an NCCL
process group.  The result must equal, bit for bit on every rank, the rank-
ordered fp32 sum of the bf16 partials rounded to bf16 -- over consecutive calls
(both buffer parities), in place, for the decode sizes M = 1 and 8, and inside
a replayed CUDA graph.  Skipped with fewer than two GPUs."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG

pytestmark = pytest.mark.gpu
TP = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expected(parts):
    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for p in parts:
        acc += p.float()
    return acc.to(torch.bfloat16)


def _rank_main(rank, port):
    import sys
    if PKG not in sys.path:
        sys.path.insert(0, PKG)
    import _b200kv
    import tp
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=TP, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ar = tp.PeerAllreduce()
    try:
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        for n in (4096, 8 * 4096, 4096, 4096, 8 * 4096):  # both parities, two sizes
            x = torch.randn(n, device=dev, generator=g).to(torch.bfloat16)
            parts = [torch.empty_like(x) for _ in range(TP)]
            dist.all_gather(parts, x)
            want = _expected(parts)
            y = ar(x.clone())
            assert torch.equal(y, want), n
        # captured in a CUDA graph, replayed: three calls per replay
        bufs = [torch.empty(4096, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for b in bufs:
                ar(b.normal_())
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for b in bufs:
                ar(b)
        for _ in range(2):
            srcs = [torch.randn(4096, device=dev, generator=g).to(torch.bfloat16) for _ in bufs]
            wants = []
            for sbuf in srcs:
                parts = [torch.empty_like(sbuf) for _ in range(TP)]
                dist.all_gather(parts, sbuf)
                wants.append(_expected(parts))
            for b, sbuf in zip(bufs, srcs):
                b.copy_(sbuf)
            graph.replay()
            torch.cuda.synchronize()
            for b, w in zip(bufs, wants):
                assert torch.equal(b, w)
        del graph
        torch.cuda.synchronize()
        assert _b200kv.device_status() == 0
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        ar.close()
        dist.destroy_process_group()


def test_peer_allreduce_two_gpus():
    if torch.cuda.device_count() < TP:
        pytest.skip("needs two GPUs")
    mp.spawn(_rank_main, args=(_free_port(),), nprocs=TP, join=True)


def _decoder_rank(rank, port):
    """The tensor-parallel decoder (2 ranks) against the CPU oracle of the whole
    model with the row-parallel partials rounded to bf16 before their sum (the
    numerics of tensor parallelism): each rank's logits are its vocab slice of
    the oracle's, the greedy tokens agree where the oracle's top two are
    separated."""
    import sys
    from conftest import ORACLE
    for p in (PKG, ORACLE):
        if p not in sys.path:
            sys.path.insert(0, p)
    import decoder
    import decoder_oracle as DO
    import tp
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=TP, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ar = tp.PeerAllreduce()
    try:
        cfg = decoder.DecoderConfig(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128,
                                    inter=1024, vocab=1000)
        seed, B, max_ctx = 5, 2, 64

        def gather(out, inp):
            dist.all_gather_into_tensor(out.view(-1), inp.contiguous().view(-1))
        # e8m0 scales 2^-9..2^-6: attention scores of order one, so the model is not
        # so sensitive that one bf16 rounding of a partial changes later tokens
        scales = (118, 122)
        dec = decoder.MXFP4Decoder(cfg, dev, B, max_ctx, seed=seed, tp=TP, rank=rank, allreduce=ar,
                                   gather=gather, gen_device="cpu", scales=scales)
        layers = []
        for li in range(cfg.layers):
            lay = decoder.random_layer(cfg, li, seed, "cpu", scales)
            layers.append({k: ((v[0], v[1].t().contiguous()) if isinstance(v, tuple) else v)
                           for k, v in lay.items()})
        weights = dict(decoder.random_head(cfg, seed, "cpu"), layers=layers)
        nb = B * dec.maxblk
        caches = [{"k": torch.zeros(nb, 16, cfg.kv_heads, 128, dtype=torch.float8_e4m3fn),
                   "v": torch.zeros(nb, 16, cfg.kv_heads, 128, dtype=torch.float8_e4m3fn),
                   "ks": 1 / 8, "vs": 1 / 8} for _ in range(cfg.layers)]
        table = DO.rope_table(max_ctx, 128, cfg.rope_theta)
        bt = dec.block_table.cpu()
        tokens = torch.tensor([3, 7], dtype=torch.int64)
        dec.tokens.copy_(tokens)
        positions = torch.zeros(B, dtype=torch.int32)
        vl = cfg.vocab // TP
        for step in range(5):
            want = DO.decode_step(cfg, weights, caches, tokens, positions, bt, table, tp=TP)
            nxt = dec.step().cpu()
            got = dec.logits.cpu()
            mine = want[:, rank * vl:(rank + 1) * vl]
            err = float((got - mine).abs().max() / want.abs().max())
            assert err < 2e-2, (rank, step, err)
            top2 = want.topk(2, dim=1).values
            sep = (top2[:, 0] - top2[:, 1]) > 4 * float((got - mine).abs().max())
            assert torch.equal(nxt[sep], want.argmax(1)[sep]), (rank, step)
            tokens = nxt.clone()
            positions = positions + 1
        torch.cuda.synchronize()
        import _b200kv
        assert _b200kv.device_status() == 0
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        ar.close()
        dist.destroy_process_group()


def test_tensor_parallel_decoder_two_gpus():
    if torch.cuda.device_count() < TP:
        pytest.skip("needs two GPUs")
    mp.spawn(_decoder_rank, args=(_free_port(),), nprocs=TP, join=True)


def _fused_rank_main(rank, port):
    """b200kv_mxfp4_gemm_allreduce on two GPUs: every rank's K shard of the
    row-parallel product; every rank must get, bit for bit, the rank-ordered
    sum of the plain products' bf16 partials, over mixed shapes and M, both
    parities, and graph replays; then the tensor-parallel decoder with o and
    down fused gives the same logits as with the separate allreduce."""
    import sys
    if PKG not in sys.path:
        sys.path.insert(0, PKG)
    import _b200kv
    import decoder
    import h4mv
    import tp
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=TP, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ar = tp.PeerAllreduce()
    try:
        g = torch.Generator(device=dev).manual_seed(200 + rank)
        sets = {}
        for K in (2048, 7168):
            W = torch.randint(0, 256, (4096, K // 2), dtype=torch.uint8, device=dev, generator=g)
            St = torch.randint(118, 124, (4096, K // 32), dtype=torch.uint8, device=dev, generator=g)
            sets[K] = (W, h4mv.pack_scales(St, 4096, K)[0])
        for call, (K, M) in enumerate([(2048, 1), (7168, 1), (2048, 8), (2048, 3), (7168, 8), (2048, 1)]):
            W, P = sets[K]
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            part = h4mv.mxfp4_gemm(x, W, P)
            parts = [torch.empty_like(part) for _ in range(TP)]
            dist.all_gather(parts, part)
            want = _expected(parts)
            got = ar.gemm(x, W, P, torch.empty_like(part))
            torch.cuda.synchronize()
            assert torch.equal(got, want), (rank, call, K, M)
        # three fused calls per graph replay
        W, P = sets[2048]
        xs = [torch.empty(2, 2048, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        outs = [torch.empty(2, 4096, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        for x in xs:
            x.normal_(generator=g)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for x, o in zip(xs, outs):
                ar.gemm(x, W, P, o)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for x, o in zip(xs, outs):
                ar.gemm(x, W, P, o)
        for _ in range(2):
            wants = []
            for x in xs:
                x.copy_(torch.randn(2, 2048, device=dev, generator=g))
                part = h4mv.mxfp4_gemm(x, W, P)
                parts = [torch.empty_like(part) for _ in range(TP)]
                dist.all_gather(parts, part)
                wants.append(_expected(parts))
            graph.replay()
            torch.cuda.synchronize()
            for o, w in zip(outs, wants):
                assert torch.equal(o, w)
        del graph
        # the decoder: o and down fused vs separate allreduce
        cfg = decoder.DecoderConfig(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128,
                                    inter=1024, vocab=1000)

        def gather(out, inp):
            dist.all_gather_into_tensor(out.view(-1), inp.contiguous().view(-1))
        decs = [decoder.MXFP4Decoder(cfg, dev, 2, 64, seed=5, tp=TP, rank=rank, allreduce=ar, gather=gather,
                                     gen_device="cpu", fuse_allreduce=f) for f in (True, False)]
        assert decs[0]._fused_ar and not decs[1]._fused_ar
        for d in decs:
            d.tokens.copy_(torch.tensor([3, 7]))
        for step in range(4):
            for d in decs:
                d.step()
            torch.cuda.synchronize()
            assert torch.equal(decs[0].logits, decs[1].logits), (rank, step)
        assert _b200kv.device_status() == 0
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        ar.close()
        dist.destroy_process_group()


def test_fused_gemm_allreduce_two_gpus():
    if torch.cuda.device_count() < TP:
        pytest.skip("needs two GPUs")
    mp.spawn(_fused_rank_main, args=(_free_port(),), nprocs=TP, join=True)
