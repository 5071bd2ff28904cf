"""Tensor-parallel layout (tp.py) on CPU: two gloo ranks shard a seeded layer
the way the multi-GPU bench does and, with the CPU oracle standing in for the
kernels, reproduce the unsharded results.  Row-parallel partials summed by the
allreduce match the full product to fp32 rounding (sum order differs);
column-parallel rows and kv-head shards of attention match exactly."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ORACLE, PKG

TP = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port):
    import sys
    for p in (PKG, ORACLE):
        if p not in sys.path:
            sys.path.insert(0, p)
    import fp8kv_oracle as FO
    import mxfp4_oracle as MO
    import tp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=TP)
    try:
        # row-parallel (o, down): K split, partial outputs summed
        W, S, St, X = MO.make_case(96, 1024, 3, seed=5)
        full = MO.mxfp4_linear_reference(W, S, X)
        Ws, Sts = tp.row_shard(W, St, rank, TP)
        k = 1024 // TP
        part = MO.mxfp4_linear_reference(Ws, Sts.t().contiguous(), X[:, rank * k:(rank + 1) * k])
        tp.allreduce_(part)
        assert torch.allclose(part, full, rtol=1e-5, atol=1e-5 * full.abs().max().item())

        # column-parallel (gate_up): N split, rows of the full output
        Wc, Stc = tp.col_shard(W, St, rank, TP)
        n = 96 // TP
        col = MO.mxfp4_linear_reference(Wc, Stc.t().contiguous(), X)
        assert torch.equal(col, full[:, rank * n:(rank + 1) * n])

        # fused qkv: this rank's q, k and v heads
        hq, hkv, d = 8, 4, 32
        Wq, Sq, Stq, Xq = MO.make_case((hq + 2 * hkv) * d, 256, 2, seed=6)
        fq = MO.mxfp4_linear_reference(Wq, Sq, Xq)
        Wqs, Stqs = tp.qkv_shard(Wq, Stq, hq, hkv, d, rank, TP)
        sq = MO.mxfp4_linear_reference(Wqs, Stqs.t().contiguous(), Xq)
        assert torch.equal(sq, fq[:, tp.qkv_rows(hq, hkv, d, rank, TP)])

        # attention by kv head: the heads of this rank, same numbers
        c = FO.make_decode_case(2, [300, 77], hq=8, hkv=4, seed=7)
        fa = FO.decode_reference(c["q"], c["k_cache"], c["v_cache"], c["qsl"], c["seq_lens"],
                                 c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
        hqs = 8 // TP
        qa = c["q"][:, rank * hqs:(rank + 1) * hqs]
        sa = FO.decode_reference(qa, tp.kv_head_shard(c["k_cache"], rank, TP),
                                 tp.kv_head_shard(c["v_cache"], rank, TP), c["qsl"], c["seq_lens"],
                                 c["block_table"], c["k_scale"], c["v_scale"], c["sm_scale"])
        assert torch.equal(sa, fa[:, rank * hqs:(rank + 1) * hqs])
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_layout_two_gloo_ranks():
    mp.spawn(_rank_main, args=(_free_port(),), nprocs=TP, join=True)


def test_shard_argument_checks():
    import tp
    W = torch.zeros(10, 48, dtype=torch.uint8)
    S = torch.zeros(10, 3, dtype=torch.uint8)
    with pytest.raises(ValueError):
        tp.col_shard(W, S, 0, 4)      # 10 rows over 4 ranks
    with pytest.raises(ValueError):
        tp.row_shard(W, S, 0, 2)      # K/tp = 48 is not a multiple of 32
    with pytest.raises(ValueError):
        tp.qkv_rows(32, 8, 128, 0, 3)
