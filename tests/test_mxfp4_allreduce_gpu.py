"""The row-parallel MXFP4 product with its allreduce in the epilogue
(b200kv_mxfp4_gemm_allreduce) on one B200 at tp = 1: the rank pushes its tile
partials into its own communication buffer and sums them back, so the result
must equal b200kv_mxfp4_gemm bit for bit over consecutive calls (both buffer
parities, the per-tile call counters advancing), mixed shapes sharing one
buffer set, and CUDA-graph replays.  The two-GPU exchange is in
test_allreduce_gpu.py."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


class _SelfComm:
    """One rank's buffer set, as tp.PeerAllreduce builds it for tp = 1."""

    def __init__(self):
        from _b200kv import check, lib
        self.lib = lib
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        check(lib.b200kv_comm_alloc(ctypes.byref(own), handle), "b200kv_comm_alloc")
        self.own = own.value
        self.bufs = (ctypes.c_void_p * 1)(own.value)

    def gemm(self, x, W, packed, out):
        from _b200kv import check
        M, K = x.shape
        check(self.lib.b200kv_mxfp4_gemm_allreduce(W.data_ptr(), packed.data_ptr(), x.data_ptr(), out.data_ptr(),
                                                   W.shape[0], K, M, self.bufs, 0, 1,
                                                   torch.cuda.current_stream(x.device).cuda_stream),
              "b200kv_mxfp4_gemm_allreduce")
        return out

    def close(self):
        torch.cuda.synchronize()
        self.lib.b200kv_comm_free(self.own)


def _weights(N, K, seed, dev):
    import h4mv
    g = torch.Generator().manual_seed(seed)
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g).to(dev)
    St = torch.randint(118, 124, (N, K // 32), dtype=torch.uint8, generator=g).to(dev)
    return W, h4mv.pack_scales(St, N, K)[0]


def test_single_rank_equals_plain_gemm(cuda):
    import h4mv
    comm = _SelfComm()
    try:
        sets = {K: _weights(4096, K, K, cuda) for K in (2048, 14336 // 2)}
        g = torch.Generator(device=cuda).manual_seed(0)
        for call, (K, M) in enumerate([(2048, 1), (2048, 1), (7168, 8), (2048, 3), (7168, 1), (2048, 8)]):
            W, P = sets[K]
            x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
            want = h4mv.mxfp4_gemm(x, W, P)
            got = comm.gemm(x, W, P, torch.empty_like(want))
            assert torch.equal(got, want), (call, K, M)
        import _b200kv
        assert _b200kv.device_status() == 0
    finally:
        comm.close()


@pytest.mark.parametrize("ks", [1, 2, 4])
def test_single_rank_every_k_split(cuda, monkeypatch, ks):
    import h4mv
    comm = _SelfComm()
    try:
        W, P = _weights(1024, 4096, ks, cuda)
        x = torch.randn(5, 4096, device=cuda).to(torch.bfloat16)
        monkeypatch.setenv("B200KV_MMA_KSPLIT", str(ks))
        want = h4mv.mxfp4_gemm(x, W, P)
        for _ in range(3):
            assert torch.equal(comm.gemm(x, W, P, torch.empty_like(want)), want)
    finally:
        comm.close()


def test_single_rank_graph_replay(cuda):
    import h4mv
    comm = _SelfComm()
    try:
        W, P = _weights(4096, 2048, 1, cuda)
        x = torch.empty(2, 2048, dtype=torch.bfloat16, device=cuda)
        outs = [torch.empty(2, 4096, dtype=torch.bfloat16, device=cuda) for _ in range(3)]
        x.normal_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for o in outs:
                comm.gemm(x, W, P, o)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for o in outs:
                comm.gemm(x, W, P, o)
        for rep in range(3):
            x.copy_(torch.randn(2, 2048, device=cuda))
            want = h4mv.mxfp4_gemm(x, W, P)
            graph.replay()
            torch.cuda.synchronize()
            for o in outs:
                assert torch.equal(o, want), rep
        del graph
        import _b200kv
        assert _b200kv.device_status() == 0
    finally:
        comm.close()


def test_rejects_bad_arguments(cuda):
    from _b200kv import lib
    INVALID, UNSUPPORTED = 1, 2  # status codes of include/b200kv.h
    comm = _SelfComm()
    try:
        W, P = _weights(4096, 256, 0, cuda)
        x = torch.zeros(2, 256, dtype=torch.bfloat16, device=cuda)
        out = torch.empty(2, 4096, dtype=torch.bfloat16, device=cuda)
        st = torch.cuda.current_stream().cuda_stream
        args = (W.data_ptr(), P.data_ptr(), x.data_ptr(), out.data_ptr())
        assert lib.b200kv_mxfp4_gemm_allreduce(*args, 4096, 256, 2, None, 0, 1, st) == INVALID
        assert lib.b200kv_mxfp4_gemm_allreduce(*args, 4096, 256, 2, comm.bufs, 1, 1, st) == INVALID  # rank >= tp
        assert lib.b200kv_mxfp4_gemm_allreduce(*args, 4096, 256, 2, comm.bufs, 0, 9, st) == INVALID  # tp > 8
        assert lib.b200kv_mxfp4_gemm_allreduce(*args, 4000, 256, 2, comm.bufs, 0, 1, st) == UNSUPPORTED  # N % 128
        W2, P2 = _weights(8192, 256, 0, cuda)
        x8 = torch.zeros(8, 256, dtype=torch.bfloat16, device=cuda)
        o8 = torch.empty(8, 8192, dtype=torch.bfloat16, device=cuda)
        # M N above the line area of a buffer (8 x 4096 elements)
        assert lib.b200kv_mxfp4_gemm_allreduce(W2.data_ptr(), P2.data_ptr(), x8.data_ptr(), o8.data_ptr(), 8192,
                                               256, 8, comm.bufs, 0, 1, st) == UNSUPPORTED
    finally:
        comm.close()
