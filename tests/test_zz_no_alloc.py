"""The allocation-free wide MXFP4 GEMM (b200kv_mxfp4_gemm_wide_noalloc), for
callers that cannot allocate device memory, e.g. an engine whose KV-cache pool
already holds all free HBM or a C host without a device allocator: its scratch
is an array inside the library.  Called twice in a row through the C ABI with
different inputs, each result equals the workspace entry point's output for
the same inputs (same kernels, same arithmetic); sizes past the array's limit
are refused.  Collected last so that a run stopping at a failure here has run
every other test."""
import pytest
import torch

import mxfp4_oracle as MO

pytestmark = pytest.mark.gpu


def test_two_calls_match_workspace_entry_point(cuda):
    import h4mv
    from _b200kv import lib
    stream = torch.cuda.current_stream().cuda_stream
    for (N, K, M, seed) in [(4096, 4096, 64, 1), (1000, 14336, 100, 2), (256, 16384, 128, 3)]:
        W, S, St, X = MO.make_case(N, K, M, seed=seed)
        Wd, Xd = W.to(cuda), X.to(cuda)
        packed, _ = h4mv.pack_scales(St.to(cuda), N, K)
        want = h4mv.mxfp4_gemm_wide(Xd, Wd, packed)
        got = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        rc = lib.b200kv_mxfp4_gemm_wide_noalloc(Wd.data_ptr(), packed.data_ptr(), Xd.data_ptr(), K,
                                                got.data_ptr(), N, K, M, stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(got, want), (N, K, M)
        ref = MO.mxfp4_linear_reference(W, S, X)
        assert MO.rel_to_max_err(got.float().cpu(), ref) < 5e-3


def test_refuses_sizes_past_the_scratch(cuda):
    from _b200kv import lib
    W = torch.zeros(128, 64, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    big = torch.zeros(129, 128, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(129, 128, dtype=torch.bfloat16, device=cuda)
    assert lib.b200kv_mxfp4_gemm_wide_noalloc(W.data_ptr(), W.data_ptr(), big.data_ptr(), 128,
                                              out.data_ptr(), 128, 128, 129, stream) == 4
    assert lib.b200kv_mxfp4_gemm_wide_noalloc(W.data_ptr(), W.data_ptr(), big.data_ptr(), 16512,
                                              out.data_ptr(), 128, 16512, 1, stream) == 4
    # M = 128 fills the array to its last byte at K = 16384; one more k-step is refused
    assert lib.b200kv_mxfp4_gemm_wide_noalloc(W.data_ptr(), W.data_ptr(), big.data_ptr(), 16512,
                                              out.data_ptr(), 128, 16512, 128, stream) == 4
    # argument errors come first, as in the workspace entry point
    assert lib.b200kv_mxfp4_gemm_wide_noalloc(None, W.data_ptr(), big.data_ptr(), 128,
                                              out.data_ptr(), 128, 128, 129, stream) == 1
    assert lib.b200kv_mxfp4_gemm_wide_noalloc(W.data_ptr(), W.data_ptr(), big.data_ptr(), 64,
                                              out.data_ptr(), 128, 128, 129, stream) == 1
