"""Greedy argmax over fp32 logits rows (b200kv_argmax_rows) on the B200,
against torch.max(dim=1): the same maximum, and on ties the lowest index."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _argmax(x):
    from _b200kv import check, lib
    rows, cols = x.shape
    val = torch.full((rows,), float("nan"), device=x.device)
    idx = torch.full((rows,), -1, dtype=torch.int64, device=x.device)
    check(lib.b200kv_argmax_rows(x.data_ptr(), x.stride(0), rows, cols, val.data_ptr(), idx.data_ptr(),
                                 torch.cuda.current_stream(x.device).cuda_stream), "b200kv_argmax_rows")
    torch.cuda.synchronize()
    return val, idx


@pytest.mark.parametrize("rows,cols", [(1, 128256), (4, 128256), (8, 16032), (3, 7), (2, 1), (5, 1000)])
def test_matches_torch_max(cuda, rows, cols):
    g = torch.Generator(device=cuda).manual_seed(rows * 131 + cols)
    x = torch.randn(rows, cols, device=cuda, generator=g) * 5
    val, idx = _argmax(x)
    want_v, want_i = x.max(dim=1)
    assert torch.equal(val, want_v)
    assert torch.equal(idx, want_i)


def test_ties_take_the_lowest_index(cuda):
    x = torch.zeros(3, 128256, device=cuda) - 1.0
    x[0, [5, 70000, 128255]] = 3.0         # across chunks of different CTAs
    x[1, [16031, 16032]] = 2.0             # the boundary between two CTAs' chunks
    x[2, :] = 0.25                         # every element equal
    _, idx = _argmax(x)
    assert idx.tolist() == [5, 16031, 0]


def test_row_stride_and_null_value(cuda):
    from _b200kv import check, lib
    x = torch.randn(4, 3000, device=cuda)
    view = x[:, 100:2100]                  # row stride 3000, 2000 columns
    idx = torch.empty(4, dtype=torch.int64, device=cuda)
    check(lib.b200kv_argmax_rows(view.data_ptr(), view.stride(0), 4, 2000, None, idx.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream), "b200kv_argmax_rows")
    torch.cuda.synchronize()
    assert torch.equal(idx, view.max(dim=1).indices)


def test_argument_errors(cuda):
    from _b200kv import lib
    A = torch.zeros(16, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    assert lib.b200kv_argmax_rows(None, 4, 1, 4, None, A.data_ptr(), st) == 1
    assert lib.b200kv_argmax_rows(A.data_ptr(), 4, 1, 8, None, A.data_ptr(), st) == 1  # ld < cols
    assert lib.b200kv_argmax_rows(A.data_ptr(), 4, 0, 4, None, A.data_ptr(), st) == 1
