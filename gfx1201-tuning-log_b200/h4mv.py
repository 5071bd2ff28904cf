"""MXFP4 W4A16 matvec -- host entry points over libb200kv.so.

`launch` mirrors the reference test helper h4mv/h4mv_test.py:13-15 (same
argument order, raw ctypes call of h4mv_launch on the current stream);
`mxfp4_gemv` is the checked torch-level entry used by the op override
(fp8kv_hipw4.py) and by the benchmarks.
"""
import torch

import ctypes

from _b200kv import CHAIN_STORE, CHAIN_SWIGLU, ChainOp, check, lib

MAX_M = 8


def launch(W, St, X, Y, N, K, M):
    """Raw reference-style launch: h4mv_launch(W, St, X, Y, N, K, M, stream)."""
    lib.h4mv_launch(W.data_ptr(), St.data_ptr(), X.data_ptr(), Y.data_ptr(), N, K, M,
                    torch.cuda.current_stream().cuda_stream)
    check(lib.b200kv_last_error(), "h4mv_launch")


def mxfp4_gemv(x, weight, scale_t, out=None):
    """out[M, N] = x[M, K] @ dequant(weight [N, K/2] e2m1, scale_t [N, K/32] e8m0)^T.

    x bf16 contiguous with 1 <= M <= 8; weight uint8; scale_t uint8 (already
    transposed to [N, K/32]).  Returns bf16 [M, N].
    """
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bfloat16 tensor")
    if weight.dtype != torch.uint8 or scale_t.dtype != torch.uint8:
        raise TypeError("weight and scale must be uint8")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] * 2 != K or tuple(scale_t.shape) != (N, K // 32):
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w={tuple(weight.shape)} "
                         f"s={tuple(scale_t.shape)}")
    if not (weight.is_contiguous() and scale_t.is_contiguous()):
        raise ValueError("weight and scale must be contiguous")
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
    check(lib.b200kv_mxfp4_gemv(weight.data_ptr(), scale_t.data_ptr(), x.data_ptr(),
                                out.data_ptr(), N, K, M,
                                torch.cuda.current_stream(x.device).cuda_stream),
          "b200kv_mxfp4_gemv")
    return out


# ---- block-scaled tensor-core path (load-time packed scales) -------------------
SCALES_TRANSPOSED = 0   # St [N, K/32]
SCALES_CHECKPOINT = 1   # S [K/32, N]


def pack_scales(scales, N, K, layout=SCALES_TRANSPOSED):
    """Pack e8m0 scales into the tensor core's scale-factor atoms (once per
    weight).  Returns (packed uint8 tensor, has_edge) where has_edge reports
    scale bytes 0 or 255, which the tensor-core MMA reads as 2^-127 / NaN but
    the reference kernel as 0.0 / inf (keep such weights on mxfp4_gemv).
    Synchronises once to read the flag: call at load time, not per step."""
    nbytes = lib.b200kv_mxfp4_packed_scales_bytes(N, K)
    if nbytes == 0:
        raise ValueError(f"tensor-core path needs K % 128 == 0 (K={K})")
    if scales.dtype != torch.uint8 or not scales.is_contiguous():
        raise TypeError("scales must be a contiguous uint8 tensor")
    want = (N, K // 32) if layout == SCALES_TRANSPOSED else (K // 32, N)
    if tuple(scales.shape) != want:
        raise ValueError(f"scales shape {tuple(scales.shape)} != {want}")
    dev = scales.device
    packed = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    edge = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib.b200kv_mxfp4_pack_scales(scales.data_ptr(), layout, packed.data_ptr(), N, K,
                                       edge.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
          "b200kv_mxfp4_pack_scales")
    return packed, bool(edge.item())


def mxfp4_gemm(x, weight, packed_scales, out=None):
    """out[M, N] = x[M, K] @ dequant(weight, scales)^T on block-scaled tcgen05
    MMAs with scales packed by pack_scales(): 1 <= M <= 8 (K % 128 == 0) on the
    skinny kernel, larger M on mxfp4_gemm_wide (K % 128 == 0)."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bfloat16 tensor")
    if weight.dtype != torch.uint8 or not weight.is_contiguous():
        raise TypeError("weight must be a contiguous uint8 tensor")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] * 2 != K:
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w={tuple(weight.shape)}")
    if M > MAX_M:
        return mxfp4_gemm_wide(x, weight, packed_scales, out)
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
    check(lib.b200kv_mxfp4_gemm(weight.data_ptr(), packed_scales.data_ptr(), x.data_ptr(),
                                out.data_ptr(), N, K, M,
                                torch.cuda.current_stream(x.device).cuda_stream),
          "b200kv_mxfp4_gemm")
    return out


# (device index, stream handle) -> workspace of the wide GEMM's activation terms;
# calls on one stream run in order, so they can share it.  A workspace that is
# outgrown is kept alive, never freed: a CUDA graph captured with it (vLLM
# captures one per batch size, in one memory pool) still writes to it.
_workspaces = {}
_outgrown = []


def wide_workspace(M, K, device, stream):
    """The cached workspace for an (M, K) call on `stream` (grown on demand)."""
    need = lib.b200kv_mxfp4_gemm_wide_workspace_bytes(M, K)
    if need == 0:
        raise ValueError(f"wide GEMM needs K % 128 == 0 (K={K})")
    key = (device.index, stream.cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        if ws is not None:
            _outgrown.append(ws)
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def mxfp4_gemm_wide(x, weight, packed_scales, out=None, workspace=None):
    """out[M, N] = x[M, K] @ dequant(weight, scales)^T for wide batches on
    block-scaled tcgen05 MMAs (kind::mxf8f6f4: e2m1 weights, x as two exact
    e4m3 terms).  x bf16 2-D with unit inner stride (row stride a multiple of
    8), K % 128 == 0, scales packed by pack_scales().  The activation terms go
    to `workspace` (uint8, b200kv_mxfp4_gemm_wide_workspace_bytes) or to a
    buffer cached per device and stream."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a 2-D bfloat16 tensor with unit inner stride")
    if weight.dtype != torch.uint8 or not weight.is_contiguous():
        raise TypeError("weight must be a contiguous uint8 tensor")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] * 2 != K:
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w={tuple(weight.shape)}")
    stream = torch.cuda.current_stream(x.device)
    if workspace is None:
        workspace = wide_workspace(M, K, x.device, stream)
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
    check(lib.b200kv_mxfp4_gemm_wide(weight.data_ptr(), packed_scales.data_ptr(), x.data_ptr(),
                                     x.stride(0), workspace.data_ptr(), workspace.numel(),
                                     out.data_ptr(), N, K, M, stream.cuda_stream),
          "b200kv_mxfp4_gemm_wide")
    return out


def mxfp4_gemm_swiglu(x, weight, packed_scales, out=None, workspace=None):
    """act[M, I] = bf16(bf16(silu(g)) * u) of the gate_up projection, the
    activation applied in the GEMM's epilogue: `weight` is the [2 I, K/2] gate
    and up rows in gate_up_row_order(I) (scales packed after the permutation).
    Bit for bit mxfp4_gemm on the unpermuted weight followed by the SwiGLU
    kernel.  1 <= M <= 8 on the skinny kernel, larger M on the wide GEMM."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a 2-D bfloat16 tensor with unit inner stride")
    if weight.dtype != torch.uint8 or not weight.is_contiguous():
        raise TypeError("weight must be a contiguous uint8 tensor")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] * 2 != K:
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w={tuple(weight.shape)}")
    if N % 128:
        raise ValueError(f"SwiGLU epilogue needs 2 I % 128 == 0 (N={N})")
    if out is None:
        out = torch.empty((M, N // 2), device=x.device, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(x.device)
    if M <= MAX_M and x.is_contiguous():
        check(lib.b200kv_mxfp4_gemm_swiglu(weight.data_ptr(), packed_scales.data_ptr(), x.data_ptr(),
                                           out.data_ptr(), N, K, M, stream.cuda_stream),
              "b200kv_mxfp4_gemm_swiglu")
        return out
    if workspace is None:
        workspace = wide_workspace(M, K, x.device, stream)
    check(lib.b200kv_mxfp4_gemm_wide_swiglu(weight.data_ptr(), packed_scales.data_ptr(), x.data_ptr(),
                                            x.stride(0), workspace.data_ptr(), workspace.numel(),
                                            out.data_ptr(), N, K, M, stream.cuda_stream),
          "b200kv_mxfp4_gemm_wide_swiglu")
    return out


def gate_up_row_order(inter, device=None):
    """Row order of a fused [gate; up] weight ([2 inter, K], gate rows first) for
    the SwiGLU epilogues (mxfp4_gemm_swiglu, the chain's CHAIN_SWIGLU): blocks
    of 64 gate rows followed by the matching 64 up rows.  Apply once at load
    time to the weight's rows (and to its scales before packing);
    inter % 64 == 0."""
    if inter % 64:
        raise ValueError(f"SwiGLU interleave needs inter % 64 == 0 (inter={inter})")
    t = torch.arange(inter // 64, device=device)
    r = torch.arange(64, device=device)
    gate = (t[:, None] * 64 + r[None, :])
    return torch.stack([gate, gate + inter], dim=1).reshape(-1)


# ---- chains of dependent matvecs in one persistent launch ----------------------------
class MXFP4Chain:
    """A fixed list of dependent MXFP4 matvecs (1 <= M <= 8) run by one
    persistent launch (b200kv_mxfp4_chain).  Each op is a dict with
    `weight` (uint8 [N, K/2]), `scales` (packed by pack_scales), `out` (bf16
    [M, N], or [M, N/2] for epilogue CHAIN_SWIGLU) and either `x` (bf16 [M, K]
    with unit inner stride) or `x_from` (index of an earlier op whose output is
    x); optional `epilogue`.  The workspace, with its per-tile counters and
    ready flags, belongs to this object: it is zeroed once here and must not be
    shared with another chain.  Call run() on the stream the inputs were
    written on (CUDA-graph capturable)."""

    def __init__(self, ops, M, device):
        self.M = M
        self.device = torch.device(device)
        self._keep = []
        arr = (ChainOp * len(ops))()
        for j, o in enumerate(ops):
            w, p, out = o["weight"], o["scales"], o["out"]
            N, K = w.shape[0], w.shape[1] * 2
            x_from = o.get("x_from", -1)
            epi = o.get("epilogue", CHAIN_STORE)
            if w.dtype != torch.uint8 or not w.is_contiguous():
                raise TypeError("weight must be a contiguous uint8 tensor")
            if out.dtype != torch.bfloat16 or out.stride(-1) != 1:
                raise ValueError("out must be bf16 with unit inner stride")
            x = o.get("x")
            if x_from < 0:
                if x is None or x.dtype != torch.bfloat16 or x.stride(-1) != 1 or x.shape[-1] != K:
                    raise ValueError(f"op {j}: x must be bf16 [M, {K}] with unit inner stride")
            arr[j].weight = w.data_ptr()
            arr[j].packed_scales = p.data_ptr()
            arr[j].x = x.data_ptr() if x_from < 0 else 0
            arr[j].x_stride = x.stride(0) if x_from < 0 else 0
            arr[j].out = out.data_ptr()
            arr[j].out_stride = out.stride(0)
            arr[j].N, arr[j].K, arr[j].x_from, arr[j].epilogue = N, K, x_from, epi
            self._keep += [w, p, out] + ([x] if x_from < 0 else [])
        self._ops = arr
        self._n = len(ops)
        nbytes = lib.b200kv_mxfp4_chain_workspace_bytes(arr, self._n, M)
        if nbytes == 0:
            raise ValueError("invalid chain (shapes, x_from, epilogue or M)")
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)

    def run(self):
        check(lib.b200kv_mxfp4_chain(self._ops, self._n, self.M, self.workspace.data_ptr(),
                                     self.workspace.numel(), torch.cuda.current_stream(self.device).cuda_stream),
              "b200kv_mxfp4_chain")
