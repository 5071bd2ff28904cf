"""Tensor-parallel layout of the 7B hot path over `tp` ranks, one per GPU.

Attention is independent per kv head, so rank r owns kv heads
[r*HKV/tp, (r+1)*HKV/tp) and the query heads that share them.  qkv and gate_up
are column-parallel (each rank computes a block of their output rows: for qkv
the q, k and v rows of its heads); o and down are row-parallel (each rank
holds a block of their input dimension K and produces a partial of the full
output), followed by one allreduce (sum) of the [M, hidden] partials.

MXFP4 stores one e8m0 scale per 32 consecutive k and packs k pairs into bytes
(low nibble = even k), so a K split at a multiple of 32 is a plain column slice
of both the packed weight [N, K/2] and the scales [N, K/32]; the tensor-core
kernel additionally wants K % 256 per rank (true for the 7B shapes up to tp 8).
"""
import torch


def _check(n, tp, what):
    if n % tp:
        raise ValueError(f"{what} ({n}) is not divisible by tp={tp}")
    return n // tp


def col_shard(W, S, rank, tp):
    """Column-parallel: rows [rank*N/tp, (rank+1)*N/tp) of W [N, K/2] and of
    the transposed scales S [N, K/32]."""
    n = _check(W.shape[0], tp, "N")
    return W[rank * n:(rank + 1) * n], S[rank * n:(rank + 1) * n]


def row_shard(W, S, rank, tp):
    """Row-parallel: k in [rank*K/tp, (rank+1)*K/tp) -- byte columns of W and
    scale columns of S."""
    K = W.shape[1] * 2
    k = _check(K, tp, "K")
    if k % 32:
        raise ValueError(f"K/tp={k} must be a multiple of 32 (one scale per 32 k)")
    return (W[:, rank * k // 2:(rank + 1) * k // 2].contiguous(),
            S[:, rank * k // 32:(rank + 1) * k // 32].contiguous())


def qkv_rows(hq, hkv, d, rank, tp):
    """Output rows of the fused qkv projection ([q | k | v], head-major) owned
    by `rank`: its q heads, then its k heads, then its v heads."""
    q = _check(hq, tp, "query heads")
    kv = _check(hkv, tp, "kv heads")
    qr = torch.arange(rank * q * d, (rank + 1) * q * d)
    kr = hq * d + torch.arange(rank * kv * d, (rank + 1) * kv * d)
    vr = (hq + hkv) * d + torch.arange(rank * kv * d, (rank + 1) * kv * d)
    return torch.cat([qr, kr, vr])


def qkv_shard(W, S, hq, hkv, d, rank, tp):
    rows = qkv_rows(hq, hkv, d, rank, tp).to(W.device)
    return W.index_select(0, rows).contiguous(), S.index_select(0, rows).contiguous()


def kv_head_shard(cache, rank, tp):
    """Kv-head slice of a paged cache [NB, PBLK, HKV, D] (a strided view)."""
    h = _check(cache.shape[2], tp, "kv heads")
    return cache[:, :, rank * h:(rank + 1) * h, :]


def allreduce_(t, group=None):
    """In-place sum over the tensor-parallel group (NCCL on GPUs, gloo on CPU);
    a no-op for a single rank."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class PeerAllreduce:
    """The tensor-parallel allreduce on b200kv's one-shot kernel: every rank
    writes its partial into every rank's communication buffer over NVLink
    (CUDA IPC mappings of plain device memory, no multicast) and sums the tp
    partials in rank order, so all ranks get identical bytes.  Collective to
    construct (the IPC handles travel over the process group); all ranks must
    then make the same sequence of calls.  Capturable in CUDA graphs."""

    def __init__(self, group=None):
        import ctypes
        import torch.distributed as dist
        from _b200kv import check, lib
        self._lib, self._check, self._ct = lib, check, ctypes
        self.rank = dist.get_rank(group)
        self.tp = dist.get_world_size(group)
        # two buffer sets: the one-shot kernel's and the fused GEMV's (their
        # call counters count different things)
        owns, handles = [], []
        for _ in range(2):
            own = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            check(lib.b200kv_comm_alloc(ctypes.byref(own), handle), "b200kv_comm_alloc")
            owns.append(own.value)
            handles.append(bytes(handle))
        everyone = [None] * self.tp
        dist.all_gather_object(everyone, handles, group=group)
        self._peers, sets = [], []
        for k in range(2):
            ptrs = []
            for r in range(self.tp):
                if r == self.rank:
                    ptrs.append(owns[k])
                    continue
                p = ctypes.c_void_p()
                check(lib.b200kv_comm_open(everyone[r][k], ctypes.byref(p)), "b200kv_comm_open")
                ptrs.append(p.value)
                self._peers.append(p.value)
            sets.append((ctypes.c_void_p * self.tp)(*ptrs))
        self._owns = owns
        self._bufs, self._gemm_bufs = sets
        dist.barrier(group=group)

    def __call__(self, t):
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise TypeError("PeerAllreduce takes a contiguous bf16 tensor")
        self._check(self._lib.b200kv_allreduce_oneshot(
            t.data_ptr(), t.data_ptr(), t.numel(), self._bufs, self.rank, self.tp,
            torch.cuda.current_stream(t.device).cuda_stream), "b200kv_allreduce_oneshot")
        return t

    def gemm(self, x, weight, packed_scales, out):
        """out[M, N] = the sum over ranks of x @ dequant(weight)^T, the
        row-parallel MXFP4 product with the allreduce in its epilogue
        (b200kv_mxfp4_gemm_allreduce, M <= 8): bit for bit h4mv.mxfp4_gemm
        followed by this allreduce, in one launch."""
        M, K = x.shape
        N = weight.shape[0]
        if x.dtype != torch.bfloat16 or not x.is_contiguous() or out.shape != (M, N) or not out.is_contiguous():
            raise ValueError("gemm takes contiguous bf16 x [M, K] and out [M, N]")
        self._check(self._lib.b200kv_mxfp4_gemm_allreduce(
            weight.data_ptr(), packed_scales.data_ptr(), x.data_ptr(), out.data_ptr(), N, K, M,
            self._gemm_bufs, self.rank, self.tp, torch.cuda.current_stream(x.device).cuda_stream),
            "b200kv_mxfp4_gemm_allreduce")
        return out

    def close(self):
        """Unmap the peers' buffers and free this rank's; call after every rank
        has finished its last allreduce (e.g. after a barrier)."""
        for p in self._peers:
            self._lib.b200kv_comm_close(p)
        for p in self._owns:
            self._lib.b200kv_comm_free(p)
        self._peers, self._owns = [], []
