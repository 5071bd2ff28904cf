"""ORACLE -- test infrastructure, not product code.

CPU restatement of the reference's MXFP4 W4A16 matvec checker and codecs.  Only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
legs may import this module, and only as the checker or the timed CPU
baseline; the product path (libb200kv.so) never calls it.

Follows:
  * h4mv/h4mv_test.py:16-17  E2M1 value table
  * h4mv/h4mv_test.py:19-32  reference(): LUT dequant, exp2(S-127) group scale,
                             chunked fp32 matmul (device parameterised here)
  * h4mv/h4mv.cu:33-41       e2m1 bit decode (zero iff (v & 7) == 0, subnormal 0.5)
  * h4mv/h4mv.cu:72          kernel's scale: fp32 bit pattern (b << 23), so that
                             b == 0 gives 0.0 and b == 255 gives +inf
  * h4mv/h4mv.cu:43-104      h4mv_kernel_order_reference(): the reference
                             kernel's own order of operations (per-lane group
                             partials, scale multiply, wave32 xor reduction,
                             round-half-up to bf16), bit for bit
Pinned by the reference's own known-answer tests (one-hot probes,
h4mv/h4mv_test.py:38-52 and w4-hip-demo/probe_w4hip.py:13-47), restated in
tests/test_oracle_pins.py, by exhaustive codec tables (tests/test_codecs.py)
checked against the reference's E2M1 table and torch's float8_e8m0fnu dtype,
and by outputs of the reference kernel itself compiled for the CPU
(oracle/Makefile -> oracle/_ref/libh4mv_ref.so; committed as
tests/golden/h4mv_ref_cases.npz by tests/golden/gen_h4mv_golden.py).
"""
import numpy as np
import torch

# h4mv/h4mv_test.py:16-17
E2M1_LUT = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
            -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def e2m1_decode_bits(code):
    """e2m1 code (0..15) -> float, from the bit fields (h4mv/h4mv.cu:33-41)."""
    code = int(code)
    s, e, m = code >> 3, (code >> 1) & 3, code & 1
    if code & 7 == 0:
        mag = 0.0
    elif e == 0:
        mag = 0.5 * m                  # subnormal: 0.5 = 1.0 * 2^-1
    else:
        mag = (1.0 + 0.5 * m) * 2.0 ** (e - 1)
    return -mag if s else mag


def e8m0_exp2(b):
    """Scale of h4mv_test.reference: 2^(b-127) for every byte (b=255 -> inf)."""
    with np.errstate(over="ignore"):
        return np.exp2(np.asarray(b, dtype=np.float64) - 127.0).astype(np.float32)


def e8m0_bits(b):
    """Scale of the reference kernel (h4mv.cu:72): fp32 with bits (b << 23)."""
    b = np.asarray(b, dtype=np.uint32)
    return (b << np.uint32(23)).view(np.float32)


def dequant_weight(W, S, scale_mode="exp2"):
    """W uint8 [N, K/2], S uint8 [K/32, N] (checkpoint layout) -> fp32 [N, K]."""
    W = torch.as_tensor(W)
    S = torch.as_tensor(S)
    N, KW = W.shape
    K = KW * 2
    lut = torch.tensor(E2M1_LUT, dtype=torch.float32)
    w = torch.empty(N, K, dtype=torch.float32)
    w[:, 0::2] = lut[(W & 0xF).long()]
    w[:, 1::2] = lut[(W >> 4).long()]
    s_np = S.numpy().T  # [N, K/32]
    sc = e8m0_exp2(s_np) if scale_mode == "exp2" else e8m0_bits(s_np)
    sc = torch.from_numpy(np.ascontiguousarray(sc))
    return (w.view(N, K // 32, 32) * sc.view(N, K // 32, 1)).view(N, K)


def mxfp4_linear_reference(W, S, X, chunk=2048, scale_mode="exp2"):
    """fp32 result of x @ dequant(W, S)^T (h4mv/h4mv_test.py:19-32).

    W uint8 [N, K/2]; S uint8 [K/32, N]; X bf16/fp32 [M, K].  CPU tensors.
    scale_mode "exp2" follows the test reference, "bits" the kernel (h4mv.cu:72).
    The per-group structure (scale applied to the group's partial sum) is
    mathematically identical to scaling the dequantised weights.
    """
    W = torch.as_tensor(W).cpu()
    S = torch.as_tensor(S).cpu()
    X = torch.as_tensor(X).cpu()
    N, KW = W.shape
    K = KW * 2
    M = X.shape[0]
    xf = X.float()
    out = torch.empty(M, N, dtype=torch.float32)
    for r0 in range(0, N, chunk):
        r1 = min(r0 + chunk, N)
        ws = dequant_weight(W[r0:r1], S[:, r0:r1], scale_mode)
        out[:, r0:r1] = xf @ ws.t()
    return out


def rel_to_max_err(y, ref):
    """max |y - ref| / max |ref| (h4mv/h4mv_test.py:74)."""
    y = torch.as_tensor(y).float()
    ref = torch.as_tensor(ref).float()
    return ((y - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def make_case(N, K, M, seed, s_lo=119, s_hi=126):
    """Config-2 synthetic inputs: uniform W bytes (both nibbles uniform over the
    16 codes), e8m0 scales uniform in [s_lo, s_hi) i.e. 2^-8..2^-2, x ~ N(0,1)
    bf16.  Returns (W [N,K/2], S [K/32,N], St [N,K/32], X [M,K]) CPU tensors."""
    g = torch.Generator().manual_seed(seed)
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    S = torch.randint(s_lo, s_hi, (K // 32, N), dtype=torch.uint8, generator=g)
    X = torch.randn(M, K, generator=g).to(torch.bfloat16)
    return W, S, S.t().contiguous(), X


def h4mv_kernel_order_reference(W, St, X):
    """bf16 output of the reference kernel h4mv_t<MT> (h4mv/h4mv.cu:43-104) in
    its own order of operations, as uint16 bits [M, N]:
      * lane l (of a 32-wide wave per output row) takes groups g = l, l+32, ...
        (h4mv.cu:68); per group, part = sum over the 16 weight bytes in order of
        dot2(w pair, x pair, part) -- two exact products and the fp32 running
        value summed and rounded once (the fused dot2 model of
        oracle/h4mv_host/hip/hip_runtime.h) -- then acc += part * 2^(b-127)
        with the scale as fp32 bits b << 23 (h4mv.cu:72,90);
      * the 32 lane sums are reduced by xor shuffles 16, 8, 4, 2, 1 (h4mv.cu:96-97);
      * lane 0 rounds fp32 -> bf16 as (f >> 16) + ((f >> 15) & 1), i.e. ties
        away from zero (h4mv.cu:101).
    W uint8 [N, K/2], St uint8 [N, K/32] (transposed scales), X bf16 [M, K]."""
    W = np.asarray(torch.as_tensor(W).cpu().numpy(), dtype=np.uint8)
    St = np.asarray(torch.as_tensor(St).cpu().numpy(), dtype=np.uint8)
    xf = torch.as_tensor(X).cpu().float().numpy().astype(np.float64)  # bf16 values, exact
    N, KW = W.shape
    K = 2 * KW
    M = xf.shape[0]
    ngrp = K // 32
    lut = np.array(E2M1_LUT, dtype=np.float64)
    w = np.empty((N, K), dtype=np.float64)
    w[:, 0::2] = lut[W & 0xF]
    w[:, 1::2] = lut[W >> 4]
    sc = e8m0_bits(St)                                    # [N, ngrp] fp32
    lanes = np.arange(32)
    acc = np.zeros((N, 32, M), dtype=np.float32)
    for gi in range(-(-ngrp // 32)):
        g = gi * 32 + lanes                               # group of each lane
        valid = g < ngrp
        gc = np.where(valid, g, 0)
        part = np.zeros((N, 32, M), dtype=np.float32)
        for i in range(16):                               # the 16 weight bytes of a group
            k0 = 32 * gc + 2 * i
            p0 = w[:, k0][:, :, None] * xf[:, k0].T[None, :, :]
            p1 = w[:, k0 + 1][:, :, None] * xf[:, k0 + 1].T[None, :, :]
            part = ((p0 + p1) + part.astype(np.float64)).astype(np.float32)
        with np.errstate(over="ignore", invalid="ignore"):
            term = (part * sc[:, gc][:, :, None]).astype(np.float32)
            acc = np.where(valid[None, :, None], (acc + term).astype(np.float32), acc)
    v = acc
    with np.errstate(over="ignore", invalid="ignore"):
        for off in (16, 8, 4, 2, 1):
            v = (v + v[:, lanes ^ off, :]).astype(np.float32)
    f = v[:, 0, :].T.copy().view(np.uint32)              # [M, N]
    return ((f >> np.uint32(16)) + ((f >> np.uint32(15)) & np.uint32(1))).astype(np.uint16)


def bf16_bits_to_float(bits):
    """uint16 bf16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint32) << np.uint32(16)).view(np.float32)
