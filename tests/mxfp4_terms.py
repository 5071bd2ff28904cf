"""Test helpers shared by the tensor-core MXFP4 kernel tests (M <= 8 and wide
batches): a CPU restatement of the kernels' two-term e4m3 activation split,
the one-rounding bound, and inputs whose fp32 sums are exact."""
import torch

import mxfp4_oracle as MO


def e4m3_terms_reference(x):
    """CPU restatement of the activation split of both tensor-core kernels: per
    32-element block two e4m3 terms, each with scale 2^(floor(log2 m) - 7) for
    the block maximum m of what is left (2^0 for an all-zero block), codes
    rounded to nearest even.  Returns the value the two terms represent."""
    r = x.double().reshape(x.shape[0], -1, 32).clone()
    total = torch.zeros_like(r)
    for _ in range(2):
        mx = r.abs().amax(-1, keepdim=True)
        s = torch.where(mx > 0, torch.exp2(torch.floor(torch.log2(mx.clamp(min=1e-300))) - 7),
                        torch.ones_like(mx))
        q = (r / s).float().to(torch.float8_e4m3fn).double() * s
        total += q
        r = r - q
    return total.view_as(x).float()


def within_one_rounding(Y, ref):
    """Every output within one bf16 rounding of the fp32 reference, plus 1e-6
    of the largest output (fp32 summation order).  Returns (ok, worst excess)."""
    tol = ref.abs() * 2.0 ** -8 + 1e-6 * ref.abs().max()
    return bool(((Y - ref).abs() <= tol).all()), float(((Y - ref).abs() - tol).max())


def integer_case(N, K, M, seed):
    """Weights uniform over the 16 codes with scale 2^0 and x integers in
    [-8, 8]: every product is a multiple of 1/2 and every partial sum is exact
    in fp32, so the bf16 result is unique.  Returns (W, St, X, ref)."""
    g = torch.Generator().manual_seed(seed)
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    St = torch.full((N, K // 32), 127, dtype=torch.uint8)
    X = torch.randint(-8, 9, (M, K), generator=g).to(torch.bfloat16)
    ref = (X.double() @ MO.dequant_weight(W, St.t().contiguous()).double().t()).to(torch.bfloat16)
    return W, St, X, ref.float()


def one_hot_weights(N, K):
    """Row n holds code 2 (1.0) at k = n, so out[m, n] = x[m, n] * scale."""
    W = torch.zeros(N, K // 2, dtype=torch.uint8)
    for n in range(min(N, K)):
        W[n, n // 2] = 2 if n % 2 == 0 else (2 << 4)
    return W


def wide_binade_x(M, K, lo, seed, hi=0):
    """bf16 values with random 8-bit significands and exponents in [lo, hi]."""
    g = torch.Generator().manual_seed(seed)
    mant = 1.0 + torch.randint(0, 128, (M, K), generator=g).float() / 128.0
    sign = torch.where(torch.rand(M, K, generator=g) < 0.5, -1.0, 1.0)
    return (sign * mant * torch.exp2(torch.randint(lo, hi + 1, (M, K), generator=g).float())).to(torch.bfloat16)
