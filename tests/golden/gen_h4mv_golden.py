"""Generate golden vectors by running the REFERENCE's own MXFP4 matvec kernel
h4mv_t<MT> (h4mv/h4mv.cu:43-104) on the CPU.

Run in a container that has the reference checkout:

    make -C oracle REF=/path/to/gfx1201-tuning-log    # -> oracle/_ref/libh4mv_ref.so
    python tests/golden/gen_h4mv_golden.py

oracle/Makefile compiles the kernel unmodified with g++ through a host
stand-in for <hip/hip_runtime.h> (oracle/h4mv_host/): threads as coroutines,
wave32 xor shuffles, the kernel's LDS byte LUT, its per-lane group partials,
its scale multiply and its round-half-up to bf16 all run as written; only its
inline v_dot2_f32_bf16 is replaced by a fused two-term dot product with one
rounding (stated in the stand-in header).

Output: tests/golden/h4mv_ref_cases.npz (small; committed): per case the
inputs W [N, K/2] u8, St [N, K/32] u8, X [M, K] bf16 bits and the kernel's
output bf16 bits [M, N].  Cases: config-2 data (codes uniform over the 16
values, scales 2^-8..2^-2, x ~ N(0, 1)) at K = 4096 and 14336 and M = 1, 4, 8
on row subsets of the 7B shapes (every row is computed independently), a
group count that is not a multiple of the wave (33 groups), the 32-position
one-hot probe of h4mv/h4mv_test.py:38-52, the structured full row of
w4-hip-demo/probe_w4hip.py:33-47 (x = k % 7 - 3, scale 2^0), and the edge
scale bytes 0 and 255.
"""
import ctypes
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import mxfp4_oracle as MO  # noqa: E402

LIB = os.path.join(ROOT, "oracle", "_ref", "libh4mv_ref.so")


def load_ref():
    lib = ctypes.CDLL(LIB)
    lib.h4mv_host_launch.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3
    lib.h4mv_host_launch.restype = ctypes.c_int
    return lib


def run_ref(lib, W, St, X):
    """Reference kernel on the host: W u8 [N, K/2], St u8 [N, K/32], X bf16 [M, K]
    -> bf16 bits [M, N]."""
    N, K, M = W.shape[0], W.shape[1] * 2, X.shape[0]
    Wn = np.ascontiguousarray(torch.as_tensor(W).numpy())
    Sn = np.ascontiguousarray(torch.as_tensor(St).numpy())
    Xn = np.ascontiguousarray(torch.as_tensor(X).contiguous().view(torch.int16).numpy())
    out = np.zeros((M, N), dtype=np.uint16)
    rc = lib.h4mv_host_launch(Wn.ctypes.data, Sn.ctypes.data, Xn.ctypes.data, out.ctypes.data, N, K, M)
    if rc != 0:
        raise RuntimeError(f"h4mv_host_launch failed ({rc})")
    return out


def cases():
    out = {}
    for name, (N, K) in (("qkv", (6144, 4096)), ("down", (4096, 14336))):
        for M in (1, 4, 8):
            W, S, St, X = MO.make_case(N, K, M, seed=100 + M + K)
            out[f"{name}_m{M}"] = (W[:8], St[:8], X)   # 8 rows of the shape
    W, S, St, X = MO.make_case(40, 1056, 5, seed=7)     # 33 groups: lanes 0 and 1 take two
    out["groups33_m5"] = (W, St, X)
    # one-hot probe (h4mv_test.py:38-52): weight 1.0 at k in every row, x = e_k
    N, K, M = 4, 32, 8
    for k in range(32):
        W = torch.zeros(N, K // 2, dtype=torch.uint8)
        W[:, k // 2] = 2 if k % 2 == 0 else (2 << 4)
        X = torch.zeros(M, K, dtype=torch.bfloat16)
        X[:, k] = 1.0
        out[f"onehot_k{k:02d}"] = (W, torch.full((N, 1), 127, dtype=torch.uint8), X)
    # structured full row (probe_w4hip.py:33-47): x = k % 7 - 3, scale 2^0
    g = torch.Generator().manual_seed(0)
    W = torch.randint(0, 256, (8, 2048), dtype=torch.uint8, generator=g)
    X = (torch.arange(4096, dtype=torch.float32).remainder(7) - 3).to(torch.bfloat16).view(1, -1)
    out["structured_row"] = (W, torch.full((8, 128), 127, dtype=torch.uint8), X)
    # the kernel's edge scale bytes: 0 -> 0.0, 255 -> inf (h4mv.cu:72)
    W, S, St, X = MO.make_case(16, 512, 2, seed=9)
    St = St.clone()
    St[3, 1] = 0
    St[5, :] = 0
    St[9, 2] = 255
    out["edge_scales_m2"] = (W, St, X)
    return out


def main():
    lib = load_ref()
    arrays = {}
    for name, (W, St, X) in cases().items():
        arrays[f"{name}/W"] = W.numpy()
        arrays[f"{name}/St"] = St.numpy()
        arrays[f"{name}/X"] = X.contiguous().view(torch.int16).numpy()
        arrays[f"{name}/out"] = run_ref(lib, W, St, X)
    path = os.path.join(HERE, "h4mv_ref_cases.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path}: {len(arrays) // 4} cases, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
