"""Pins the CPU oracle (CPU-only tests).

1. Attention: the oracle against the REFERENCE's own Triton kernels executed on
   CPU by the Triton interpreter (fixtures from tests/golden/gen_golden.py).
   Tolerance: the reference's own test bound, max abs < 0.05
   (vllm-fp8kv/fp8kv_v3.py:168, prefill_test.py:49), and rel-to-max < 2e-2.
2. MXFP4: the reference's known-answer tests, restated -- the 32-position
   one-hot probe at M=8 (h4mv/h4mv_test.py:38-52) and the structured full-row
   check with x = arange % 7 - 3 (w4-hip-demo/probe_w4hip.py:33-47).
"""
import os

import numpy as np
import pytest
import torch

import fp8kv_oracle as FO
import mxfp4_oracle as MO

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_triton_cases.npz")


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def _fp8(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)


def load_golden_cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    cases = {}
    for n in names:
        c = {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")}
        cases[n] = c
    return cases


def golden_decode_inputs(c):
    hq, hkv, k1, isbf, nsplit = (int(x) for x in c["meta"])
    kv = _bf16 if isbf else _fp8
    return dict(q=_bf16(c["q"]), k_cache=kv(c["k"]), v_cache=kv(c["v"]),
                qsl=torch.from_numpy(c["qsl"]), seq_lens=torch.from_numpy(c["seq_lens"]),
                block_table=torch.from_numpy(c["bt"]), k_scale=float(c["scales"][0]),
                v_scale=float(c["scales"][1]), sm_scale=128 ** -0.5,
                out_by_qsl=bool(k1), nsplit=nsplit)


def golden_prefill_inputs(c):
    hq, hkv, q0, qlen = (int(x) for x in c["meta"])
    return dict(q=_bf16(c["q"]), k_cache=_fp8(c["k"]), v_cache=_fp8(c["v"]),
                block_table=torch.from_numpy(c["bt"]), k_scale=float(c["scales"][0]),
                v_scale=float(c["scales"][1]), sm_scale=128 ** -0.5, q0=q0, qlen=qlen)


CASES = load_golden_cases()
DEC = [n for n in CASES if n.startswith("dec")]
PRE = [n for n in CASES if n.startswith("pre")]


@pytest.mark.parametrize("name", DEC)
def test_decode_oracle_matches_reference_kernel(name):
    c = CASES[name]
    a = golden_decode_inputs(c)
    ref = FO.decode_reference(a["q"], a["k_cache"], a["v_cache"], a["qsl"], a["seq_lens"],
                              a["block_table"], a["k_scale"], a["v_scale"], a["sm_scale"],
                              out_by_qsl=a["out_by_qsl"], out_rows=a["q"].shape[0])
    got = _bf16(c["out"]).float()
    rows = a["qsl"][:-1].long() if a["out_by_qsl"] else torch.arange(a["seq_lens"].numel())
    err = (got[rows] - ref[rows]).abs().max().item()
    assert err < 0.05, err
    assert err / ref[rows].abs().max().item() < 2e-2


@pytest.mark.parametrize("name", PRE)
def test_prefill_oracle_matches_reference_kernel(name):
    c = CASES[name]
    a = golden_prefill_inputs(c)
    cu = torch.tensor([0, a["qlen"]], dtype=torch.int32)
    lens = torch.tensor([a["q0"] + a["qlen"]], dtype=torch.int32)
    ref = FO.prefill_reference(a["q"], a["k_cache"], a["v_cache"], cu, lens, a["block_table"],
                               a["k_scale"], a["v_scale"], a["sm_scale"])
    got = _bf16(c["out"]).float()
    err = (got - ref).abs().max().item()
    assert err < 0.05, err
    assert err / ref.abs().max().item() < 2e-2


def test_gemv_oracle_one_hot_probe():
    # h4mv/h4mv_test.py:38-52: weight code 2 (= 1.0) at one k, x one-hot, scale 127
    N, K, M = 4, 32, 8
    S = torch.full((K // 32, N), 127, dtype=torch.uint8)
    for k in range(32):
        W = torch.zeros(N, K // 2, dtype=torch.uint8)
        W[:, k // 2] = 2 if k % 2 == 0 else (2 << 4)
        X = torch.zeros(M, K, dtype=torch.bfloat16)
        X[:, k] = 1.0
        Y = MO.mxfp4_linear_reference(W, S, X)
        assert torch.equal(Y, torch.ones(M, N)), k


def test_gemv_oracle_structured_row():
    # w4-hip-demo/probe_w4hip.py:33-47: N=8, K=4096, S=127, x = arange % 7 - 3
    g = torch.Generator().manual_seed(0)
    N, K = 8, 4096
    W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    S = torch.full((K // 32, N), 127, dtype=torch.uint8)
    X = (torch.arange(K, dtype=torch.float32) % 7 - 3).to(torch.bfloat16).view(1, K)
    lut = np.array(MO.E2M1_LUT, dtype=np.float64)
    w = np.empty((N, K))
    w[:, 0::2] = lut[(W.numpy() & 0xF)]
    w[:, 1::2] = lut[(W.numpy() >> 4)]
    exact = w @ X.double().numpy()[0]            # small integers / halves: exact
    Y = MO.mxfp4_linear_reference(W, S, X)[0].double().numpy()
    np.testing.assert_array_equal(Y, exact)


def test_gemv_oracle_scale_modes():
    W, S, St, X = MO.make_case(64, 256, 3, seed=5)
    a = MO.mxfp4_linear_reference(W, S, X, scale_mode="exp2")
    b = MO.mxfp4_linear_reference(W, S, X, scale_mode="bits")
    assert torch.equal(a, b)  # identical away from the 0 / 255 edge codes
    S0 = S.clone()
    S0[0, 0] = 0
    c = MO.mxfp4_linear_reference(W, S0, X, scale_mode="bits")
    d = MO.mxfp4_linear_reference(W[0:1, :16], S0[:1, :1], X[:, :32], scale_mode="bits")
    assert torch.all(d == 0) and torch.isfinite(c).all()


# ---- MXFP4: outputs of the reference kernel itself ----------------------------------
# tests/golden/h4mv_ref_cases.npz holds outputs of h4mv_t<MT> (h4mv/h4mv.cu:43-104)
# compiled for the CPU (oracle/Makefile, tests/golden/gen_h4mv_golden.py).
H4MV_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "h4mv_ref_cases.npz")
H4MV_REF_LIB = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libh4mv_ref.so")


def _h4mv_cases():
    z = np.load(H4MV_GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    return {n: (z[n + "/W"], z[n + "/St"], _bf16(z[n + "/X"]), z[n + "/out"]) for n in names}


H4MV = _h4mv_cases()


@pytest.mark.parametrize("name", sorted(H4MV))
def test_kernel_order_oracle_matches_reference_kernel_outputs(name):
    """The restatement of the reference kernel's order of operations gives its
    outputs bit for bit (every case, edge scale bytes 0 and 255 included)."""
    W, St, X, out = H4MV[name]
    assert np.array_equal(MO.h4mv_kernel_order_reference(W, St, X), out)


@pytest.mark.parametrize("name", sorted(n for n in H4MV if not n.startswith("edge")))
def test_checker_oracle_within_one_rounding_of_reference_kernel(name):
    """The fp32 oracle every GPU test checks against (h4mv_test.py:19-32) is within
    one bf16 rounding of the reference kernel's outputs: they differ only in fp32
    summation order and in the final rounding (the kernel rounds ties away from
    zero, torch to even)."""
    W, St, X, out = H4MV[name]
    S = torch.from_numpy(St).t().contiguous()
    ref = MO.mxfp4_linear_reference(torch.from_numpy(W), S, X, scale_mode="bits").numpy()
    got = MO.bf16_bits_to_float(out)
    tol = np.abs(ref) * 2.0 ** -8 + 1e-6 * np.abs(ref).max()
    assert bool((np.abs(got - ref) <= tol).all())


def test_reference_kernel_one_hot_and_structured_row():
    """The known-answer probes, answered by the reference kernel itself: every
    one-hot position gives exactly 1.0 for all M = 8 rows (h4mv_test.py:38-52),
    and the structured row equals the exact integer dot product
    (probe_w4hip.py:33-47: small integers, every sum exact in fp32)."""
    for k in range(32):
        W, St, X, out = H4MV[f"onehot_k{k:02d}"]
        assert bool((MO.bf16_bits_to_float(out) == 1.0).all()), k
    W, St, X, out = H4MV["structured_row"]
    exact = MO.mxfp4_linear_reference(torch.from_numpy(W), torch.from_numpy(St).t().contiguous(), X)
    assert np.array_equal(MO.bf16_bits_to_float(out), exact.to(torch.bfloat16).float().numpy())


def _load_h4mv_ref():
    import ctypes
    import subprocess
    if not os.path.exists(H4MV_REF_LIB):
        ref = os.environ.get("B200KV_REFERENCE", "/root/reference")
        if not os.path.exists(os.path.join(ref, "h4mv", "h4mv.cu")):
            pytest.skip("reference checkout absent and oracle/_ref not built")
        subprocess.run(["make", "-C", os.path.dirname(os.path.dirname(H4MV_REF_LIB)), f"REF={ref}"],
                       check=True, stdout=subprocess.DEVNULL)
    lib = ctypes.CDLL(H4MV_REF_LIB)
    lib.h4mv_host_launch.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3
    lib.h4mv_host_launch.restype = ctypes.c_int
    return lib


@pytest.mark.parametrize("N,K,M,seed", [(12, 4096, 1, 1), (9, 14336, 8, 2), (33, 2048, 3, 3), (7, 1056, 6, 4)])
def test_reference_kernel_host_build_matches_kernel_order_oracle(N, K, M, seed):
    """Fresh inputs through the reference kernel's host build (oracle/_ref) and
    the kernel-order restatement: identical bits."""
    lib = _load_h4mv_ref()
    W, S, St, X = MO.make_case(N, K, M, seed=seed)
    out = np.zeros((M, N), dtype=np.uint16)
    Xn = np.ascontiguousarray(X.view(torch.int16).numpy())
    Wn, Sn = np.ascontiguousarray(W.numpy()), np.ascontiguousarray(St.numpy())
    assert lib.h4mv_host_launch(Wn.ctypes.data, Sn.ctypes.data, Xn.ctypes.data, out.ctypes.data, N, K, M) == 0
    assert np.array_equal(MO.h4mv_kernel_order_reference(W, St, X), out)
