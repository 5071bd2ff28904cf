"""Generate golden vectors by running the REFERENCE's own Triton kernels on CPU.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/gen_golden.py /path/to/gfx1201-tuning-log

The reference kernels (vllm-fp8kv/fp8kv_v3.py, fp8kv_kernel.py,
fp8kv_prefill.py) are imported from that checkout and executed with the Triton
interpreter (TRITON_INTERPRET=1) on CPU tensors.  Triton 3.6's interpreter
multiplies bfloat16 dot operands as raw uint16 bit patterns; the patch below
widens bf16 operands to fp32 first, which is what the GPU tensor-core dot does
(exact bf16 products, fp32 accumulation).  Nothing else in the reference
kernels is changed: the split/reduce structure, the bf16 rounding of P, the
scale folding and the block-table gather all run as written.

Output: tests/golden/ref_triton_cases.npz (small; committed).  The GPU test
suite and the CPU oracle tests replay these inputs.
"""
import importlib.util
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _patch_interpreter_bf16_dot():
    orig = _interp.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        def widen(h):
            if h.dtype.scalar == tl.bfloat16:
                data = _interp._convert_float(h.data, tl.bfloat16, tl.float32, None).view(np.float32)
                return _interp.TensorHandle(data, tl.float32)
            return h
        a2, b2 = widen(a), widen(b)
        if a2 is not a or b2 is not b:
            return _interp.TensorHandle(np.matmul(a2.data, b2.data, dtype=np.float32) + d.data,
                                        d.dtype.scalar)
        return orig(self, a, b, d, input_precision, max_num_imprecise_acc)

    _interp.InterpreterBuilder.create_dot = create_dot


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _quant(x):
    s = float(x.abs().max()) / 448.0
    return (x / s).to(torch.float8_e4m3fn), s


def _paged(g, nb, pblk, hkv, d, dtype):
    k = torch.randn(nb, pblk, hkv, d, generator=g)
    v = torch.randn(nb, pblk, hkv, d, generator=g)
    if dtype == torch.float8_e4m3fn:
        (kq, ks), (vq, vs) = _quant(k), _quant(v)
        return kq, vq, ks, vs
    return k.to(dtype), v.to(dtype), 1.0, 1.0


def _block_table(g, ns, lens, pblk, nb):
    nblk = [max(1, -(-L // pblk)) for L in lens]
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(ns, max(nblk), dtype=torch.int32)
    pos = 0
    for s in range(ns):
        bt[s, :nblk[s]] = perm[pos:pos + nblk[s]]
        pos += nblk[s]
    return bt


def _u(t):
    """Raw little-endian bits of a tensor as a numpy array (fp8 -> u8, bf16 -> u16)."""
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main(ref_root):
    _patch_interpreter_bf16_dot()
    v3 = _load(os.path.join(ref_root, "vllm-fp8kv", "fp8kv_v3.py"), "ref_fp8kv_v3")
    k1 = _load(os.path.join(ref_root, "vllm-fp8kv", "fp8kv_kernel.py"), "ref_fp8kv_kernel")
    pf = _load(os.path.join(ref_root, "vllm-fp8kv", "fp8kv_prefill.py"), "ref_fp8kv_prefill")
    out = {}
    pblk, d = 16, 128

    # ---- decode cases: (name, module, hq, hkv, lens, dtype, ks_mult, vs_mult, nsplit, qsl)
    dec = [
        ("dec_v3_gqa4_ragged", "v3", 8, 2, [37, 64, 1], torch.float8_e4m3fn, 0.5, 2.0, 4, None),
        ("dec_v3_h32_empty_splits", "v3", 32, 8, [5], torch.float8_e4m3fn, 1.0, 1.0, 8, None),
        ("dec_v3_gqa2", "v3", 4, 2, [20, 33], torch.float8_e4m3fn, 1.0, 1.0, 2, None),
        ("dec_v3_h32_ctx70", "v3", 32, 8, [70], torch.float8_e4m3fn, 1.0, 1.0, 8, None),
        ("dec_k1_bf16_qsl", "k1", 8, 2, [40, 17], torch.bfloat16, 1.0, 1.0, 0, [1, 3, 5]),
        ("dec_k1_fp8", "k1", 8, 2, [29, 48, 16], torch.float8_e4m3fn, 1.0, 1.0, 0, None),
    ]
    for i, (name, mod, hq, hkv, lens, dt, ksm, vsm, nsplit, qsl) in enumerate(dec):
        g = torch.Generator().manual_seed(1000 + i)
        ns = len(lens)
        nb = sum(max(1, -(-L // pblk)) for L in lens) + 1
        kc, vc, ks, vs = _paged(g, nb, pblk, hkv, d, dt)
        ks, vs = ks * ksm, vs * vsm
        bt = _block_table(g, ns, lens, pblk, nb)
        qsl_t = torch.arange(ns + 1, dtype=torch.int32) if qsl is None else torch.tensor(qsl, dtype=torch.int32)
        T = int(qsl_t[-1]) + 1 if qsl is not None else ns
        q = torch.randn(T, hq, d, generator=g).to(torch.bfloat16)
        slens = torch.tensor(lens, dtype=torch.int32)
        o = torch.zeros(T, hq, d, dtype=torch.bfloat16)
        kst = torch.tensor([ks], dtype=torch.float32)
        vst = torch.tensor([vs], dtype=torch.float32)
        if mod == "v3":
            v3.run(q, kc, vc, o, qsl_t, slens, bt, kst, vst, d ** -0.5, nsplit=nsplit)
        else:
            k1.run(q, kc, vc, o, qsl_t, slens, bt, kst, vst, d ** -0.5)
        out.update({f"{name}/q": _u(q), f"{name}/k": _u(kc), f"{name}/v": _u(vc),
                    f"{name}/qsl": qsl_t.numpy(), f"{name}/seq_lens": slens.numpy(),
                    f"{name}/bt": bt.numpy(), f"{name}/scales": np.array([ks, vs], np.float32),
                    f"{name}/out": _u(o),
                    f"{name}/meta": np.array([hq, hkv, 1 if mod == "k1" else 0,
                                              1 if dt == torch.bfloat16 else 0, nsplit], np.int32)})
        print(name, "done")

    # ---- prefill cases (single sequence, block_table row 0): (name, hq, hkv, q0, qlen, ksm, vsm)
    pre = [
        ("pre_first_chunk", 8, 2, 0, 48, 1.0, 1.0),
        ("pre_continuation_scaled", 8, 2, 50, 20, 0.5, 2.0),
        ("pre_h32_tail", 32, 8, 33, 17, 1.0, 1.0),
    ]
    for i, (name, hq, hkv, q0, qlen, ksm, vsm) in enumerate(pre):
        g = torch.Generator().manual_seed(2000 + i)
        ctx = q0 + qlen
        nb = -(-ctx // pblk) + 1
        kc, vc, ks, vs = _paged(g, nb, pblk, hkv, d, torch.float8_e4m3fn)
        ks, vs = ks * ksm, vs * vsm
        bt = _block_table(g, 1, [ctx], pblk, nb)
        q = torch.randn(qlen, hq, d, generator=g).to(torch.bfloat16)
        o = torch.zeros(qlen, hq, d, dtype=torch.bfloat16)
        pf.run(q, kc, vc, o, bt, torch.tensor([ks]), torch.tensor([vs]), d ** -0.5, q0, qlen)
        out.update({f"{name}/q": _u(q), f"{name}/k": _u(kc), f"{name}/v": _u(vc),
                    f"{name}/bt": bt.numpy(), f"{name}/scales": np.array([ks, vs], np.float32),
                    f"{name}/out": _u(o), f"{name}/meta": np.array([hq, hkv, q0, qlen], np.int32)})
        print(name, "done")

    path = os.path.join(HERE, "ref_triton_cases.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: gen_golden.py <reference checkout>")
    main(sys.argv[1])
