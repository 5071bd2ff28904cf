"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/b200kv.h declares, and rejects bad arguments with the documented status
codes before touching a device."""
import ctypes
import os
import re

import pytest
import torch

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "b200kv.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("defined",)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for must in ("b200kv_mxfp4_gemv", "h4mv_launch", "b200kv_decode_attn",
                 "b200kv_kv_write", "b200kv_status_string"):
        assert must in names


def test_library_exports_every_declared_symbol(libpath):
    lib = ctypes.CDLL(libpath)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings(b200):
    lib = b200.lib
    assert lib.b200kv_status_string(0) == b"ok"
    for code in range(1, 7):
        assert lib.b200kv_status_string(code) not in (b"ok", b"unknown status")
    assert lib.b200kv_status_string(99) == b"unknown status"
    assert lib.b200kv_version() >= 100


def test_gemv_argument_validation(b200):
    lib = b200.lib
    A = 0x10000  # never dereferenced: every call below fails validation first
    assert lib.b200kv_mxfp4_gemv(None, A, A, A, 8, 32, 1, None) == 1
    assert lib.b200kv_mxfp4_gemv(A, A, A, A, 0, 32, 1, None) == 1
    assert lib.b200kv_mxfp4_gemv(A, A, A, A, 8, 32, 9, None) == 2
    assert lib.b200kv_mxfp4_gemv(A, A, A, A, 8, 33, 1, None) == 2
    assert lib.b200kv_mxfp4_gemv(A + 8, A, A, A, 8, 32, 1, None) == 3
    assert lib.b200kv_mxfp4_gemv(A, A, A + 4, A, 8, 32, 1, None) == 3
    lib.h4mv_launch(A, A, A, A, 8, 32, 9, None)
    assert lib.b200kv_last_error() == 2


def test_wide_gemm_argument_validation(b200):
    lib = b200.lib
    A = 0x10000  # never dereferenced: every call below fails validation first
    need = lib.b200kv_mxfp4_gemm_wide_workspace_bytes(100, 1024)
    assert need == 2 * 128 * 1024 + 2 * 8 * 512
    assert lib.b200kv_mxfp4_gemm_wide_workspace_bytes(100, 1000) == 0
    assert lib.b200kv_mxfp4_gemm_wide(None, A, A, 1024, A, need, A, 8, 1024, 100, None) == 1
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A, 1000, A, need, A, 8, 1024, 100, None) == 1  # stride < K
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A, 1000, A, need, A, 8, 1000, 100, None) == 2  # K % 128
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A + 8, 1024, A, need, A, 8, 1024, 100, None) == 3
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A, 1028, A, need, A, 8, 1024, 100, None) == 3  # stride % 8
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A, 1024, A + 64, need, A, 8, 1024, 100, None) == 3
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A, 1024, A, need - 1, A, 8, 1024, 100, None) == 4
    assert lib.b200kv_mxfp4_gemm_wide(A, A, A, 1024, None, need, A, 8, 1024, 100, None) == 4


@pytest.mark.skipif(torch.cuda.is_available(), reason="fake pointers are only safe without a GPU")
def test_gemv_no_device(b200):
    A = 0x10000
    assert b200.lib.b200kv_mxfp4_gemv(A, A, A, A, 8, 32, 1, None) == 6


def _decode_call(lib, **over):
    A = 0x10000
    args = dict(q=A, qst=32 * 128, qsh=128, k=A, v=A, sk0=16 * 8 * 128, sk1=8 * 128, sk2=128,
                sv0=16 * 8 * 128, sv1=8 * 128, sv2=128, out=A, ost=32 * 128, osh=128,
                qsl=A, sl=A, bt=A, bts=4, ks=A, vs=A, sm=0.088, ns=2, hq=32, hkv=8, d=128,
                pblk=16, nblk=0, maxblk=4, hint=0, kvdt=0, obq=0, nsplit=0, st=None)
    args.update(over)
    a = args
    return lib.b200kv_decode_attn(a["q"], a["qst"], a["qsh"], a["k"], a["v"], a["sk0"], a["sk1"],
                                  a["sk2"], a["sv0"], a["sv1"], a["sv2"], a["out"], a["ost"],
                                  a["osh"], a["qsl"], a["sl"], a["bt"], a["bts"], a["ks"], a["vs"],
                                  a["sm"], a["ns"], a["hq"], a["hkv"], a["d"], a["pblk"],
                                  a["nblk"], a["maxblk"], a["hint"], a["kvdt"], a["obq"], a["nsplit"],
                                  a["st"])


def test_decode_argument_validation(b200):
    lib = b200.lib
    assert _decode_call(lib, q=None) == 1
    assert _decode_call(lib, d=64) == 2
    assert _decode_call(lib, hq=24) == 2           # GQA 3
    assert _decode_call(lib, hq=30) == 1           # not a multiple of HKV
    assert _decode_call(lib, kvdt=7) == 2
    assert _decode_call(lib, ks=None) == 1         # fp8 needs scales
    assert _decode_call(lib, nsplit=17) == 2       # more than 16 CTAs per cluster
    assert _decode_call(lib, sk1=8 * 128 + 1) == 3  # row not 16-B aligned
    assert _decode_call(lib, k=0x10008) == 3


def _mixed_call(lib, cu=0x10000, lens=0x10000, maxq=4, q=0x10000, hq=32, d=128, maxblk=8):
    A = 0x10000  # never dereferenced: every call below fails validation first
    return lib.b200kv_attn_varlen_mixed(q, 32 * 128, 128, A, A, 16 * 8 * 128, 8 * 128, 128,
                                        16 * 8 * 128, 8 * 128, 128, A, 32 * 128, 128, cu, lens, A, 8,
                                        A, A, 0.088, 2, maxq, 100, hq, 8, d, 16, 64, maxblk, 0, 16, None)


def test_mixed_attention_argument_validation(b200):
    """b200kv_attn_varlen_mixed needs the varlen form (cu_seqlens_q, seq_lens)
    and a positive max_qlen, then validates as the decode and prefill calls."""
    lib = b200.lib
    assert _mixed_call(lib, cu=None) == 1
    assert _mixed_call(lib, lens=None) == 1
    assert _mixed_call(lib, maxq=0) == 1
    assert _mixed_call(lib, q=None) == 1
    assert _mixed_call(lib, hq=24) == 2           # GQA 3
    assert _mixed_call(lib, d=64) == 2
    assert _mixed_call(lib, maxblk=0) == 1


@pytest.mark.skipif(torch.cuda.is_available(), reason="fake pointers are only safe without a GPU")
def test_decode_no_device(b200):
    assert _decode_call(b200.lib) == 6


def test_kv_write_argument_validation(b200):
    lib = b200.lib
    A = 0x10000

    def call(**o):
        a = dict(key=A, kst=1024, ksh=128, val=A, vst=1024, vsh=128, kc=A, vc=A, sk0=16384,
                 sk1=1024, sk2=128, sv0=16384, sv1=1024, sv2=128, slots=A, ks=A, vs=A, T=4,
                 hkv=8, d=128, pblk=16, dt=0)
        a.update(o)
        return lib.b200kv_kv_write(a["key"], a["kst"], a["ksh"], a["val"], a["vst"], a["vsh"],
                                   a["kc"], a["vc"], a["sk0"], a["sk1"], a["sk2"], a["sv0"],
                                   a["sv1"], a["sv2"], a["slots"], a["ks"], a["vs"], a["T"],
                                   a["hkv"], a["d"], a["pblk"], a["dt"], None)
    assert call(key=None) == 1
    assert call(d=24) == 2
    assert call(dt=5) == 2
    assert call(ks=None) == 1
    assert call(sk1=1000) == 3
    assert call(kst=1020) == 3


def test_allreduce_argument_validation(b200):
    lib = b200.lib
    bufs = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    A = 0x30000
    assert lib.b200kv_allreduce_oneshot(None, A, 4096, bufs, 0, 2, None) == 1
    assert lib.b200kv_allreduce_oneshot(A, A, 4096, bufs, 2, 2, None) == 1        # rank outside tp
    assert lib.b200kv_allreduce_oneshot(A, A, 4096, bufs, 0, 9, None) == 1        # more than 8 ranks
    assert lib.b200kv_allreduce_oneshot(A, A, 4100, bufs, 0, 2, None) == 2        # n % 8
    assert lib.b200kv_allreduce_oneshot(A, A, 8 * 4096 + 8, bufs, 0, 2, None) == 2
    assert lib.b200kv_allreduce_oneshot(A + 8, A, 4096, bufs, 0, 2, None) == 3    # 16-byte rule
    assert lib.b200kv_comm_buffer_bytes() > 2 * 8 * 8 * 4096 * 2
