"""Route small-M MXFP4 linears through the B200 matvec -- the drop-in for the
reference module h4mv/fp8kv_hipw4.py.

With FP8KV_HIPW4=1 the CUDA implementation of the op radiance::mxfp4_linear
(x, weight, weight_scale, wref) -> Tensor is replaced, as in the reference
(fp8kv_hipw4.py:14-99):

  * gate (fp8kv_hipw4.py:70-76): x 2-D, contiguous, bf16, 1 <= M <= MAX_M;
    K % 32 == 0; N >= 8; weight_scale rows == K/32; weight 16-byte aligned;
  * the checkpoint's scale layout [K/32, N] is repacked once and cached by
    (data_ptr, shape), never while a CUDA graph is being captured
    (fp8kv_hipw4.py:32-43): into tensor-core scale atoms for the block-scaled
    tcgen05 kernels (h4mv.mxfp4_gemm) when K % 128 == 0 and no scale byte is
    0 or 255, else into [N, K/32] for the CUDA-core kernel (h4mv.mxfp4_gemv);
    prepack() does this at load time (the reference's "P2 load-time repack",
    docs/06-w4gemm-hip-roadmap.md:54-55);
  * out = torch.empty(M, N, bf16) and one launch on the current stream;
  * everything else goes to the op's original CUDA body.

FP8KV_HIPW4_MAX_M keeps the reference's default of 4; the B200 kernel itself
handles M <= 8 (the reference capped at 4 because of a gfx1201 M=8 cliff).

Stock vLLM 0.22 has no caller of radiance::mxfp4_linear (the reference's fork
routed its MXFP4 linear method there); its Quark OCP-MX scheme runs W4A16
MXFP4 layers in emulation, whose dequantization needs the amd-quark package.
With FP8KV_HIPW4=1 install_quark_hook() therefore also hooks that scheme:
process_weights_after_loading keeps the scales in the op's [K/32, N] layout
and prepacks them, so a CUDA-graph capture of a freshly loaded model never
reaches the lazy repack, and apply_weights sends bf16 activations of those
layers through the op (other layers and dtypes keep the scheme's own path).

The reference stole the body of the radiance fork's op once that module
appeared (a 1500 x 0.2 s poll, fp8kv_hipw4.py:45-59).  The fork is not part
of this environment, so when `radiance_mxfp4` cannot be imported this module
defines the op schema itself; the original body is then `mxfp4_linear_chunked`,
which runs the wide-batch tensor-core GEMM (h4mv.mxfp4_gemm_wide, the
reference's dequant + matmul path for M > 8) or, for weights off the
tensor-core path, the B200 matvec over 8-row slices of x, so no shape falls
back to a CPU or Python implementation.
"""
import os
import sys
import threading

OP = "radiance::mxfp4_linear"
SCHEMA = "mxfp4_linear(Tensor x, Tensor weight, Tensor weight_scale, Tensor wref) -> Tensor"

_state = {"installed": False, "lib": None, "fast": 0, "slow": 0, "calls": 0, "logged": False}
_repack_cache = {}


def max_m():
    return int(os.environ.get("FP8KV_HIPW4_MAX_M", "4"))


def _capturing(t):
    import torch
    return t.is_cuda and torch.cuda.is_current_stream_capturing()


def scale_t_for(s):
    """weight_scale [K/32, N] -> [N, K/32] contiguous, cached by (data_ptr, shape);
    None while capturing a CUDA graph (no allocations or side launches then).
    The cache entry holds the source tensor too, so its address cannot be
    freed and handed to another tensor while the entry exists."""
    key = ("t", s.data_ptr(), tuple(s.shape), s.device)
    ent = _repack_cache.get(key)
    if ent is not None:
        return ent[1]
    if _capturing(s):
        return None
    st = s.t().contiguous()
    if len(_repack_cache) > 512:
        _repack_cache.clear()
    _repack_cache[key] = (s, st)
    return st


def packed_scales_for(s, N, K):
    """weight_scale [K/32, N] -> the tensor-core scale atoms (h4mv.pack_scales),
    cached like scale_t_for; False when the weight cannot take the
    tensor-core path (K % 128, or scale bytes 0 / 255), None during capture."""
    import h4mv
    key = ("p", s.data_ptr(), tuple(s.shape), s.device)
    ent = _repack_cache.get(key)
    if ent is not None:
        return ent[1]
    if _capturing(s):
        return None
    packed = False
    if K % 128 == 0:
        p, edge = h4mv.pack_scales(s.contiguous(), N, K, h4mv.SCALES_CHECKPOINT)
        packed = False if edge else p
    if len(_repack_cache) > 512:
        _repack_cache.clear()
    _repack_cache[key] = (s, packed)
    return packed


def prepack(weight, weight_scale):
    """Load-time repack of one MXFP4 weight (weight uint8 [N, K/2], weight_scale
    uint8 [K/32, N], the op's layout) into the caches the op reads: the
    tensor-core scale atoms, or the [N, K/32] transpose for weights off the
    tensor-core path.  Call outside CUDA-graph capture; returns True when the
    tensor-core atoms were packed."""
    N, K = weight.shape[0], weight.shape[1] * 2
    packed = packed_scales_for(weight_scale, N, K) if weight.data_ptr() % 16 == 0 else False
    if packed is False:
        scale_t_for(weight_scale)
    return packed is not None and packed is not False


QUARK_MODULE = "vllm.model_executor.layers.quantization.quark.schemes.quark_ocp_mx"


def _w4a16_mxfp4(scheme):
    """vLLM's Quark OCP-MX scheme with MXFP4 weights and unquantized activations."""
    return getattr(scheme, "weight_dtype", None) == "mxfp4" and getattr(scheme, "input_dtype", "") is None


def install_quark_hook():
    """Hook vLLM's QuarkOCP_MX for W4A16 MXFP4 layers (idempotent): the scales
    are kept in the op's [K/32, N] layout and prepacked when the weights are
    loaded, and bf16 activations go through radiance::mxfp4_linear.  Returns
    False when vLLM's scheme cannot be imported."""
    try:
        import importlib
        cls = importlib.import_module(QUARK_MODULE).QuarkOCP_MX
    except Exception:
        return False
    if getattr(cls, "_b200kv_hooked", False):
        return True
    orig_process, orig_apply = cls.process_weights_after_loading, cls.apply_weights

    def process_weights_after_loading(self, layer):
        orig_process(self, layer)
        if _w4a16_mxfp4(self) and layer.weight.is_cuda and layer.weight.dtype == __import__("torch").uint8:
            ws = layer.weight_scale.data
            K = layer.weight.shape[1] * 2
            ckpt = ws if ws.shape[0] == K // 32 else ws.t().contiguous()  # -> [K/32, N]
            layer._b200kv_scale_ckpt = ckpt
            prepack(layer.weight.data, ckpt)

    def apply_weights(self, layer, x, bias=None):
        import torch
        ckpt = getattr(layer, "_b200kv_scale_ckpt", None)
        if ckpt is not None and x.is_cuda and x.dtype == torch.bfloat16:
            w = layer.weight
            y = torch.ops.radiance.mxfp4_linear(x.reshape(-1, x.shape[-1]).contiguous(), w, ckpt, w)
            y = y.reshape(*x.shape[:-1], w.shape[0])
            return y + bias if bias is not None else y
        return orig_apply(self, layer, x, bias)

    cls.process_weights_after_loading = process_weights_after_loading
    cls.apply_weights = apply_weights
    cls._b200kv_hooked = True
    sys.stderr.write("[hipw4] quark W4A16 MXFP4 hook installed\n")
    return True


def eligible(x, weight, weight_scale, m_limit):
    """The reference's gate (fp8kv_hipw4.py:70-76)."""
    import torch
    if not (torch.is_tensor(x) and x.dim() == 2 and x.is_contiguous()
            and x.dtype == torch.bfloat16 and 1 <= x.shape[0] <= m_limit):
        return False
    N = weight.shape[0]
    K = weight.shape[1] * 2
    return (K % 32 == 0 and N >= 8 and weight_scale.shape[0] == K // 32
            and weight.data_ptr() % 16 == 0 and weight.dtype == torch.uint8)


def mxfp4_linear_chunked(x, weight, weight_scale, wref=None):
    """x [M, K] @ dequant(weight, weight_scale)^T for any M (weight_scale in
    the checkpoint layout): M > 8 on the wide-batch tensor-core GEMM when the
    weight's scales pack, else the B200 matvec on 8-row slices of x."""
    import torch

    import h4mv
    M = x.shape[0]
    N, K = weight.shape[0], weight.shape[1] * 2
    if M > h4mv.MAX_M and weight.data_ptr() % 16 == 0:
        packed = packed_scales_for(weight_scale, N, K)
        if packed is not None and packed is not False:
            return h4mv.mxfp4_gemm_wide(x.contiguous().to(torch.bfloat16), weight, packed)
    st = scale_t_for(weight_scale)
    if st is None:
        raise RuntimeError("mxfp4_linear: scale repack needed during CUDA graph capture; "
                           "run one eager call first")
    xc = x.contiguous().to(torch.bfloat16)
    out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
    for m0 in range(0, M, h4mv.MAX_M):
        h4mv.mxfp4_gemv(xc[m0:m0 + h4mv.MAX_M], weight, st, out=out[m0:m0 + h4mv.MAX_M])
    return out


def _define_op_if_missing(m_limit):
    """Define radiance::mxfp4_linear when the fork is absent, with the patched
    implementation over the chunked body as its CUDA kernel.  Returns False
    when the op already exists."""
    import torch
    try:
        torch.ops.radiance.mxfp4_linear
        return False
    except (AttributeError, RuntimeError):
        pass
    lib = torch.library.Library("radiance", "DEF")
    lib.define(SCHEMA)
    lib.impl("mxfp4_linear", make_patched(mxfp4_linear_chunked, m_limit), "CUDA")

    def _meta(x, weight, weight_scale, wref):
        return x.new_empty((x.shape[0], weight.shape[0]), dtype=torch.bfloat16)
    lib.impl("mxfp4_linear", _meta, "Meta")
    _state["lib"] = lib
    _state["installed"] = True
    return True


def make_patched(body, m_limit):
    import torch

    import h4mv

    def _patched(x, weight, weight_scale, wref):
        try:
            if _state["calls"] < 3:
                _state["calls"] += 1
                sys.stderr.write(f"[hipw4] call#{_state['calls']} x={tuple(x.shape)}/{x.dtype}"
                                 f"/c={x.is_contiguous()} w={tuple(weight.shape)}/{weight.dtype}"
                                 f" s={tuple(weight_scale.shape)}"
                                 f" cap={_capturing(x)}\n")
            if eligible(x, weight, weight_scale, m_limit):
                N, K = weight.shape[0], weight.shape[1] * 2
                packed = packed_scales_for(weight_scale, N, K) if weight.data_ptr() % 16 == 0 else False
                if packed is not None and packed is not False:
                    out = h4mv.mxfp4_gemm(x, weight, packed)
                else:
                    st = scale_t_for(weight_scale) if packed is False else None
                    out = h4mv.mxfp4_gemv(x, weight, st) if st is not None else None
                if out is not None:
                    _state["fast"] += 1
                    if not _state["logged"]:
                        _state["logged"] = True
                        sys.stderr.write(f"[hipw4] ENGAGED N={weight.shape[0]} K={weight.shape[1] * 2} "
                                         f"M={x.shape[0]}\n")
                    return out
        except Exception as e:
            sys.stderr.write(f"[hipw4] fast path failed ({e!r}), falling back\n")
        _state["slow"] += 1
        return body(x, weight, weight_scale, wref)

    return _patched


def _override(body):
    import torch
    patched = make_patched(body, max_m())
    lib = torch.library.Library("radiance", "IMPL")
    lib.impl("mxfp4_linear", patched, "CUDA")
    _state["impl_lib"] = lib
    _state["installed"] = True
    sys.stderr.write("[hipw4] op impl overridden\n")


def _install():
    if os.environ.get("FP8KV_HIPW4", "0") != "1":
        return False
    if _state["installed"]:
        return True
    try:
        import torch  # noqa: F401

        import h4mv  # noqa: F401  (loads libb200kv.so: fail here, not on the first call)
    except Exception as e:
        sys.stderr.write(f"[hipw4] lib load fail: {e}\n")
        return False
    try:
        import radiance_mxfp4 as rm  # noqa: F401
        have_fork = True
    except Exception:
        have_fork = False
    if not have_fork:
        if _define_op_if_missing(max_m()):
            sys.stderr.write("[hipw4] installed (radiance op defined here)\n")
        else:
            _override(mxfp4_linear_chunked)
            sys.stderr.write("[hipw4] installed\n")
        install_quark_hook()
        return True

    def _poll():
        body = None
        for _ in range(1500):
            try:
                import radiance_mxfp4 as rm
                if getattr(rm, "WPERM", False):
                    sys.stderr.write("[hipw4] WPERM=1, standing down\n")
                    return
                f = rm.mxfp4_linear
                body = f._backend_fns.get("cuda") or f._init_fn
                break
            except Exception:
                import time
                time.sleep(0.2)
        if body is None:
            sys.stderr.write("[hipw4] radiance module never appeared\n")
            return
        _override(body)

    threading.Thread(target=_poll, daemon=True).start()
    sys.stderr.write("[hipw4] installed\n")
    return True


_install()
