"""The drop-in inside a running vLLM 0.22 engine: the reference's acceptance
check (its playbook greps `[fp8kv-override] ENGAGED` from a serving engine and
compares greedy outputs), here with vllm.LLM in a child process.

A tiny random-init Llama (2 layers, head_dim 128, 2 query heads on 1 kv head,
vocab 1024; its lm_head scaled up so greedy tokens are far from ties) is saved
to a temporary directory and served with kv_cache_dtype="fp8" on the Triton
attention backend, the package directory on PYTHONPATH so its sitecustomize
installs the overrides (FP8KV_OVERRIDE=1: decode batches on the split-K decode
kernel; FP8KV_PREFILL=1: prefill and mixed batches on the varlen kernel).
Checks: the ENGAGED line, and the patch's dispatch counters show both decode
and prefill batches on this package's kernels with no fallback after a failed
fast path; the same prompts twice in one engine give identical tokens; and
the greedy tokens equal those of the same engine with the overrides off
(vLLM's own Triton kernels, given the same bf16 queries) up to the first
step where the two differ, and that step is a near-tie of the baseline (its
top two log-probabilities within 1 nat, where this model's logits spread
over about ten): the kernels round P differently (f16 here, bf16 there), so
a near-tie may go either way, and after it the sequences part."""
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import PKG

pytestmark = pytest.mark.gpu

CHILD = r'''
import json, os, sys
if os.environ.get("ENGINE_TEST_BF16_QUERY") == "1":
    # the baseline run: vLLM's own kernel, with the bf16 queries the drop-in keeps
    # (vLLM on CUDA would otherwise quantise them to fp8 before an fp8-KV backend)
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl
    _orig_init = TritonAttentionImpl.__init__
    def _init(self, *a, **k):
        _orig_init(self, *a, **k)
        self.supports_quant_query_input = False
    TritonAttentionImpl.__init__ = _init
from vllm import LLM, SamplingParams
llm = LLM(model=sys.argv[1], skip_tokenizer_init=True, kv_cache_dtype="fp8", dtype="bfloat16",
          enforce_eager=True, gpu_memory_utilization=0.2, max_model_len=2048, max_num_seqs=8,
          attention_backend="TRITON_ATTN", seed=0)
prompts = [{"prompt_token_ids": [(7 * i + 3 * n) % 1000 + 5 for i in range(n)]} for n in (5, 300, 1200, 77)]
sp = SamplingParams(temperature=0.0, max_tokens=24, detokenize=False, logprobs=2)
runs, margins = [], None
for _ in range(2):
    outs = llm.generate(prompts, sp)
    runs.append([list(o.outputs[0].token_ids) for o in outs])
    # per step: log p(top 1) - log p(top 2), how far the greedy choice was from a tie
    margins = [[(lambda v: v[0] - v[1])(sorted((x.logprob for x in step.values()), reverse=True) + [-1e30])
                for step in o.outputs[0].logprobs] for o in outs]
counts = None
if "fp8kv_override" in sys.modules:  # the engine runs in this process: the patch's dispatch counters
    counts = dict(sys.modules["fp8kv_override"]._state.get("counts") or {})
if "fp8kv_hipw4" in sys.modules:  # radiance::mxfp4_linear calls: skinny kernel / wide-batch body
    st = sys.modules["fp8kv_hipw4"]._state
    counts = dict(counts or {}, mxfp4_fast=st.get("fast", 0), mxfp4_wide=st.get("slow", 0),
                  quark_hooked=bool(getattr(sys.modules.get(
                      "vllm.model_executor.layers.quantization.quark.schemes.quark_ocp_mx"), "QuarkOCP_MX",
                      None) and sys.modules["vllm.model_executor.layers.quantization.quark.schemes.quark_ocp_mx"]
                      .QuarkOCP_MX.__dict__.get("_b200kv_hooked", False)))
print("RESULT " + json.dumps({"runs": runs, "margins": margins, "counts": counts}), flush=True)
'''


def _model(path):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=128, max_position_embeddings=4096,
                      rms_norm_eps=1e-5, rope_theta=10000.0, tie_word_embeddings=False, torch_dtype="bfloat16")
    torch.manual_seed(0)
    m = LlamaForCausalLM(cfg).to(torch.bfloat16)
    with torch.no_grad():
        m.lm_head.weight.mul_(30.0)
    m.save_pretrained(path)


def _serve(model_dir, override, tmp_path, extra_env=None):
    env = dict(os.environ)
    env["PYTHONPATH"] = PKG + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    env.update({"FP8KV_OVERRIDE": "1" if override else "0", "FP8KV_PREFILL": "1" if override else "0",
                "ENGINE_TEST_BF16_QUERY": "0" if override else "1",
                "VLLM_ENABLE_V1_MULTIPROCESSING": "0", "VLLM_NO_USAGE_STATS": "1", "DO_NOT_TRACK": "1",
                "HF_HUB_OFFLINE": "1", "TRANSFORMERS_OFFLINE": "1"})
    env.update(extra_env or {})
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    r = subprocess.run([sys.executable, str(script), str(model_dir)], env=env, capture_output=True, text=True,
                       timeout=900)
    log = r.stdout + r.stderr
    assert r.returncode == 0, log[-4000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")]
    assert line, log[-4000:]
    return json.loads(line[-1][len("RESULT "):]), log


def test_engine_with_overrides(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    model_dir = tmp_path / "tiny-llama"
    _model(model_dir)
    res, log = _serve(model_dir, True, tmp_path)
    assert "[fp8kv-override] ENGAGED" in log, log[-4000:]
    assert "fast path failed" not in log, log[-4000:]
    counts = res["counts"]
    assert counts and counts["decode"] > 0 and counts["prefill"] > 0, counts
    runs = res["runs"]
    assert runs[0] == runs[1]  # deterministic across two generate calls
    base, base_log = _serve(model_dir, False, tmp_path)
    assert "[fp8kv-override] ENGAGED" not in base_log
    for ours, theirs, margin in zip(runs[0], base["runs"][0], base["margins"]):
        n = next((i for i, (a, b) in enumerate(zip(ours, theirs)) if a != b), None)
        if n is not None:
            assert margin[n] < 1.0, (n, ours, theirs, margin, counts)


# ---- an MXFP4 (Quark OCP-MX, W4A16) checkpoint through the load-time hook ----
LINEARS = {"self_attn.q_proj": (256, 256), "self_attn.k_proj": (128, 256), "self_attn.v_proj": (128, 256),
           "self_attn.o_proj": (256, 256), "mlp.gate_proj": (512, 256), "mlp.up_proj": (512, 256),
           "mlp.down_proj": (256, 512)}
QUARK_CONFIG = {
    "quant_method": "quark", "export": {"kv_cache_group": [], "pack_method": "reorder"},
    "exclude": ["lm_head"], "layer_quant_config": {}, "layer_type_quant_config": {},
    "global_quant_config": {"weight": {"dtype": "fp4", "qscheme": "per_group", "group_size": 32,
                                       "scale_format": "e8m0", "is_dynamic": False, "symmetric": None,
                                       "ch_axis": -1, "round_method": "half_even", "scale_type": "float"},
                            "input_tensors": None, "output_tensors": None, "bias": None},
}


def _quark_pair(tmp_path):
    """The same random MXFP4 weights twice: as a Quark OCP-MX checkpoint (uint8
    e2m1 codes [N, K/2], uint8 e8m0 scales [N, K/32]) and as a bf16 checkpoint of
    their exact dequantisation (e2m1 x 2^k with |k| small is exact in bf16)."""
    import json as _json

    from safetensors.torch import save_file

    import mxfp4_oracle as MO
    _model(tmp_path / "bf16")
    bf16_dir, quark_dir = tmp_path / "bf16", tmp_path / "quark"
    quark_dir.mkdir()
    from safetensors.torch import load_file
    sd = load_file(str(bf16_dir / "model.safetensors"))
    g = torch.Generator().manual_seed(11)
    qsd = {k: v for k, v in sd.items() if not any(f".{n}." in k for n in LINEARS)}
    for li in range(2):
        for name, (N, K) in LINEARS.items():
            W = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
            St = torch.randint(119, 124, (N, K // 32), dtype=torch.uint8, generator=g)
            key = f"model.layers.{li}.{name}"
            qsd[key + ".weight"] = W
            qsd[key + ".weight_scale"] = St
            sd[key + ".weight"] = MO.dequant_weight(W, St.t().contiguous()).to(torch.bfloat16)
    save_file(sd, str(bf16_dir / "model.safetensors"), metadata={"format": "pt"})
    save_file(qsd, str(quark_dir / "model.safetensors"), metadata={"format": "pt"})
    cfg = _json.loads((bf16_dir / "config.json").read_text())
    cfg["quantization_config"] = QUARK_CONFIG
    (quark_dir / "config.json").write_text(_json.dumps(cfg))
    (quark_dir / "generation_config.json").write_text((bf16_dir / "generation_config.json").read_text())
    return quark_dir, bf16_dir


def test_engine_quark_mxfp4_checkpoint(tmp_path):
    """A Quark OCP-MX W4A16 checkpoint served by vllm.LLM with FP8KV_HIPW4=1:
    vLLM's QuarkOCP_MX loads it, the hook packs each layer's scale atoms at load
    time and sends its bf16 activations through radiance::mxfp4_linear (the
    tensor-core MXFP4 kernels: the skinny one for decode, the wide GEMM for the
    prompt).  Greedy tokens equal those of the bf16 twin (the same weights
    dequantised, on vLLM's bf16 linear layers) up to the first step that is a
    near-tie of the twin (top two log-probabilities within 1 nat); the same
    prompts twice give identical tokens."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    quark_dir, bf16_dir = _quark_pair(tmp_path)
    res, log = _serve(quark_dir, True, tmp_path, {"FP8KV_HIPW4": "1", "FP8KV_HIPW4_MAX_M": "8"})
    counts = res["counts"]
    assert "[hipw4] quark W4A16 MXFP4 hook installed" in log, log[-4000:]
    assert "fast path failed" not in log, log[-4000:]
    assert counts["quark_hooked"] and counts["mxfp4_fast"] > 0 and counts["mxfp4_wide"] > 0, counts
    runs = res["runs"]
    assert runs[0] == runs[1]
    twin, _ = _serve(bf16_dir, True, tmp_path)
    for ours, theirs, margin in zip(runs[0], twin["runs"][0], twin["margins"]):
        n = next((i for i, (a, b) in enumerate(zip(ours, theirs)) if a != b), None)
        if n is not None:
            assert margin[n] < 1.0, (n, ours, theirs, margin, counts)
