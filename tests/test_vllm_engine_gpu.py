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


def _serve(model_dir, override, tmp_path):
    env = dict(os.environ)
    env["PYTHONPATH"] = PKG + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    env.update({"FP8KV_OVERRIDE": "1" if override else "0", "FP8KV_PREFILL": "1" if override else "0",
                "ENGINE_TEST_BF16_QUERY": "0" if override else "1",
                "VLLM_ENABLE_V1_MULTIPROCESSING": "0", "VLLM_NO_USAGE_STATS": "1", "DO_NOT_TRACK": "1",
                "HF_HUB_OFFLINE": "1", "TRANSFORMERS_OFFLINE": "1"})
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
