"""In-engine profiler window -- the counterpart of the reference's
profiling/fp8kv_profhook.py.

When FP8KV_PROF_OUT is set, EngineCore.step (and step_with_batch_queue) is
wrapped so that steps FP8KV_PROF_START .. +FP8KV_PROF_STEPS run under
torch.profiler; the key_averages table (CUDA time) and the total device-busy
time are written to FP8KV_PROF_OUT (reference fp8kv_profhook.py:5,21-57).  The
hook polls for vLLM's EngineCore the way the reference does, because
sitecustomize runs before vLLM is imported.
"""
import os
import sys
import threading
import time

_state = {"step": 0, "prof": None, "done": False}


def _config():
    return (int(os.environ.get("FP8KV_PROF_START", "20")),
            int(os.environ.get("FP8KV_PROF_STEPS", "20")),
            os.environ.get("FP8KV_PROF_OUT"))


def wrap_step(fn, start, steps, out_path):
    """Return fn wrapped with the profiler window (exposed for tests)."""
    def wrapped(*a, **kw):
        import torch
        i = _state["step"]
        _state["step"] += 1
        if i == start and not _state["done"]:
            _state["prof"] = torch.profiler.profile(
                activities=[torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA])
            _state["prof"].__enter__()
        r = fn(*a, **kw)
        if i == start + steps - 1 and _state["prof"] is not None:
            p = _state["prof"]
            p.__exit__(None, None, None)
            _state["prof"] = None
            _state["done"] = True
            ka = p.key_averages()
            busy = sum(e.self_device_time_total for e in ka) / 1e3
            with open(out_path, "w") as f:
                f.write(ka.table(sort_by="self_cuda_time_total", row_limit=40))
                f.write(f"\nsteps={steps} device_busy_ms={busy:.3f} per_step_ms={busy / steps:.3f}\n")
            sys.stderr.write(f"[fp8kv-prof] wrote {out_path}\n")
        return r
    return wrapped


def _install():
    start, steps, out = _config()
    if not out:
        return False

    def _poll():
        for _ in range(3000):
            try:
                from vllm.v1.engine.core import EngineCore
                for name in ("step", "step_with_batch_queue"):
                    if hasattr(EngineCore, name):
                        setattr(EngineCore, name, wrap_step(getattr(EngineCore, name), start, steps, out))
                sys.stderr.write("[fp8kv-prof] hooked EngineCore\n")
                return
            except Exception:
                time.sleep(0.1)

    threading.Thread(target=_poll, daemon=True).start()
    return True


_install()
