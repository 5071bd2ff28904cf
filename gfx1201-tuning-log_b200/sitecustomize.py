# Interpreter-start hook: put this directory on PYTHONPATH (where the reference
# used /opt/fp8kv, h4mv/serve-h4mv.sh:19) and Python imports this file, which
# loads the overrides in the reference's order (vllm-fp8kv/sitecustomize.py:1-24);
# each import is isolated so a missing piece never stops the others.
try:
    import fp8kv_override  # noqa: F401
except Exception:
    pass
try:
    import fp8kv_profhook  # noqa: F401
except Exception:
    pass
try:
    import fp8kv_w4patch  # noqa: F401  (the reference's dead-end prototype: not shipped)
except Exception:
    pass
try:
    import fp8kv_hipw4  # noqa: F401
except Exception:
    pass
try:
    import fp8kv_prof_prefill  # noqa: F401  (absent from the reference too)
except Exception:
    pass
try:
    import fp8kv_prefill  # noqa: F401
except Exception:
    pass
