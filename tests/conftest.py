import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gfx1201-tuning-log_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")

for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def _ensure_library():
    so = os.path.join(PKG, "libb200kv.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", PKG, "-j4"], check=True, stdout=subprocess.DEVNULL)
    return so


@pytest.fixture(scope="session")
def libpath():
    return _ensure_library()


@pytest.fixture(scope="session")
def b200(libpath):
    import _b200kv
    return _b200kv


@pytest.fixture(scope="session")
def cuda(libpath):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, _ = torch.cuda.get_device_capability()
    assert major >= 10, "GPU tests need an sm_100 device"
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """Every GPU test must leave the library's device status word at 0: a
    kernel whose bounded wait ran out records a status there instead of
    hanging, and its outputs may still look right."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    import torch
    if not torch.cuda.is_available():
        yield
        return
    _ensure_library()
    import _b200kv
    torch.cuda.synchronize()
    _b200kv.reset_device_status()
    yield
    torch.cuda.synchronize()
    st = _b200kv.device_status()
    _b200kv.reset_device_status()
    assert st == 0, f"a kernel reported device status {st:#x} (a bounded wait ran out)"
