import os
import sys

import pytest

# torch first: libiq.so links libnccl.so.2, and whichever NCCL is loaded first is
# the one the process keeps; torch's CUDA library needs the NCCL it ships with,
# so it must load before anything pulls in libiq.so (e.g. the drop-in shim build)
try:
    import torch  # noqa: F401
except Exception:
    pass

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "int-llm_b200", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libiq.so)")
    config.addinivalue_line("markers", "slow: long CPU oracle run")


def pytest_collection_modifyitems(config, items):
    # gpu tests are skipped (not failed) when no CUDA device is visible
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
