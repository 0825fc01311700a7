import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

CACHE = os.environ.get("DCB_TEST_CACHE", "/tmp/demucs_b200_test_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no sm_100 GPU in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def rel_l2(got, ref):
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    den = np.linalg.norm(ref)
    num = np.linalg.norm(got - ref)
    return float(num / den) if den > 0 else float(num)


def model_files(name: str, layer_scale=0.3, seed=1):
    """Seeded synthetic weights for one of demucs_cuda_b200.synth's configurations."""
    from demucs_cuda_b200 import synth
    cfg = {"tiny": synth.TINY, "short": synth.SHORT, "full": synth.FULL}[name]
    d = os.path.join(CACHE, f"{name}_s{seed}_ls{layer_scale}")
    w, c = synth.write_model(d, cfg, seed=seed, layer_scale=layer_scale)
    return cfg, w, c


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    from demucs_cuda_b200 import require_gpu
    require_gpu()
    return torch
