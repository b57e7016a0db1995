import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="module", params=["kq", "lane"])
def gemv_ctx(request):
    """A context whose batch-1 Q4_K / Q5_K / Q6_K matmuls take the tensor-core GEMV at every
    launch size ("kq") or always the lane GEMV ("lane"); by default the library picks by
    launch size, so both kernels are exercised on the small test shapes this way. The
    library reads these settings when the context is created."""
    import torch
    import rust_interference_engine_b200 as rie
    keys = ("RIE_GEMV_KQ", "RIE_GEMV_KQ_MIN_MB")
    old = {k: os.environ.get(k) for k in keys}
    os.environ["RIE_GEMV_KQ"] = "1" if request.param == "kq" else "0"
    os.environ["RIE_GEMV_KQ_MIN_MB"] = "0"
    try:
        ctx = rie.Context(0, torch.cuda.current_stream())
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return torch, rie, ctx
