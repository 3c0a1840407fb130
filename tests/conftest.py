import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "s-moe_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def ctx():
    """One context for the session, bound to a torch stream that is also
    torch's current stream while the tests run: tensors the tests allocate,
    fill and read back are then ordered with the context's kernels."""
    import torch
    import smoe_cuda
    c = smoe_cuda.Context(0)
    s = torch.cuda.Stream()
    c.set_stream(s.cuda_stream)
    with torch.cuda.stream(s):
        yield c
    c.synchronize()
    c.close()
