import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "voyager-compiler_b200"), os.path.dirname(__file__)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size case, minutes on CPU")


@pytest.fixture(autouse=True)
def _device_wait_status(request):
    """After every GPU test: no tcgen05 / barrier kernel of the library gave
    up a bounded wait during it (the sticky device word, read and cleared).
    Tests that make a wait run out on purpose clear the word themselves."""
    yield
    if request.node.get_closest_marker("gpu") is None or "voyager_b200" not in sys.modules:
        return
    import torch

    if not torch.cuda.is_available():
        return
    import voyager_b200

    voyager_b200.check_errors()
