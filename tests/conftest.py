import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more CUDA devices")


def assert_close(actual, expected, *, rtol=1e-5, atol=1e-6):
    import torch
    torch.testing.assert_close(actual, expected, rtol=rtol, atol=atol)


@pytest.fixture(autouse=True)
def _clear_native_error_words(request):
    """Each GPU test starts with clear native error words, so a test that expects
    (and checks) a timeout code cannot leak it into the next test."""
    if request.node.get_closest_marker("gpu") is not None:
        import torch
        if torch.cuda.is_available():
            from torch_einshard_b200.ops import _native
            _native.reset_errors()
    yield
