import os
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "nnc-py_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

# Where the reference checkout lives (codegen and pin tests that need it skip
# when it is absent): the build entry's default unless NNC_REFERENCE is set.
import __graft_entry__  # noqa: E402

os.environ.setdefault("NNC_REFERENCE", str(__graft_entry__.REFERENCE))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA operator library)")


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA operator library on device 0; loading failures are errors."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nnc_cuda import lib

    so = lib.load()
    torch.cuda.init()
    assert so.nnc_cuda_init(0) == 0, so.nnc_cuda_get_last_error_string()
    return so


@pytest.fixture(autouse=True)
def _clear_cuda_status(request):
    if "cuda_lib" in request.fixturenames:
        so = request.getfixturevalue("cuda_lib")
        so.nnc_cuda_clear_error()
        so.nnc_cuda_set_precision(0)
    yield
