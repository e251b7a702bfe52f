import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA; run with -m 'not gpu' here")
    return torch.device("cuda", 0)


REFERENCE_COPY = ROOT / "baseline" / "_ref"


@pytest.fixture
def reference_engine():
    """The reference engine (``mini_engine``) imported from the private copy under ``baseline/_ref``.

    Skips when the copy is absent.  Importing ``mini_engine`` repoints TMPDIR,
    CUDA_CACHE_PATH, TORCH_EXTENSIONS_DIR and other cache variables at
    directories inside the copy (``mini_engine/runtime.py:8-29``); they are
    restored afterwards, and the reference modules are dropped from
    ``sys.modules`` so every test starts from an unpatched package.
    """
    import os
    import tempfile

    if not (REFERENCE_COPY / "mini_engine").is_dir():
        pytest.skip("reference copy not present under baseline/_ref")
    saved_env, saved_tmp = dict(os.environ), tempfile.tempdir
    sys.path.insert(0, str(REFERENCE_COPY))
    try:
        import mini_engine

        yield mini_engine
    finally:
        sys.path.remove(str(REFERENCE_COPY))
        for name in [n for n in sys.modules if n == "mini_engine" or n.startswith("mini_engine.")]:
            del sys.modules[name]
        os.environ.clear()
        os.environ.update(saved_env)
        tempfile.tempdir = saved_tmp
