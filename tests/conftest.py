import os
import subprocess
import sys
import tempfile

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: multi-minute CPU oracle runs")


def _gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def lib():
    """The product library, built in-tree if missing."""
    import lunelette_b200
    if not os.path.exists(lunelette_b200.LIBRARY_PATH):
        from lunelette_b200 import build
        build.build()
    return lunelette_b200.library()


@pytest.fixture(scope="session")
def oracle():
    from tests import oracle_lib
    return oracle_lib.load()


@pytest.fixture(scope="session")
def ref_lib():
    """The reference's own portable C compiled by oracle/Makefile, when present."""
    import ctypes
    path = os.path.join(REPO, "oracle", "_ref", "libref.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    return ctypes.CDLL(path)


@pytest.fixture(scope="session")
def checkpoint_path(lib):
    """Seed-0 synthetic checkpoint (3.8 GB), written once per machine."""
    import lunelette_b200
    path = os.environ.get("LUNELETTE_CHECKPOINT")
    if not path:
        path = os.path.join(tempfile.gettempdir(), "lunelette_synth_seed0.safetensors")
    if not os.path.exists(path):
        tmp = path + ".partial%d" % os.getpid()
        lunelette_b200.synth_checkpoint(tmp, 0)
        os.replace(tmp, path)
    return path
