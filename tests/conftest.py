import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
    config.addinivalue_line("markers", "slow: CPU test that takes more than ~20 s")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def blob_path():
    from qwen_fpga_b200 import synth
    return synth.ensure_blob(1234)


@pytest.fixture(scope="session")
def blob(blob_path):
    from qwen_fpga_b200 import synth
    return synth.Blob(blob_path)


@pytest.fixture(scope="session")
def fq_weights(blob):
    return blob.fake_quant()


@pytest.fixture(scope="session")
def cfg():
    from qwen_fpga_b200 import synth
    return synth.model_config()


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(REPO, "tests", "golden")
