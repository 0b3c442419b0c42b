import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kraken-infer_b200")
for p in (PKG, ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def _build_once():
    # Builds the CUDA library and the CPU oracle when their sources are newer
    # than the binaries (no-op otherwise).
    import build as kib_build  # kraken-infer_b200/build.py
    kib_build.build()
    oracle_so = os.path.join(ROOT, "oracle", "_ref", "liboracle.so")
    src = os.path.join(ROOT, "oracle", "kib_oracle.cpp")
    if not os.path.exists(oracle_so) or os.path.getmtime(src) > os.path.getmtime(oracle_so):
        subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle")])


_build_once()


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] >= 10
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no sm_100 GPU on this machine")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def ctx():
    import kib
    c = kib.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def oracle():
    import oracle_lib
    return oracle_lib.Oracle()


@pytest.fixture(scope="session")
def tmpdir_session(tmp_path_factory):
    return tmp_path_factory.mktemp("kib")
