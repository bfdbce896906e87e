import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden_hashes():
    return json.loads((GOLDEN / "block_hashes.json").read_text())


@pytest.fixture(scope="session")
def golden_records():
    return {c["case"]: c for c in json.loads((GOLDEN / "kv_records.json").read_text())}


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    """Build libcrosscache.so (incremental) before any test imports it."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_cc_build", ROOT / "demo_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    if os.environ.get("CROSSCACHE_SKIP_BUILD") != "1":
        mod.build()
    yield
