import hashlib
import json
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "tinyllm-pynq-z2_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the compiled library")
    config.addinivalue_line("markers", "slow: long-running parity case")


def cuda_ok():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_tiny():
    return json.loads((GOLDEN / "tiny_request.json").read_text())


@pytest.fixture(scope="session")
def golden_shipped():
    return json.loads((GOLDEN / "shipped_request.json").read_text())


@pytest.fixture(scope="session")
def golden_codec():
    return json.loads((GOLDEN / "codec.json").read_text())


@pytest.fixture(scope="session")
def tiny_files(tmp_path_factory, golden_tiny):
    """The tiny synthetic model of the golden request, regenerated from its seed
    and checked against the recorded SHA-256 (pins the writer + generator)."""
    from q6w_b200 import format as fmt

    d = tmp_path_factory.mktemp("tiny")
    b, m = d / "tiny.bin", d / "tiny.json"
    fmt.write_synthetic(fmt.TINY_ARGS, golden_tiny["seed"], b, m)
    assert hashlib.sha256(b.read_bytes()).hexdigest() == golden_tiny["binary_sha256"]
    return b, m


def _shipped_candidates():
    """Directories that may hold the shipped QAT artifact: $Q6W_SHIPPED_DIR,
    the artifacts folder of a reference checkout named by $Q6W_REFERENCE, and
    tests/golden/shipped/ (an uncommitted local copy made by
    ``tests/golden/make_golden.py --copy-shipped``)."""
    cands = []
    if os.environ.get("Q6W_SHIPPED_DIR"):
        cands.append(Path(os.environ["Q6W_SHIPPED_DIR"]))
    if os.environ.get("Q6W_REFERENCE"):
        cands.append(Path(os.environ["Q6W_REFERENCE"]) / "quantization" / "artifacts")
    cands.append(GOLDEN / "shipped")
    return cands


@pytest.fixture(scope="session")
def shipped_files(golden_shipped):
    """The shipped QAT artifact (binary + manifest); skips when no copy is found."""
    name = golden_shipped["binary_file"]
    for c in _shipped_candidates():
        b, m = c / name, c / name.replace(".bin", ".json")
        if b.exists() and m.exists():
            return b, m
    pytest.skip("shipped Q6W artifact not available (set Q6W_SHIPPED_DIR or run make_golden.py --copy-shipped)")


@pytest.fixture(scope="session")
def shipped_files_env(shipped_files):
    """The shipped QAT artifact for the GPU tests (same lookup)."""
    return shipped_files


def small_model_files(tmp_path_factory, args, seed, tag):
    from q6w_b200 import format as fmt

    d = tmp_path_factory.mktemp(tag)
    b, m = d / f"{tag}.bin", d / f"{tag}.json"
    fmt.write_synthetic(args, seed, b, m)
    return b, m
