"""pytest setup: the ``gpu`` marker, the package loader and golden-fixture access.

``-m "not gpu"`` runs the oracle-vs-golden pins, host logic and C-ABI export
checks on CPU; ``-m gpu`` runs the kernel parity tests through the C-ABI.
"""
from __future__ import annotations

import importlib.util
import json
import pathlib
import sys

import numpy as np
import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"


def _register_package() -> None:
    if "nanopointllm_b200" in sys.modules:
        return
    pkg = REPO / "nano-pointllm_b200"
    spec = importlib.util.spec_from_file_location(
        "nanopointllm_b200", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["nanopointllm_b200"] = mod
    spec.loader.exec_module(mod)


if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
_register_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: larger CPU cases")


def golden(name: str):
    path = GOLDEN / name
    if name.endswith(".json"):
        return json.loads(path.read_text())
    return np.load(path, allow_pickle=False)


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"kernels are built for sm_100a, device is sm_{major}{minor}")
    return torch.device("cuda:0")
