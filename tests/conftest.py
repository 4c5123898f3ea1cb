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


def assert_match_until_tie(tokens, logits, ref_tokens, ref_logits, tie_tol, atol, min_steps=0):
    """Per sequence: identical greedy tokens and logits within atol up to the
    sequence's first differing token, which must be a near-tie of the
    reference (its logits for the two tokens closer than tie_tol); later steps
    of that sequence follow another history and are not compared."""
    steps, batch = ref_tokens.shape
    for b in range(batch):
        diff = np.nonzero(tokens[:, b] != ref_tokens[:, b])[0]
        stop = int(diff[0]) if diff.size else steps
        np.testing.assert_allclose(logits[:stop + (stop < steps), b], ref_logits[:stop + (stop < steps), b],
                                   atol=atol, rtol=0, err_msg=f"sequence {b}")
        if stop < steps:
            row = ref_logits[stop, b]
            margin = abs(float(row[ref_tokens[stop, b]]) - float(row[tokens[stop, b]]))
            assert margin < tie_tol, f"sequence {b} step {stop}: tokens differ with margin {margin}"
        assert stop >= min_steps or stop == steps, f"sequence {b} diverged at step {stop}"
