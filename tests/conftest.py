"""Shared fixtures.  `-m "not gpu"` runs the oracle, host logic and ABI checks
on CPU; `-m gpu` runs the parity tests of the CUDA path against the oracle
and the reference-generated golden fixtures (tests/golden/)."""
from __future__ import annotations

import importlib
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size BASELINE configuration")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("cis2-lab-archive_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("cis2-lab-archive_b200.synth")


@pytest.fixture(scope="session")
def synth_root(synth):
    root = synth.default_root()
    os.makedirs(root, exist_ok=True)
    return root


@pytest.fixture(scope="session")
def oracle():
    import pyoracle
    return pyoracle


def load_golden(name: str) -> dict:
    with open(os.path.join(GOLDEN, name + ".json")) as f:
        return json.load(f)


def golden_names() -> list[str]:
    """Decode fixtures (math_sweep.json holds the pinned-function sweep instead)."""
    return sorted(f[:-5] for f in os.listdir(GOLDEN) if f.endswith(".json") and not f.startswith("math_"))


def golden_prompts(synth, g: dict) -> list:
    spec = g["prompts"]
    if spec[0] == "workload":
        _, w, first, count = spec
        return list(synth.prompt_ids(w, n_seq=count, first=first))
    _, seed, lens = spec
    return [synth.random_prompts(g["model"], 1, L, seed, first=i)[0] for i, L in enumerate(lens)]
