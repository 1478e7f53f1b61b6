"""Shared fixtures.  `-m "not gpu"` runs the oracle, host logic and ABI checks
on CPU; `-m gpu` runs the parity tests of the CUDA path against the oracle
and the reference-generated golden fixtures (tests/golden/)."""
from __future__ import annotations

import importlib
import json
import os
import sys

import numpy as np
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
    if spec[0] == "workload_idx":
        _, w, idx = spec
        return [synth.prompt_ids(w, n_seq=1, first=i)[0] for i in idx]
    _, seed, lens = spec
    return [synth.random_prompts(g["model"], 1, L, seed, first=i)[0] for i, L in enumerate(lens)]


def argmax_edge_rows(V: int) -> list[np.ndarray]:
    """Rows exercising the selection clause of code/cis2-fp/src/main.rs:1161-1169
    (first index of the strict maximum): exact ties at spread positions,
    +0/-0 ties, NaN at index 0 and NaN elsewhere, infinities, all-equal."""
    rng = np.random.default_rng(V)
    rows = []
    base = lambda: rng.normal(0, 1, V).astype(np.float32)
    for i, j in [(0, V - 1), (V // 3, V // 3 + 1), (7 % V, V - 2), (V - 2, V - 1)]:
        r = base()
        r[[i, j]] = np.float32(9.5)
        rows.append(r)
    r = base()
    idx = np.sort(rng.choice(V, size=min(5, V), replace=False))
    r[idx] = np.float32(11.25)  # five-way tie
    rows.append(r)
    for a, b in [(np.float32(-0.0), np.float32(0.0)), (np.float32(0.0), np.float32(-0.0))]:
        r = -np.abs(base()) - np.float32(1.0)
        i, j = V // 4, V // 2 + 3
        r[i], r[j] = a, b
        rows.append(r)
    r = base()
    r[0] = np.nan
    r[V // 2] = np.float32(50.0)
    rows.append(r)  # NaN at index 0 selects 0
    r = base()
    r[rng.choice(np.arange(1, V), size=min(9, V - 1), replace=False)] = np.nan
    r[V - 1] = np.float32(40.0)
    r[1] = np.nan
    rows.append(r)  # NaNs elsewhere are never selected
    r = np.full(V, np.nan, dtype=np.float32)
    r[0] = np.float32(-3.0)
    rows.append(r)  # every other value NaN
    r = np.full(V, -np.inf, dtype=np.float32)
    rows.append(r)  # all -inf
    r = base()
    r[[V // 5, V - 1]] = np.inf
    rows.append(r)  # +inf tie
    rows.append(np.full(V, np.float32(0.125)))  # all equal
    return rows

