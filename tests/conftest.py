"""Shared test set-up: the package loader, the `gpu` marker, fixtures."""
from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "paris-hackathon-2026-inference_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    """Import the package directory (hyphenated name) as `paris_moe_b200`."""
    name = "paris_moe_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


PM = load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built library")


def load_golden(name):
    d = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    meta = json.loads(bytes(d["meta"]).decode())
    return d, meta


def golden_inputs(meta, device="cpu"):
    """Regenerate the fixture's seeded weights and hidden states."""
    from paris_moe_b200 import workload as W
    shape = W.MoEShape(H=meta["H"], E=meta["E"], K=meta["K"], I=meta["I"], Is=meta["Is"])
    wts = W.make_weights(shape, seed=meta["seed"], zipf_s=meta["zipf_s"], device=device)
    x = W.make_hidden(meta["T"], shape, seed=meta["seed"], zipf=meta["zipf_s"] is not None,
                      device=device)
    return shape, wts, x


@pytest.fixture(scope="session")
def pm():
    return PM
