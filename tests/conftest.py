"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def kcmm_lib():
    from lattice_b200 import build, kcmm

    build.build()
    return kcmm.KcmmLibrary()


@pytest.fixture
def host_pool_factory(kcmm_lib, monkeypatch):
    """Pools on the host VMM backend (allocator logic without a GPU)."""
    from lattice_b200 import kcmm

    monkeypatch.setenv("KCMM_VMM_BACKEND", "host")
    made = []

    def make(**kw):
        kw.setdefault("num_layers", 2)
        cfg = kcmm.make_config(**kw)
        pool = kcmm_lib.create_pool(cfg)
        made.append(pool)
        return pool

    yield make
    for p in made:
        p.destroy()


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np

    g = ROOT / "tests" / "golden"
    return {
        "kats": json.loads((g / "reference_kats.json").read_text()),
        "ref": dict(np.load(g / "ref_kernels.npz")),
    }
