"""Test configuration: the ``gpu`` marker, repo root on sys.path, shared fixtures.

``-m "not gpu"`` runs on a CPU-only machine: the oracle against the golden
fixtures, host logic, and the C ABI's exports and argument checks.
``-m gpu`` runs the parity tests of the CUDA library through its C ABI.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def reference_root() -> Path | None:
    """The reference checkout, when present: $JOULE_REFERENCE, else a
    `reference` directory beside this repository. Only CPU tests use it; GPU
    tests and the bench never read it."""
    import os
    cand = os.environ.get("JOULE_REFERENCE")
    p = Path(cand) if cand else ROOT.parent / "reference"
    return p if (p / "src" / "jouleai" / "native" / "backend.py").exists() else None


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_loader():
    return golden


_LAYER_CACHE: dict = {}


def seeded_layer(tag: str):
    """The full-size benchmark layers the golden fixtures were made from."""
    from oracle import layer as olayer
    shapes = {"olmoe": (2048, 64, 8, 1024, 0), "qwen3": (2048, 128, 8, 768, 1)}
    if tag not in _LAYER_CACHE:
        d, E, k, m, norm = shapes[tag]
        _LAYER_CACHE[tag] = olayer.make_layer(d, E, k, m, norm, seed_router=0, seed_experts=1)
    return _LAYER_CACHE[tag]


def stored_small_layer(g: dict):
    """A small golden layer rebuilt from the arrays stored in its fixture."""
    from oracle.layer import Q4Layer
    d, E, k, m, norm = (int(v) for v in g["cfg"])
    lay = Q4Layer(d, E, k, m, norm, g["gate_w"].copy(), [[None] * E for _ in range(3)],
                  [[None] * E for _ in range(3)])
    for e in range(E):
        for p in range(2):
            lay.scales[p][e] = g["scales"][p][e].copy()
            lay.packed[p][e] = g["packed"][p][e].copy()
        lay.scales[2][e] = g["scales_down"][e].copy()
        lay.packed[2][e] = g["packed_down"][e].copy()
    return lay


SMALL = ["moe_small_b1", "moe_small_b5", "moe_small_b16", "moe_small_ties",
         "moe_small_collide", "moe_small_saturate"]
BIG = [f"moe_{t}_b{b}" for t in ("olmoe", "qwen3") for b in (1, 4, 16)]
