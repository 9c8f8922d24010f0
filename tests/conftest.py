"""Shared fixtures. GPU tests carry @pytest.mark.gpu and call the native library through
its C ABI; CPU tests cover the oracle, host logic and the library's exported surface."""

from __future__ import annotations

import dataclasses
import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) and the built native library")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return json.loads((GOLDEN / f"{name}.json").read_text())

    return load


@pytest.fixture(scope="session")
def tiny_models(tmp_path_factory):
    """C1 (tied head) and C1u (untied head) synthetic fp32 pairs, seed 0, as written by the
    fixture generator: {name: (target_dir, drafter_dir, target_weights, drafter_weights)}."""
    from woodcock_b200 import synthetic as syn

    out = {}
    for name, tie in (("c1", True), ("c1u", False)):
        ts = dataclasses.replace(syn.TINY_TARGET, tie_embeddings=tie)
        root = tmp_path_factory.mktemp(name)
        out[name] = syn.make_pair(root, "c1", seed=0, dtype="F32", target_spec=ts)
    return out


@pytest.fixture(scope="session")
def prompt64():
    from woodcock_b200 import synthetic as syn

    return syn.prompt_ids(64, 4096, seed=0)


def weights_checksum(w: dict) -> float:
    return float(sum(float(np.abs(v).sum()) for v in w.values()))
