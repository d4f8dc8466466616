"""The workloads the golden vectors are made from, regenerated from seeds by the tests."""
from __future__ import annotations

from localstrm_b200 import workloads as wl
from tests.golden.edge_cases import edge_workloads


def golden_sets() -> dict:
    sets = {
        "cfg1": wl.config1(seed=0),
        "cfg2": wl.config2(seed=0),
        "cfg3": wl.config3(seed=0, B=64),
        "cfg5": wl.config5(seed=0, B=16),
    }
    sets.update(edge_workloads())
    return sets
