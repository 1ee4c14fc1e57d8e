"""bench.py's line contract on CPU: the workload object ('config') is the same in the GPU arm
and the reference arm at every N, so the two lines describe the same measurement."""

from __future__ import annotations

import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_workload_config_is_the_workload_alone():
    b = _bench()
    c1 = b.workload_config(1, 402171)
    assert c1 == {"workload": b.CONFIG3_WORKLOAD, "batch": 256, "vocab": 151_936,
                  "hist_nnz": 402171}
    for world in (2, 4, 8):
        c = b.workload_config(world)
        assert c["batch"] == 1024 and c["vocab"] == 248_320
        assert f"over {world} GPUs" in c["workload"]


def test_both_arms_build_config_from_the_same_function():
    src = (ROOT / "bench.py").read_text()
    # the GPU arm at N = 1 and N > 1, and the reference arm, all take workload_config(...)
    assert src.count('"config": workload_config(') == 3
