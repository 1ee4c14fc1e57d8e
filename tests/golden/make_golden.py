"""Generate ``sampler_golden.npz`` from vinfer's own reference sampler.

Run where the reference source tree is available (it is pure Python + torch)::

    VINFER_REFERENCE_SRC=<path to vinfer>/src python tests/golden/make_golden.py

It imports ``vinfer.runtime.sampler`` (``filtered_probs``, ``sample``, ``SamplingParams``) and
records, on seeded synthetic rows:

* ``fp_*``: ``filtered_probs(logits, params)`` for temperature / top-k / top-p grids, on the
  reference's own toy vector (``tests/unit/runtime/test_sampler.py:10``), random rows of
  several vocab sizes (float32 and bf16-valued), and tie-heavy rows;
* ``greedy_*``: ``sample(..., temperature=0)`` ids (first index of the maximum);
* ``race_*``: ``sample(logits, params, seed, position)`` ids, which pin
  ``oracle/reference_port.py``'s exponential race bit-exactly.

The file is small (< 1 MB) and committed; the GPU box never needs the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).with_name("sampler_golden.npz")


def _import_reference():
    src = os.environ.get("VINFER_REFERENCE_SRC")
    if src:
        sys.path.insert(0, src)
    from vinfer.runtime import sampler  # noqa: PLC0415

    return sampler


def main() -> None:
    ref = _import_reference()
    g = torch.Generator().manual_seed(1234)
    out: dict[str, np.ndarray] = {}

    rows: list[torch.Tensor] = []
    names: list[str] = []
    rows.append(torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -3.0]))
    names.append("toy")
    for V in (96, 1000, 4096):
        for sigma in (0.5, 2.0):
            x = torch.randn(V, generator=g) * sigma
            spikes = torch.randperm(V, generator=g)[:3]
            x[spikes] += 6.0
            rows.append(x)
            names.append(f"f32_v{V}_s{sigma}")
            rows.append(x.to(torch.bfloat16).float())
            names.append(f"bf16_v{V}_s{sigma}")
    # ties: a flat row, and a row whose maximum is shared by 50 tokens
    rows.append(torch.zeros(500))
    names.append("flat500")
    x = torch.randn(2000, generator=g)
    tie = torch.randperm(2000, generator=g)[:50]
    x[tie] = 5.0
    rows.append(x)
    names.append("tie50_v2000")

    grid = []
    for t in (0.5, 0.7, 1.0, 1.5):
        for k in (0, 1, 3, 20, 50):
            for p in (1.0, 0.9, 0.5, 0.1):
                grid.append((t, k, p))
    params_arr = np.array(grid, dtype=np.float64)

    for i, (name, x) in enumerate(zip(names, rows, strict=True)):
        out[f"logits_{i}"] = x.numpy().astype(np.float32)
        probs = []
        for t, k, p in grid:
            sp = ref.SamplingParams(temperature=t, top_k=int(k), top_p=p)
            probs.append(ref.filtered_probs(x, sp).numpy())
        out[f"fp_{i}"] = np.stack(probs).astype(np.float32)
        out[f"greedy_{i}"] = np.array(
            [ref.sample(x, ref.SamplingParams(temperature=0), 0, 0)], dtype=np.int64
        )
        races = []
        for j, (t, k, p) in enumerate(grid[::7]):
            sp = ref.SamplingParams(temperature=t, top_k=int(k), top_p=p)
            seed, pos = 11 + j, 3 * j
            races.append([j * 7, seed, pos, ref.sample(x, sp, seed, pos)])
        out[f"race_{i}"] = np.array(races, dtype=np.int64)
    out["names"] = np.array(names)
    out["grid"] = params_arr
    out["position_seed"] = np.array(
        [[s, p, ref.position_seed(s, p)] for s in (0, 7, 8, 2**40) for p in (0, 1, 99, 151935)],
        dtype=np.uint64,
    )
    out["torch_version"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KiB) with {len(names)} rows")


if __name__ == "__main__":
    main()
