"""Every registered sampler backend against the CPU oracle, on this machine's devices, in fp32
and bf16 -- the reference's contract-test pattern (``tests/unit/kernels/
test_backend_contract.py:1-40``): a backend that cannot run in a (device, dtype) context is
skipped with the registry's own reason, so ``b200`` runs on a B200 and ``reference`` wherever
vinfer is importable.

The ``b200`` backend also registers into vinfer's real ``BackendRegistry`` (when the reference
tree is present): the same decorator arguments, the same ``unsupported`` reason off a B200, and
``resolve`` raising instead of falling back (``src/vinfer/kernels/registry.py:84-88``).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.helpers import compare
from vinfer_b200 import SAMPLER, BackendContext
from vinfer_b200.kernels.sampler import b200 as b200_mod
from vinfer_b200.sampling import RowParams
from vinfer_b200.workloads import Workload

REF_SRC = Path("/root/reference/src")
DEVICES = [pytest.param(torch.device("cpu"), id="cpu"),
           pytest.param(torch.device("cuda", 0), id="cuda", marks=pytest.mark.gpu)]
DTYPES = [torch.float32, torch.bfloat16]

PARAMS = [
    dict(temperature=0.0),
    dict(temperature=1.0, top_k=1),
    dict(temperature=0.7, top_k=20),
    dict(temperature=1.3, top_k=50, top_p=0.9),
    dict(temperature=0.8, top_p=0.7),
    dict(temperature=1.0, top_k=20, min_p=0.05),
    dict(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.1, presence_penalty=0.5,
         frequency_penalty=0.3),
    dict(temperature=0.0, repetition_penalty=1.5),
]


def _workload(dtype: torch.dtype) -> Workload:
    B, V = len(PARAMS), 3000
    g = torch.Generator().manual_seed(17)
    x = (torch.randn(B, V, generator=g) * 2.0).to(dtype)
    rng = np.random.default_rng(17)

    def col(name, default, dt=np.float32):
        return np.array([p.get(name, default) for p in PARAMS], dtype=dt)

    w = Workload("contract", x, col("temperature", 1.0), col("top_k", 0, np.int32),
                 col("top_p", 1.0), col("min_p", 0.0), col("repetition_penalty", 1.0),
                 col("presence_penalty", 0.0), col("frequency_penalty", 0.0),
                 rng.random(B).astype(np.float32))
    ptr, ids, cnt = [0], [], []
    for r in range(B):
        top = torch.topk(x[r].float(), 30).indices.numpy()
        u, c = np.unique(np.concatenate([top[::3], rng.integers(0, V, 100)]), return_counts=True)
        ids.append(u.astype(np.int32))
        cnt.append(c.astype(np.int32))
        ptr.append(ptr[-1] + len(u))
    w.hist_row_ptr, w.hist_ids, w.hist_counts = np.array(ptr), np.concatenate(ids), np.concatenate(cnt)
    return w


def _backend(name: str, device: torch.device, dtype: torch.dtype):
    ctx = BackendContext(device, dtype)
    if (reason := SAMPLER.unsupported(name, ctx)) is not None:
        pytest.skip(reason)
    return SAMPLER.resolve(name, ctx)


@pytest.fixture(scope="module", autouse=True)
def _vinfer_on_path():
    # the reference tree, when present in this container, makes the `reference` backend runnable
    if REF_SRC.exists() and str(REF_SRC) not in sys.path:
        sys.path.insert(0, str(REF_SRC))
    yield


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("device", DEVICES)
@pytest.mark.parametrize("name", SAMPLER.names())
def test_backend_matches_the_oracle(name, device, dtype):
    from vinfer_b200.sampling import TokenHistogram  # noqa: PLC0415

    backend = _backend(name, device, dtype)
    w = _workload(dtype)
    lg = w.logits.to(device)
    params = RowParams.from_arrays(device, **w.param_arrays())
    u = torch.from_numpy(w.uniforms).to(device)
    hist = TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, device)
    probs = torch.empty(w.batch, w.vocab, dtype=torch.float32, device=device)
    ids = backend.sample_batch(lg, params, u, hist, probs_out=probs)
    if device.type == "cuda":
        torch.cuda.synchronize()
    rep = compare(w, ids.cpu().numpy(), probs.cpu().numpy())
    assert not rep.failures, (name, str(rep), rep.failures[:5])


def test_registered_names():
    assert "b200" in SAMPLER.names()
    assert "reference" in SAMPLER.names()


def test_b200_off_a_b200_reports_why_and_never_falls_back():
    ctx = BackendContext(torch.device("cpu"), torch.bfloat16)
    reason = SAMPLER.unsupported("b200", ctx)
    assert reason is not None and "does not run on cpu" in reason
    with pytest.raises(ValueError, match="sampler backend 'b200' does not run on cpu"):
        SAMPLER.resolve("b200", ctx)
    with pytest.raises(ValueError, match="unknown sampler backend 'nope'"):
        SAMPLER.resolve("nope", ctx)


@pytest.mark.skipif(not (REF_SRC / "vinfer" / "kernels" / "registry.py").exists(),
                    reason="vinfer's source tree is not present on this machine")
def test_b200_registers_into_vinfers_own_registry():
    sys.path.insert(0, str(REF_SRC))
    from vinfer.kernels.registry import BackendContext as VinferContext  # noqa: PLC0415
    from vinfer.kernels.registry import BackendRegistry as VinferRegistry  # noqa: PLC0415

    family = VinferRegistry("sampler")
    family.register("b200", devices={"cuda"}, dtypes={torch.bfloat16, torch.float32},
                    supports=b200_mod._supports)(b200_mod.B200Sampler)
    assert family.names() == ["b200"]
    with pytest.raises(ValueError, match="registered twice"):
        family.register("b200")(b200_mod.B200Sampler)
    cpu = VinferContext(torch.device("cpu"), torch.bfloat16)
    assert "does not run on cpu" in family.unsupported("b200", cpu)
    with pytest.raises(ValueError, match="sampler backend 'b200' does not run on cpu"):
        family.resolve("b200", cpu)
    assert "does not support torch.float16" in family.unsupported(
        "b200", VinferContext(torch.device("cuda"), torch.float16))
    if not torch.cuda.is_available():
        reason = family.unsupported("b200", VinferContext(torch.device("cuda"), torch.bfloat16))
        assert reason is not None and "CUDA" in reason
