"""The allocation-free entry point ``vinfer_sample_static``, against ``vinfer_sample``.

Some callers cannot allocate device memory at sampling time: a serving engine that gave nearly
all of HBM to its KV-cache pool at start-up, or a host that links only the C library and has
no device allocator of its own. ``vinfer_sample_static`` serves them from a fixed scratch array
compiled into the library. These tests call it through the C ABI and check that it returns the
same ids and probabilities as ``vinfer_sample`` with a caller workspace, on consecutive calls of
different shapes (the shared array keeps what the previous call left), and that shapes beyond
the array are refused. The file sorts last so that a stop-at-first-failure run has already run
every other test when it gets here.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from tests.helpers import PROB_RTOL, TINY, to_device
from vinfer_b200 import SAMPLER, BackendContext, _lib
from vinfer_b200.build import build
from vinfer_b200.workloads import make


def _static_call(backend, w, probs: bool):
    """One call of vinfer_sample_static on workload ``w``; returns (ids, probs) on the host."""
    lg, params, u, hist = to_device(w, backend.device)
    out = torch.full((w.batch,), -7, dtype=torch.int32, device=backend.device)
    pout = (torch.full((w.batch, w.vocab), -1.0, dtype=torch.float32, device=backend.device)
            if probs else None)
    a = backend.args(lg, params, u, hist, out, pout)
    rc = backend.lib.vinfer_sample_static(C.byref(a), backend._stream())
    _lib.check(rc, "vinfer_sample_static")
    torch.cuda.synchronize()
    backend.check()
    return out.cpu().numpy(), (pout.cpu().numpy() if probs else None)


def _workspace_call(backend, w, probs: bool):
    lg, params, u, hist = to_device(w, backend.device)
    pout = (torch.empty(w.batch, w.vocab, dtype=torch.float32, device=backend.device)
            if probs else None)
    ids = backend.sample_batch(lg, params, u, hist, probs_out=pout)
    torch.cuda.synchronize()
    backend.check()
    return ids.cpu().numpy(), (pout.cpu().numpy() if probs else None)


def _same(ref, got):
    ids_r, p_r = ref
    ids_g, p_g = got
    np.testing.assert_array_equal(ids_g, ids_r)
    if p_r is not None:
        assert np.array_equal(p_r > TINY, p_g > TINY)
        k = p_r > TINY
        rel = np.abs(p_g[k] - p_r[k]) / p_r[k]
        assert rel.size == 0 or rel.max() <= PROB_RTOL


@pytest.mark.gpu
def test_static_call_allocates_no_device_memory():
    # After a first call (which may load the library's device code and look up the scratch
    # array's address), a call of another shape with its inputs and outputs already on the
    # device must leave the device's free memory exactly as it was.
    backend = SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), torch.bfloat16))
    _static_call(backend, make(3, batch=4), probs=False)
    w = make(3, batch=40, seed=5)
    lg, params, u, hist = to_device(w, backend.device)
    out = torch.full((w.batch,), -7, dtype=torch.int32, device=backend.device)
    a = backend.args(lg, params, u, hist, out, None)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    rc = backend.lib.vinfer_sample_static(C.byref(a), backend._stream())
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    _lib.check(rc, "vinfer_sample_static")
    backend.check()
    assert free1 == free0
    assert ((out.cpu().numpy() >= 0) & (out.cpu().numpy() < w.vocab)).all()


@pytest.mark.gpu
def test_static_scratch_matches_the_workspace_entry_point():
    backend = SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), torch.bfloat16))
    # two shapes in a row: rows split across many CTAs (per-row counters and run records in
    # the scratch), then a different layout over the same array, then the first one again
    first = make(3, batch=8)                        # bf16, vocab 151,936, penalties
    second = make(1, batch=24)                      # float32 logits, another layout
    for w, probs in ((first, True), (second, False), (first, False)):
        _same(_workspace_call(backend, w, probs), _static_call(backend, w, probs))


def test_shapes_beyond_the_static_scratch_are_refused():
    build()
    lib = _lib.load()
    # the largest float32 vocabulary needs the most scratch per row; at least 63 rows fit
    def ws(rows):
        return lib.vinfer_sampler_workspace_bytes(rows, _lib.MAX_VOCAB, _lib.DTYPE_F32)
    too_big = 63
    while ws(too_big) <= _lib.STATIC_SCRATCH_BYTES:
        too_big += 1
    assert ws(too_big - 1) <= _lib.STATIC_SCRATCH_BYTES < ws(too_big)
    a = _lib.SampleArgs()
    a.logits = 256
    a.out_ids = 256
    a.dtype = _lib.DTYPE_F32
    a.batch, a.vocab, a.ld, a.vocab_total = too_big, _lib.MAX_VOCAB, _lib.MAX_VOCAB, _lib.MAX_VOCAB
    # refused before any CUDA call: this runs without a GPU
    assert lib.vinfer_sample_static(C.byref(a), None) == _lib.E_LIMIT
    with pytest.raises(RuntimeError, match="limit exceeded"):
        _lib.check(lib.vinfer_sample_static(C.byref(a), None), "vinfer_sample_static")
    assert lib.vinfer_sample_static(None, None) == _lib.E_ARG
