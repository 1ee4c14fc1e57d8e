"""Batched decode on the device (GPU only): slotted histories updated in place by
vinfer_hist_append / vinfer_hist_reset, checked against a host model step by step, and a
decode loop (sample -> count the ids -> sample) checked against the CPU oracle at every step."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.sampler_oracle import RowParams as OracleParams
from oracle.sampler_oracle import process_row
from tests.helpers import Report, report
from tests.test_decode_cpu import append_model
from vinfer_b200 import SAMPLER, BackendContext, SlotHistogram
from vinfer_b200 import _lib
from vinfer_b200.sampling import RowParams

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def backend():
    return SAMPLER.resolve("b200", BackendContext(torch.device("cuda", 0), torch.bfloat16))


def test_append_and_reset_match_the_host_model(backend):
    dev = backend.device
    rng = np.random.default_rng(3)
    S, cap = 40, 300
    rows = [rng.integers(0, 1000, rng.integers(0, 200)).tolist() for _ in range(S)]
    rows[0] = list(range(cap))  # a full slot
    slots = SlotHistogram.from_token_lists(rows, cap, dev)
    model = slots.to_counts()
    for step in range(60):
        toks = rng.integers(-1, 1000, S).astype(np.int32)
        toks[1] = 999 - step  # new ids in descending order: inserted at the front
        toks[2] = 1000 + step  # new ids in ascending order: appended at the end
        full = append_model(model, toks, cap)
        backend.append_tokens(slots, torch.from_numpy(toks).to(dev))
        got = slots.to_counts()
        assert got == model, f"step {step}"
        bits = int(backend.status[0])
        assert bool(bits & _lib.ST_HIST_FULL) == full
        backend.status.zero_()
        if step == 30:  # two requests leave; out-of-range entries are skipped
            backend.reset_slots(slots, torch.tensor([5, 7, -3, S + 9], dtype=torch.int32,
                                                    device=dev))
            model[5], model[7] = {}, {}
            assert slots.to_counts() == model
    ids, counts, lens = (x.cpu().numpy() for x in (slots.ids, slots.counts, slots.lens))
    for s in range(S):  # the padding survived every insertion: still a valid CSR history
        seg = ids[s * cap:(s + 1) * cap].astype(np.int64)
        assert np.all(seg[1:] > seg[:-1])
        assert np.all(counts[s * cap + lens[s]:(s + 1) * cap] == 0)


def test_decode_loop_matches_the_oracle_step_by_step(backend):
    dev = backend.device
    S, V, cap, steps = 64, 4096, 512, 32
    g = torch.Generator().manual_seed(11)
    rng = np.random.default_rng(11)
    kinds = [dict(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.1,
                  presence_penalty=0.5, frequency_penalty=0.3),
             dict(temperature=1.0, top_k=50, top_p=0.95, repetition_penalty=1.3),
             dict(temperature=0.9, top_k=0, top_p=0.9, presence_penalty=0.4),
             dict(temperature=0.8, top_k=30, repetition_penalty=0.9, presence_penalty=-0.3),
             dict(temperature=0.0, repetition_penalty=1.2)]
    params = [kinds[s % len(kinds)] for s in range(S)]
    col = (lambda n, d, dt=np.float32: np.array([p.get(n, d) for p in params], dt))
    arrays = dict(temperature=col("temperature", 1.0), top_k=col("top_k", 0, np.int32),
                  top_p=col("top_p", 1.0), min_p=col("min_p", 0.0),
                  repetition_penalty=col("repetition_penalty", 1.0),
                  presence_penalty=col("presence_penalty", 0.0),
                  frequency_penalty=col("frequency_penalty", 0.0))
    rp = RowParams.from_arrays(dev, **arrays)
    prompts = [rng.integers(0, V, 40).tolist() for _ in range(S)]
    slots = SlotHistogram.from_token_lists(prompts, cap, dev)
    model = slots.to_counts()
    out = torch.empty(S, dtype=torch.int32, device=dev)
    rep = Report()
    for step in range(steps):
        x = (torch.randn(S, V, generator=g) * 2.5).to(torch.bfloat16)
        for s in range(S):  # the previous tokens are likely again: penalties decide
            if model[s]:
                x[s, list(model[s])[:8]] += 6.0
        u = torch.rand(S, generator=g)
        backend.decode_step(x.to(dev), rp, u.to(dev), slots, out=out)
        ids = out.cpu().numpy()
        backend.check()
        for s in range(S):
            hid = np.array(sorted(model[s]), np.int32)
            hc = np.array([model[s][i] for i in hid], np.int32)
            p = OracleParams(**{k: float(v[s]) if k != "top_k" else int(v[s])
                                for k, v in arrays.items()})
            res = process_row(x[s].float().numpy(), p, float(u[s]), hid, hc)
            rep.rows += 1
            if res.boundary:
                rep.boundary += 1
                rep.boundary_mismatch += int(ids[s] != res.token)
            elif int(ids[s]) != res.token:
                rep.failures.append((step, s, int(ids[s]), res.token))
        # the device counted its own ids (a boundary row may differ from the oracle's)
        append_model(model, ids, cap)
        assert slots.to_counts() == model, f"histograms differ after step {step}"
    report(f"decode loop ({S} slots x {steps} steps, vocab {V})", rep)
    assert not rep.failures, (str(rep), rep.failures[:5])
