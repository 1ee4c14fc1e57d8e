"""Shared test helpers: run the B200 sampler on a workload and compare with the CPU oracle.

The comparison implements the north-star parity rules:
* greedy ids and top-k kept sets are bit-exact;
* final probabilities agree within 1e-5 relative (float32);
* sampled ids are identical except on rows whose draw, top-p or min-p decision lies within
  1e-6 of a cumulative-mass edge ("boundary" rows), which are counted and reported.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from oracle.sampler_oracle import RowParams as OracleParams
from oracle.sampler_oracle import RowResult, process_row
from vinfer_b200.sampling import RowParams, TokenHistogram
from vinfer_b200.workloads import Workload

import warnings

PROB_RTOL = 1e-5  # north-star tolerance on processed probabilities (relative, float32)
TINY = 1e-30  # probabilities this small are compared for presence only


def to_device(w: Workload, device):
    logits = w.logits.to(device)
    params = RowParams.from_arrays(device, **w.param_arrays())
    u = torch.from_numpy(w.uniforms).to(device)
    hist = None
    if w.hist_row_ptr is not None:
        hist = TokenHistogram.from_csr(w.hist_row_ptr, w.hist_ids, w.hist_counts, device)
    return logits, params, u, hist


def run_b200(backend, w: Workload, probs: bool = True, exact: bool = False,
             logits: torch.Tensor | None = None):
    lg, params, u, hist = to_device(w, backend.device)
    if logits is not None:
        lg = logits
    pout = torch.empty(w.batch, w.vocab, dtype=torch.float32, device=backend.device) if probs else None
    ids = backend.sample_batch(lg, params, u, hist, probs_out=pout, exact=exact)
    torch.cuda.synchronize()
    backend.check()
    return ids.cpu().numpy(), (pout.cpu().numpy() if probs else None)


def oracle_row(w: Workload, r: int) -> RowResult:
    x = w.logits[r].float().numpy()
    p = OracleParams(
        temperature=float(w.temperature[r]), top_k=int(w.top_k[r]), top_p=float(w.top_p[r]),
        min_p=float(w.min_p[r]), repetition_penalty=float(w.repetition_penalty[r]),
        presence_penalty=float(w.presence_penalty[r]),
        frequency_penalty=float(w.frequency_penalty[r]))
    ids = cnt = None
    if w.hist_row_ptr is not None:
        a, b = int(w.hist_row_ptr[r]), int(w.hist_row_ptr[r + 1])
        ids, cnt = w.hist_ids[a:b], w.hist_counts[a:b]
    return process_row(x, p, float(w.uniforms[r]), ids, cnt)


@dataclass
class Report:
    rows: int = 0
    boundary: int = 0
    boundary_mismatch: int = 0
    failures: list = field(default_factory=list)

    def __str__(self) -> str:
        return (f"{self.rows} rows, {self.boundary} boundary rows "
                f"({self.boundary_mismatch} of them differ), {len(self.failures)} failures")


def compare(w: Workload, ids: np.ndarray, probs: np.ndarray | None,
            rows: list[int] | None = None) -> Report:
    rep = Report()
    rows = list(range(w.batch)) if rows is None else rows
    for r in rows:
        res = oracle_row(w, r)
        rep.rows += 1
        if w.temperature[r] == 0:
            if int(ids[r]) != res.token:
                rep.failures.append((r, "greedy id", int(ids[r]), res.token))
            continue
        if res.boundary:
            rep.boundary += 1
            if int(ids[r]) != res.token:
                rep.boundary_mismatch += 1
            continue
        if int(ids[r]) != res.token:
            rep.failures.append((r, "sampled id", int(ids[r]), res.token))
        if probs is not None:
            want, got = res.probs, probs[r]
            # probabilities below float32's normal range flush to zero on the device
            differ = ((want > 0) != (got > 0)) & (np.maximum(want, got) > TINY)
            if differ.any():
                rep.failures.append((r, "kept set", int((got > 0).sum()), int((want > 0).sum())))
                continue
            k = want > TINY
            rel = np.abs(got[k] - want[k]) / want[k]
            if rel.size and rel.max() > PROB_RTOL:
                rep.failures.append((r, "probs", float(rel.max()), PROB_RTOL))
    return rep


class ParityReport(UserWarning):
    """A parity comparison's counts (rows, boundary rows, failures), reported in pytest's
    warnings summary so every run's log records them."""


def report(name: str, rep: Report) -> None:
    warnings.warn(f"parity {name}: {rep}", ParityReport, stacklevel=2)
