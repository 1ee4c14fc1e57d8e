"""The ``reference`` sampler backend: vinfer's own PyTorch sampler behind the family's interface.

``sample`` is vinfer's ``sample`` (``src/vinfer/runtime/sampler.py:68-77``) called unchanged:
temperature, top-k, top-p and the exponential race seeded by ``position_seed``. It serves the
reference's parameters only (``min_p`` and the penalties must be at their defaults, as
vinfer's server enforces, ``src/vinfer/server/protocol.py:129-158``).

``sample_batch`` is the slow restatement every faster backend is compared with, in the style of
``kernels/attention/reference.py``: per row, the penalties from the row's token counts
(repetition, then frequency x count, then presence; one float32 operation each), vinfer's
``filtered_probs`` (``sampler.py:50-65``) for temperature, top-k and top-p, min-p relative to the
largest probability, renormalisation, and the inverse-CDF draw of the caller's uniform over the
kept tokens in canonical order (descending probability, ties by ascending id). Greedy rows take
the first index of the largest penalised logit.

It runs wherever vinfer is importable (any device, any float dtype) and reports why it cannot
run otherwise; nothing resolves to it implicitly.
"""

from __future__ import annotations

import torch

from vinfer_b200.kernels.sampler.base import SAMPLER
from vinfer_b200.registry import BackendContext
from vinfer_b200.sampling import RowParams, SamplingParams, TokenHistogram


def _supports(ctx: BackendContext) -> str | None:
    try:
        import vinfer.runtime.sampler  # noqa: F401, PLC0415
    except ImportError as exc:
        return f"needs vinfer's runtime sampler (vinfer.runtime.sampler): {exc}"
    return None


@SAMPLER.register("reference", supports=_supports)
class ReferenceSampler:
    """vinfer's PyTorch sampler; one row at a time."""

    def __init__(self, ctx: BackendContext) -> None:
        from vinfer.runtime import sampler as ref  # noqa: PLC0415

        self.ctx = ctx
        self.device = torch.device(ctx.device)
        self._ref = ref

    def _params(self, temperature: float, top_k: int, top_p: float):
        return self._ref.SamplingParams(temperature=temperature, top_k=top_k, top_p=top_p)

    def sample(self, logits: torch.Tensor, params: SamplingParams, seed: int,
               position: int) -> int:
        if params.min_p != 0 or params.penalized:
            raise ValueError("the reference sampler has no min_p or penalties")
        return self._ref.sample(logits, self._params(params.temperature, params.top_k,
                                                     params.top_p), seed, position)

    def sample_batch(self, logits: torch.Tensor, params: RowParams, uniforms: torch.Tensor,
                     history: TokenHistogram | None = None, out: torch.Tensor | None = None,
                     probs_out: torch.Tensor | None = None) -> torch.Tensor:
        B, V = logits.shape
        host = {k: getattr(params, k).cpu().tolist() for k in (
            "temperature", "top_k", "top_p", "min_p", "repetition_penalty", "presence_penalty",
            "frequency_penalty")}
        u = uniforms.float().cpu().tolist()
        if history is not None:
            ptr = history.row_ptr.cpu().tolist()
            hid, hcnt = history.ids.cpu(), history.counts.cpu()
        ids = torch.empty(B, dtype=torch.int32)
        for r in range(B):
            y = logits[r].float().cpu().clone()
            rep, pres = host["repetition_penalty"][r], host["presence_penalty"][r]
            freq = host["frequency_penalty"][r]
            if history is not None and (rep != 1 or pres != 0 or freq != 0):
                t = hid[ptr[r]:ptr[r + 1]].long()
                c = hcnt[ptr[r]:ptr[r + 1]]
                keep = c > 0
                t, c = t[keep], c[keep].float()
                x = y[t]
                x = torch.where(x > 0, x / rep, x * rep)
                x = x - freq * c
                y[t] = x - pres
            T = host["temperature"][r]
            if T == 0:
                ids[r] = int(torch.argmax(y))
                if probs_out is not None:
                    probs_out[r].zero_()
                    probs_out[r, int(ids[r])] = 1.0
                continue
            p = self._ref.filtered_probs(y, self._params(T, host["top_k"][r], host["top_p"][r]))
            mp = host["min_p"][r]
            if mp > 0:
                p = torch.where(p >= mp * p.max(), p, torch.zeros_like(p))
                p = p / p.sum()
            order = torch.sort(p, descending=True, stable=True).indices
            cum = torch.cumsum(p[order].double(), 0)
            j = int(torch.searchsorted(cum, torch.tensor([u[r] * float(cum[-1])],
                                                         dtype=torch.float64), right=True))
            j = min(j, int((p[order] > 0).sum()) - 1)
            ids[r] = int(order[j])
            if probs_out is not None:
                probs_out[r] = p.to(probs_out.device)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=logits.device)
        out.copy_(ids)
        return out
