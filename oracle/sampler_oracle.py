"""CPU oracle for the token-sampling path.

TEST INFRASTRUCTURE ONLY. This module is the checker the CUDA sampler is compared against.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it;
the product path (``vinfer_b200``) never does, and fails loudly when its CUDA library is
missing instead of falling back to anything here.

It restates vinfer's reference sampler (``src/vinfer/runtime/sampler.py``, pure PyTorch) in
numpy, row by row, and extends it with the features the reference does not have but the
B200 sampler must implement. Every step states the reference line it follows, or says that it
is an extension.

Semantics (one row of ``V`` logits):

1. ``y = penalize(x)`` (extension, conventional definition): for every token id with a
   positive count ``c`` in the row's history, repetition divides a positive logit by ``rep``
   and multiplies a non-positive one by ``rep``; then ``y -= freq * c``; then ``y -= pres``.
   Every operation is one IEEE float32 operation, in that order.
2. Greedy (``temperature == 0``): the first index of ``max(y)``
   (reference ``sampler.py:70-71``; with no penalties ``y == x``).
3. ``v = y / temperature`` in float32, true division (reference ``sampler.py:52``; torch CPU
   divides, it does not multiply by a reciprocal).
4. Top-k, ``0 < k < V``: ``t = k-th largest v``; tokens with ``v < t`` are removed, every
   token tied at ``t`` is kept (reference ``sampler.py:53-55``).
5. Softmax over the kept tokens (reference ``sampler.py:56``), computed here in float64 from
   the float32 ``v`` (the exact value the float32 reference approximates).
6. Top-p, ``top_p < 1``: in canonical order, a token is dropped when the mass strictly before
   it is ``>= top_p`` (reference ``sampler.py:57-64``). Canonical order is descending ``v``,
   ties by ascending token id; the reference uses ``torch.sort``, which is not stable on CPU,
   so on rows where the cut splits a group of equal values the reference's kept set is an
   arbitrary subset of the same size (``tie_at_topp_cut`` flags those rows).
7. Min-p (extension, vLLM's definition): keep tokens whose probability is
   ``>= min_p * max probability``, i.e. ``exp(v - max v) >= min_p``.
8. Renormalise over the kept set (reference ``sampler.py:64``).
9. Draw (extension; replaces the reference's exponential race ``sampler.py:73-77``): with a
   caller uniform ``u`` in ``[0, 1)``, walk the kept tokens in canonical order and pick the
   first whose inclusive cumulative probability exceeds ``u``.

Parity is "pinned" for steps 2-6 and 8 by golden vectors generated from the reference itself
(``tests/golden/make_golden.py``); steps 1, 7 and 9 have no counterpart in the reference and
are pinned by hand-computed known-answer tests (``tests/test_oracle.py``).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32
BOUNDARY_EPS = 1e-6  # the north-star boundary rule: a margin below this is a "boundary" row


# --------------------------------------------------------------------------------------------
# seeds (reference sampler.py:44-47) and the per-position uniform (extension)
# --------------------------------------------------------------------------------------------


def position_seed(seed: int, position: int) -> int:
    """63-bit seed of ``(seed, position)``: the little-endian 8-byte blake2b digest of the
    text ``"{seed}:{position}"``, top bit cleared (reference ``sampler.py:44-47``)."""
    h = hashlib.blake2b(f"{seed}:{position}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") & ((1 << 63) - 1)


_M64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    """One SplitMix64 output for state ``x`` (Steele, Lea & Flood, OOPSLA 2014)."""
    z = (x + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def uniform_from_seed(pseed: int) -> np.float32:
    """The draw's uniform for a position seed: the top 24 bits of ``splitmix64(pseed)`` scaled
    by ``2**-24``, so it is exactly representable in float32 and lies in ``[0, 1)``."""
    return F32((splitmix64(pseed) >> 40) * (1.0 / (1 << 24)))


# --------------------------------------------------------------------------------------------
# parameters
# --------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class RowParams:
    temperature: float = 1.0  # 0 = greedy
    top_k: int = 0  # 0 = off
    top_p: float = 1.0  # 1 = off
    min_p: float = 0.0  # 0 = off
    repetition_penalty: float = 1.0  # 1 = off
    presence_penalty: float = 0.0  # 0 = off
    frequency_penalty: float = 0.0  # 0 = off


@dataclass
class RowResult:
    token: int
    probs: np.ndarray | None = None  # float32 [V]: final renormalised probabilities (None if greedy)
    kept: int = 0  # size of the final kept set
    topp_margin: float = np.inf  # distance of the top-p decision from flipping
    minp_margin: float = np.inf  # relative distance of the min-p decision from flipping
    draw_margin: float = np.inf  # distance of u from the nearest cumulative-mass edge
    tie_at_topp_cut: bool = False  # the top-p cut splits a group of equal values
    info: dict = field(default_factory=dict)

    @property
    def boundary(self) -> bool:
        return min(self.topp_margin, self.minp_margin, self.draw_margin) < BOUNDARY_EPS


# --------------------------------------------------------------------------------------------
# the row pipeline
# --------------------------------------------------------------------------------------------


def penalize(
    x: np.ndarray,
    ids: np.ndarray | None,
    counts: np.ndarray | None,
    repetition: float,
    presence: float,
    frequency: float,
) -> np.ndarray:
    """Step 1 (extension): float32 logits after repetition, frequency and presence penalties.
    History entries with a count <= 0 are ignored. Ids must be unique within a row."""
    y = np.asarray(x, dtype=F32).copy()
    if ids is None or len(ids) == 0:
        return y
    rep, pres, freq = F32(repetition), F32(presence), F32(frequency)
    ids = np.asarray(ids, dtype=np.int64)
    counts = np.asarray(counts, dtype=np.int64)
    sel = counts > 0
    ids, c = ids[sel], counts[sel].astype(F32)
    t = y[ids]
    t = np.where(t > 0, t / rep, t * rep).astype(F32)
    t = (t - (freq * c).astype(F32)).astype(F32)
    t = (t - pres).astype(F32)
    y[ids] = t
    return y


def canonical_order(v: np.ndarray) -> np.ndarray:
    """Token ids sorted by descending value, ties by ascending id (a total order)."""
    ids = np.arange(v.shape[0])
    # +0.0 and -0.0 are equal, as in the reference's comparisons: add 0 to fold -0 into +0
    return np.lexsort((ids, -(v.astype(np.float64) + 0.0)))


def process_row(
    x: np.ndarray,
    params: RowParams,
    u: float = 0.0,
    hist_ids: np.ndarray | None = None,
    hist_counts: np.ndarray | None = None,
) -> RowResult:
    """The whole path for one row: penalties → (greedy) → temperature → top-k → softmax →
    top-p → min-p → renormalise → inverse-CDF draw with ``u``."""
    x = np.asarray(x)
    V = x.shape[0]
    y = penalize(x, hist_ids, hist_counts, params.repetition_penalty, params.presence_penalty,
                 params.frequency_penalty)
    if params.temperature == 0:  # sampler.py:70-71
        return RowResult(token=int(np.argmax(y)), kept=1)

    v = (y / F32(params.temperature)).astype(F32)  # sampler.py:52
    keep = np.ones(V, dtype=bool)
    k = params.top_k
    if 0 < k < V:  # sampler.py:53-55
        kth = np.partition(v, V - k)[V - k]
        keep &= ~(v < kth)
    v64 = v.astype(np.float64)
    m = v64[keep].max()
    e = np.where(keep, np.exp(v64 - m), 0.0)  # sampler.py:56 (exact-rounding restatement)
    S = e.sum()
    p = e / S

    kept_idx = np.nonzero(keep)[0]  # kept-by-top-k tokens, then canonical order among them
    order = kept_idx[np.lexsort((kept_idx, -(v64[kept_idx] + 0.0)))]
    ps = p[order]
    n = order.shape[0]
    res = RowResult(token=-1)

    Lp, topp_margin = n, np.inf
    top_p = float(F32(params.top_p))
    if top_p < 1:  # sampler.py:57-63
        before = np.cumsum(ps) - ps
        drop = before >= top_p
        Lp = int(np.argmax(drop)) if drop.any() else n
        topp_margin = min(
            top_p - before[Lp - 1] if Lp >= 1 else np.inf,
            before[Lp] - top_p if Lp < n else np.inf,
        )
        if 0 < Lp < n:
            vs = v[order]
            res.tie_at_topp_cut = bool(vs[Lp - 1] == vs[Lp])

    Lm, minp_margin = n, np.inf
    min_p = float(F32(params.min_p))
    if min_p > 0:  # extension
        es = e[order]
        okm = es >= min_p
        Lm = max(int(np.argmin(okm)) if not okm.all() else n, 1)  # the top token always stays
        rel = np.abs(es - min_p) / min_p
        lo, hi = max(Lm - 1, 0), min(Lm + 1, n)
        minp_margin = float(rel[lo:hi].min()) if hi > lo else np.inf

    L = min(Lp, Lm)
    # a margin matters only for the cut that binds (or both, when they meet)
    res.topp_margin = topp_margin if Lp <= Lm else np.inf
    res.minp_margin = minp_margin if Lm <= Lp else np.inf

    kept_ids = order[:L]
    q = np.zeros(V, dtype=np.float64)
    q[kept_ids] = p[kept_ids] / p[kept_ids].sum()  # sampler.py:64
    res.probs = q.astype(F32)
    res.kept = L

    # inverse-CDF draw in canonical order (extension)
    c = np.cumsum(q[kept_ids])
    uu = float(F32(u))
    j = int(np.searchsorted(c, uu, side="right"))  # first j with u < c[j]
    j = min(j, L - 1)
    res.token = int(kept_ids[j])
    lo_edge = c[j - 1] if j >= 1 else None
    hi_edge = c[j] if j < L - 1 else None  # the last edge is 1 by construction
    res.draw_margin = min(
        uu - lo_edge if lo_edge is not None else np.inf,
        hi_edge - uu if hi_edge is not None else np.inf,
    )
    res.info = {"m": m, "S": S, "n_topk": n}
    return res


def filtered_probs(x: np.ndarray, params: RowParams) -> np.ndarray:
    """Probabilities after temperature, top-k, top-p (and min-p), float32 ``[V]``: the
    restatement of reference ``sampler.py:50-65`` (non-greedy rows only)."""
    if params.temperature == 0:
        raise ValueError("filtered_probs needs temperature > 0")
    return process_row(x, params).probs


# --------------------------------------------------------------------------------------------
# batches
# --------------------------------------------------------------------------------------------


@dataclass
class Batch:
    """One batch of rows in the layout the CUDA sampler reads: float32 or bf16-valued float32
    logits ``[B, V]``, per-row parameter arrays, a CSR history (row_ptr ``[B+1]``, ids sorted
    ascending within each row, counts) and one uniform per row."""

    logits: np.ndarray  # float32 [B, V] (bf16 inputs are stored here as their exact float32 values)
    temperature: np.ndarray
    top_k: np.ndarray
    top_p: np.ndarray
    min_p: np.ndarray
    repetition_penalty: np.ndarray
    presence_penalty: np.ndarray
    frequency_penalty: np.ndarray
    uniforms: np.ndarray
    hist_row_ptr: np.ndarray | None = None
    hist_ids: np.ndarray | None = None
    hist_counts: np.ndarray | None = None

    @property
    def batch(self) -> int:
        return self.logits.shape[0]

    def params(self, r: int) -> RowParams:
        return RowParams(
            temperature=float(self.temperature[r]),
            top_k=int(self.top_k[r]),
            top_p=float(self.top_p[r]),
            min_p=float(self.min_p[r]),
            repetition_penalty=float(self.repetition_penalty[r]),
            presence_penalty=float(self.presence_penalty[r]),
            frequency_penalty=float(self.frequency_penalty[r]),
        )

    def history(self, r: int) -> tuple[np.ndarray | None, np.ndarray | None]:
        if self.hist_row_ptr is None:
            return None, None
        a, b = int(self.hist_row_ptr[r]), int(self.hist_row_ptr[r + 1])
        return self.hist_ids[a:b], self.hist_counts[a:b]


def process_batch(batch: Batch, rows: list[int] | None = None) -> list[RowResult]:
    rows = range(batch.batch) if rows is None else rows
    out = []
    for r in rows:
        ids, counts = batch.history(r)
        out.append(process_row(batch.logits[r], batch.params(r), float(batch.uniforms[r]), ids,
                               counts))
    return out
