"""Seeded synthetic sampler workloads: the five benchmark configurations.

No public dataset is involved: every configuration is synthetic logits of the stated shape and
distribution, generated from ``torch.Generator().manual_seed(seed)`` (seed = configuration
number by default) so the CPU oracle and the GPU kernel see identical tensors. ``batch`` and
``vocab`` may be overridden to get a smaller case of the same distribution.

1. B=1, V=151,936, float32 N(0, 2) + 8 spikes (+12); T 0.7, top-k 20, top-p 0.8,
   repetition 1.05 over 64 uniform history tokens.
2. B=64, V=151,936, bf16 N(0, sigma), sigma ~ U[0.5, 4] per row, 1-16 spikes of +8..+15;
   per-row T in {0, 0.6, 1}, top-k in {0, 20, 50}, top-p in {1, 0.95, 0.8},
   min-p in {0, 0.05}; no penalties.
3. B=256, bf16 as 2; repetition 1.1, presence 0.5, frequency 0.3 over a 4,096-token
   Zipf(s=1.1) history per row; T 0.7, top-k 20, top-p 0.8. (The Zipf ranks map to token ids
   through one fixed seeded permutation of the vocabulary.)
4. B=1,024, V=248,320, bf16 N(0, 3) + 4 spikes (+10); T 1, top-k 50, top-p 0.9 (the
   vocab-sharded configuration).
5. B=512, V=151,936, float32 in four classes of rows (flat / one +30 token / a 1,000-way tie
   at the maximum / N(0, 1)); top-k ~ U{1..1000}, top-p ~ U[0.1, 1], T ~ U[0.1, 2];
   512-token uniform histories with repetition ~ U[1, 1.2], presence and frequency
   ~ U[0, 0.5] (the configuration names histories but no penalty values; these are chosen so
   the histories matter).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

VOCAB_QWEN3 = 151_936
VOCAB_QWEN35 = 248_320


@dataclass
class Workload:
    name: str
    logits: torch.Tensor  # [B, V], float32 or bfloat16, CPU
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
    meta: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return self.logits.shape[0]

    @property
    def vocab(self) -> int:
        return self.logits.shape[1]

    def param_arrays(self) -> dict[str, np.ndarray]:
        return {k: getattr(self, k) for k in ("temperature", "top_k", "top_p", "min_p",
                                              "repetition_penalty", "presence_penalty",
                                              "frequency_penalty")}

    @property
    def hist_nnz(self) -> int:
        return 0 if self.hist_ids is None else int(self.hist_row_ptr[-1])

    def algorithmic_bytes(self) -> int:
        """Bytes one pass must move: logits + 8 per history entry + 36 per row."""
        es = self.logits.element_size()
        return self.batch * self.vocab * es + 8 * self.hist_nnz + 36 * self.batch


def _csr(rows: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    ptr, ids, cnts = [0], [], []
    for toks in rows:
        u, c = np.unique(toks, return_counts=True)
        ids.append(u.astype(np.int32))
        cnts.append(c.astype(np.int32))
        ptr.append(ptr[-1] + len(u))
    return np.array(ptr, np.int64), np.concatenate(ids), np.concatenate(cnts)


def _pick(g: torch.Generator, choices: list[float], n: int) -> np.ndarray:
    idx = torch.randint(len(choices), (n,), generator=g).numpy()
    return np.asarray(choices, dtype=np.float64)[idx]


def _spiky(g: torch.Generator, B: int, V: int, dtype: torch.dtype) -> torch.Tensor:
    sigma = torch.rand(B, 1, generator=g) * 3.5 + 0.5
    x = torch.randn(B, V, generator=g) * sigma
    for r in range(B):
        ns = int(torch.randint(1, 17, (1,), generator=g))
        ids = torch.randperm(V, generator=g)[:ns]
        x[r, ids] += torch.randint(8, 16, (ns,), generator=g).float()
    return x.to(dtype)


def _zipf_histories(g: torch.Generator, B: int, V: int, n: int, s: float) -> list[np.ndarray]:
    ranks = torch.arange(1, V + 1, dtype=torch.float64)
    cdf = torch.cumsum(ranks.pow(-s), 0)
    cdf /= cdf[-1].clone()
    perm = torch.randperm(V, generator=g)
    out = []
    for _ in range(B):
        u = torch.rand(n, generator=g, dtype=torch.float64)
        r = torch.searchsorted(cdf, u).clamp_(max=V - 1)
        out.append(perm[r].numpy().astype(np.int64))
    return out


def make(config: int, batch: int | None = None, vocab: int | None = None,
         seed: int | None = None) -> Workload:
    g = torch.Generator().manual_seed(config if seed is None else seed)
    f32 = (lambda a: np.asarray(a, np.float32))
    if config == 1:
        B, V = batch or 1, vocab or VOCAB_QWEN3
        x = torch.randn(B, V, generator=g) * 2.0
        for r in range(B):
            x[r, torch.randperm(V, generator=g)[:8]] += 12.0
        hist = [torch.randint(V, (64,), generator=g).numpy() for _ in range(B)]
        ptr, ids, cnt = _csr(hist)
        w = Workload("config1", x, f32([0.7] * B), np.full(B, 20, np.int32), f32([0.8] * B),
                     f32([0.0] * B), f32([1.05] * B), f32([0.0] * B), f32([0.0] * B),
                     f32(torch.rand(B, generator=g).numpy()), ptr, ids, cnt)
    elif config == 2:
        B, V = batch or 64, vocab or VOCAB_QWEN3
        x = _spiky(g, B, V, torch.bfloat16)
        w = Workload("config2", x, f32(_pick(g, [0.0, 0.6, 1.0], B)),
                     _pick(g, [0, 20, 50], B).astype(np.int32), f32(_pick(g, [1.0, 0.95, 0.8], B)),
                     f32(_pick(g, [0.0, 0.05], B)), f32([1.0] * B), f32([0.0] * B),
                     f32([0.0] * B), f32(torch.rand(B, generator=g).numpy()))
    elif config == 3:
        B, V = batch or 256, vocab or VOCAB_QWEN3
        x = _spiky(g, B, V, torch.bfloat16)
        ptr, ids, cnt = _csr(_zipf_histories(g, B, V, 4096, 1.1))
        w = Workload("config3", x, f32([0.7] * B), np.full(B, 20, np.int32), f32([0.8] * B),
                     f32([0.0] * B), f32([1.1] * B), f32([0.5] * B), f32([0.3] * B),
                     f32(torch.rand(B, generator=g).numpy()), ptr, ids, cnt)
    elif config == 4:
        B, V = batch or 1024, vocab or VOCAB_QWEN35
        x = torch.empty(B, V, dtype=torch.bfloat16)
        for r0 in range(0, B, 64):
            r1 = min(B, r0 + 64)
            blk = torch.randn(r1 - r0, V, generator=g) * 3.0
            for r in range(r1 - r0):
                blk[r, torch.randperm(V, generator=g)[:4]] += 10.0
            x[r0:r1] = blk.to(torch.bfloat16)
        w = Workload("config4", x, f32([1.0] * B), np.full(B, 50, np.int32), f32([0.9] * B),
                     f32([0.0] * B), f32([1.0] * B), f32([0.0] * B), f32([0.0] * B),
                     f32(torch.rand(B, generator=g).numpy()))
    elif config == 5:
        B, V = batch or 512, vocab or VOCAB_QWEN3
        x = torch.randn(B, V, generator=g)
        cls = np.arange(B) * 4 // B  # four contiguous classes
        for r in range(B):
            if cls[r] == 0:
                x[r] = float(torch.randn(1, generator=g))
            elif cls[r] == 1:
                x[r, int(torch.randint(V, (1,), generator=g))] += 30.0
            elif cls[r] == 2:
                x[r, torch.randperm(V, generator=g)[: min(1000, V)]] = x[r].max() + 1.0
        kmax = min(1000, V)
        hist = [torch.randint(V, (512,), generator=g).numpy() for _ in range(B)]
        ptr, ids, cnt = _csr(hist)
        w = Workload("config5", x, f32((torch.rand(B, generator=g) * 1.9 + 0.1).numpy()),
                     torch.randint(1, kmax + 1, (B,), generator=g).numpy().astype(np.int32),
                     f32((torch.rand(B, generator=g) * 0.9 + 0.1).numpy()), f32([0.0] * B),
                     f32((1.0 + 0.2 * torch.rand(B, generator=g)).numpy()),
                     f32((0.5 * torch.rand(B, generator=g)).numpy()),
                     f32((0.5 * torch.rand(B, generator=g)).numpy()),
                     f32(torch.rand(B, generator=g).numpy()), ptr, ids, cnt)
        w.meta["row_class"] = cls
    else:
        raise ValueError(f"unknown configuration {config} (1..5)")
    w.meta["config"] = config
    return w


def config4_shard(rank: int, world: int, device: torch.device, batch: int = 1024,
                  vocab: int = 248_320, seed: int = 4):
    """This rank's shard of configuration 4, generated on the device: N(0, 3) logits with 4
    spikes of +10 per row at seeded global ids (the same ids on every rank), temperature 1,
    top-k 50, top-p 0.9, one seeded uniform per row shared by all ranks. The values follow the
    configuration's distribution; they are not the CPU generator's values."""
    from vinfer_b200.sampling import RowParams  # noqa: PLC0415

    lo, hi = vocab * rank // world, vocab * (rank + 1) // world
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000 + rank)
    x = torch.randn(batch, hi - lo, generator=g, device=device, dtype=torch.float32) * 3.0
    gc = torch.Generator().manual_seed(seed)
    spikes = torch.randint(vocab, (batch, 4), generator=gc)
    uniforms = torch.rand(batch, generator=gc)
    r, c = torch.nonzero((spikes >= lo) & (spikes < hi), as_tuple=True)
    x[r.to(device), (spikes[r, c] - lo).to(device)] += 10.0
    x = x.to(torch.bfloat16)
    f = np.float32
    params = RowParams.from_arrays(
        device, temperature=np.full(batch, 1.0, f), top_k=np.full(batch, 50, np.int32),
        top_p=np.full(batch, 0.9, f), min_p=np.zeros(batch, f),
        repetition_penalty=np.ones(batch, f), presence_penalty=np.zeros(batch, f),
        frequency_penalty=np.zeros(batch, f))
    return x, params, uniforms.to(device)
