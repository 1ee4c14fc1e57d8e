"""Sampling parameters, per-position seeds and the host-side packing of a batch.

``SamplingParams`` keeps every field, default and validation message of vinfer's
(``src/vinfer/runtime/sampler.py:18-41``) and adds the four the B200 sampler implements beyond
the reference: ``min_p`` and the repetition / presence / frequency penalties, all defaulting
to "off". ``position_seed`` is the reference's (``sampler.py:44-47``); the draw's uniform for
a position is derived from it with SplitMix64, so ``sample(logits, params, seed, position)``
is reproducible from ``(seed, position)`` alone, as in the reference.
"""

from __future__ import annotations

import hashlib
from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 1.0  # 0 = greedy
    top_k: int = 0  # 0 = off
    top_p: float = 1.0  # 1 = off
    seed: int | None = None  # None: the runtime picks one per request
    stop: tuple[str, ...] = ()
    stop_token_ids: tuple[int, ...] = ()
    ignore_eos: bool = False
    # extensions (no counterpart in the reference)
    min_p: float = 0.0  # 0 = off
    repetition_penalty: float = 1.0  # 1 = off
    presence_penalty: float = 0.0  # 0 = off
    frequency_penalty: float = 0.0  # 0 = off

    def __post_init__(self) -> None:
        if self.temperature < 0:
            raise ValueError(f"temperature must be >= 0, got {self.temperature}")
        if not 0 < self.top_p <= 1:
            raise ValueError(f"top_p must be in (0, 1], got {self.top_p}")
        if self.top_k < 0:
            raise ValueError(f"top_k must be >= 0, got {self.top_k}")
        if self.max_tokens < 1:
            raise ValueError(f"max_tokens must be >= 1, got {self.max_tokens}")
        if not 0 <= self.min_p <= 1:
            raise ValueError(f"min_p must be in [0, 1], got {self.min_p}")
        if not self.repetition_penalty > 0:
            raise ValueError(f"repetition_penalty must be > 0, got {self.repetition_penalty}")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0

    @property
    def penalized(self) -> bool:
        return (self.repetition_penalty != 1 or self.presence_penalty != 0
                or self.frequency_penalty != 0)


def position_seed(seed: int, position: int) -> int:
    """A 63-bit seed derived from ``(seed, position)`` (stable across runs and platforms)."""
    digest = hashlib.blake2b(f"{seed}:{position}".encode(), digest_size=8).digest()
    return int.from_bytes(digest, "little") & ((1 << 63) - 1)


_MASK64 = (1 << 64) - 1


def _splitmix64(state: int) -> int:
    """SplitMix64 (Steele, Lea & Flood, OOPSLA 2014), one output."""
    z = (state + 0x9E3779B97F4A7C15) & _MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK64
    return z ^ (z >> 31)


def position_uniform(seed: int, position: int) -> float:
    """The draw's uniform in ``[0, 1)`` for ``(seed, position)``: 24 bits, exact in float32."""
    return (_splitmix64(position_seed(seed, position)) >> 40) * (1.0 / (1 << 24))


@dataclass
class RowParams:
    """Per-row parameters as device arrays (struct of arrays), the layout the kernel reads."""

    temperature: torch.Tensor  # float32 [B]
    top_k: torch.Tensor  # int32 [B]
    top_p: torch.Tensor  # float32 [B]
    min_p: torch.Tensor  # float32 [B]
    repetition_penalty: torch.Tensor  # float32 [B]
    presence_penalty: torch.Tensor  # float32 [B]
    frequency_penalty: torch.Tensor  # float32 [B]

    @property
    def batch(self) -> int:
        return self.temperature.shape[0]

    @classmethod
    def pack(cls, params: Sequence[SamplingParams], device: torch.device | str) -> RowParams:
        f = np.array([[p.temperature, p.top_p, p.min_p, p.repetition_penalty,
                       p.presence_penalty, p.frequency_penalty] for p in params],
                     dtype=np.float32).reshape(len(params), 6)
        k = np.array([p.top_k for p in params], dtype=np.int32)
        ft = torch.from_numpy(f).to(device)
        return cls(ft[:, 0].contiguous(), torch.from_numpy(k).to(device), ft[:, 1].contiguous(),
                   ft[:, 2].contiguous(), ft[:, 3].contiguous(), ft[:, 4].contiguous(),
                   ft[:, 5].contiguous())

    @classmethod
    def from_arrays(cls, device: torch.device | str, **arrays: np.ndarray) -> RowParams:
        def f32(name: str, default: float, n: int) -> torch.Tensor:
            a = arrays.get(name)
            a = np.full(n, default, np.float32) if a is None else np.asarray(a, np.float32)
            return torch.from_numpy(np.ascontiguousarray(a)).to(device)

        n = len(arrays["temperature"])
        k = arrays.get("top_k")
        k = np.zeros(n, np.int32) if k is None else np.asarray(k, np.int32)
        return cls(f32("temperature", 1.0, n), torch.from_numpy(np.ascontiguousarray(k)).to(device),
                   f32("top_p", 1.0, n), f32("min_p", 0.0, n), f32("repetition_penalty", 1.0, n),
                   f32("presence_penalty", 0.0, n), f32("frequency_penalty", 0.0, n))


@dataclass
class TokenHistogram:
    """Per-row token counts in CSR form: ids strictly ascending within a row."""

    row_ptr: torch.Tensor  # int64 [B + 1]
    ids: torch.Tensor  # int32 [nnz]
    counts: torch.Tensor  # int32 [nnz]

    @classmethod
    def from_token_lists(cls, rows: Sequence[Sequence[int]],
                         device: torch.device | str) -> TokenHistogram:
        ptr = [0]
        ids: list[np.ndarray] = []
        cnts: list[np.ndarray] = []
        for toks in rows:
            u, c = np.unique(np.asarray(toks, dtype=np.int64), return_counts=True)
            ids.append(u.astype(np.int32))
            cnts.append(c.astype(np.int32))
            ptr.append(ptr[-1] + len(u))
        cat = (lambda xs: np.concatenate(xs) if xs else np.zeros(0, np.int32))
        return cls.from_csr(np.array(ptr, np.int64), cat(ids), cat(cnts), device)

    @classmethod
    def from_csr(cls, row_ptr: np.ndarray, ids: np.ndarray, counts: np.ndarray,
                 device: torch.device | str) -> TokenHistogram:
        row_ptr = np.asarray(row_ptr, np.int64)
        ids = np.asarray(ids, np.int32)
        for r in range(len(row_ptr) - 1):
            seg = ids[row_ptr[r]:row_ptr[r + 1]]
            if len(seg) > 1 and not np.all(seg[1:] > seg[:-1]):
                raise ValueError(f"histogram ids of row {r} must be strictly ascending")
        t = (lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device))
        # a zero-length tensor still needs a valid device pointer for the C ABI
        if len(ids) == 0:
            ids, counts = np.zeros(1, np.int32), np.zeros(1, np.int32)
        return cls(t(row_ptr), t(ids), t(np.asarray(counts, np.int32)))


HIST_PAD_ID = 0x7FFFFFFF  # VINFER_HIST_PAD_ID


@dataclass
class SlotHistogram:
    """Per-slot token counts kept on the device across decode steps (``vinfer_hist_*``).

    Slot ``s`` owns entries ``[s * cap, (s + 1) * cap)`` of ``ids`` / ``counts``: its first
    ``lens[s]`` entries are its tokens (ids strictly ascending, counts > 0), the others padding
    (count 0, ids ascending above every vocabulary id). ``history`` is therefore a CSR
    ``TokenHistogram`` the sampler reads as it is, and the backend's ``append_tokens`` updates
    it in place from the ids a step sampled, without leaving the device. The slots play the
    role of vinfer's per-request state slots (``src/vinfer/state/pool.py:70-82``).
    """

    cap: int
    ids: torch.Tensor  # int32 [slots * cap]
    counts: torch.Tensor  # int32 [slots * cap]
    lens: torch.Tensor  # int32 [slots]
    row_ptr: torch.Tensor  # int64 [slots + 1], s * cap

    @property
    def slots(self) -> int:
        return self.lens.shape[0]

    @property
    def history(self) -> TokenHistogram:
        return TokenHistogram(self.row_ptr, self.ids, self.counts)

    @staticmethod
    def host_layout(rows: Sequence[Sequence[int]], cap: int
                    ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(ids, counts, lens) of the slotted layout for the given token lists, on the host."""
        if cap < 1:
            raise ValueError("cap must be at least 1")
        n = len(rows)
        pos = np.arange(cap, dtype=np.int64)
        pad = (HIST_PAD_ID - (cap - 1 - pos)).astype(np.int32)
        ids = np.tile(pad, n)
        counts = np.zeros(n * cap, np.int32)
        lens = np.zeros(n, np.int32)
        for s, toks in enumerate(rows):
            u, c = np.unique(np.asarray(toks, dtype=np.int64), return_counts=True)
            if len(u) > cap:
                raise ValueError(f"slot {s} has {len(u)} distinct tokens, more than cap {cap}")
            if len(u) and (u[0] < 0 or u[-1] >= HIST_PAD_ID - cap):
                raise ValueError(f"slot {s} has a token id outside the vocabulary range")
            ids[s * cap:s * cap + len(u)] = u
            counts[s * cap:s * cap + len(u)] = c
            lens[s] = len(u)
        return ids, counts, lens

    @classmethod
    def from_token_lists(cls, rows: Sequence[Sequence[int]], cap: int,
                         device: torch.device | str) -> SlotHistogram:
        ids, counts, lens = cls.host_layout(rows, cap)
        t = (lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device))
        row_ptr = np.arange(len(rows) + 1, dtype=np.int64) * cap
        return cls(cap, t(ids), t(counts), t(lens), t(row_ptr))

    @classmethod
    def from_csr(cls, row_ptr: np.ndarray, ids: np.ndarray, counts: np.ndarray, cap: int,
                 device: torch.device | str) -> SlotHistogram:
        """Slots holding the rows of a CSR history (ids ascending within a row)."""
        row_ptr = np.asarray(row_ptr, np.int64)
        n = len(row_ptr) - 1
        lens = np.diff(row_ptr).astype(np.int32)
        if n and lens.max() > cap:
            raise ValueError(f"a row has {lens.max()} entries, more than cap {cap}")
        pos = np.arange(cap, dtype=np.int64)
        sid = np.tile((HIST_PAD_ID - (cap - 1 - pos)).astype(np.int32), n)
        sc = np.zeros(n * cap, np.int32)
        for r in range(n):
            a, b = row_ptr[r], row_ptr[r + 1]
            sid[r * cap:r * cap + (b - a)] = ids[a:b]
            sc[r * cap:r * cap + (b - a)] = counts[a:b]
        t = (lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device))
        return cls(cap, t(sid), t(sc), t(lens), t(np.arange(n + 1, dtype=np.int64) * cap))

    def to_counts(self) -> list[dict[int, int]]:
        """Each slot's {token: count}, read back to the host (synchronises)."""
        ids, counts, lens = (x.cpu().numpy() for x in (self.ids, self.counts, self.lens))
        out = []
        for s in range(self.slots):
            a = s * self.cap
            out.append({int(i): int(c) for i, c in zip(ids[a:a + lens[s]], counts[a:a + lens[s]])})
        return out
