"""Vocab-sharded sampling: one process per GPU, each holding a contiguous slice of the vocabulary.

This is the layout a tensor-parallel ``lm_head`` produces (``src/vinfer/models/qwen/model.py:
230-233`` computes the full ``[T, V]`` logits on one device today; sharded, rank r holds ids
``[r*V/w, (r+1)*V/w)``). One batch takes these steps on every rank, in the same order:

1. ``vinfer_sample_local`` reduces the rank's shard of each row to a fixed-size candidate record
   (penalised, temperature-scaled top-k' entries with global ids, plus the shard's maximum and
   softmax sum for rows without top-k);
2. one ``all_gather_into_tensor`` (NCCL over NVLink / NVSwitch) exchanges the records;
3. ``vinfer_sample_merge`` merges the ``world`` records of each row and applies the final top-k /
   top-p / min-p cut and the inverse-CDF draw with the row's uniform. Every rank computes the
   same ids from the same records, so nothing is broadcast;
4. a row whose cut or draw lies beyond the gathered candidates (possible only without top-k) is
   flagged; its shards are all-gathered into the full row and sampled with ``vinfer_sample``.
   Every rank takes this step for the same rows, so the collectives stay matched.

The device steps sit behind a small ``kernels`` object (``B200ShardKernels`` here) so that the
orchestration -- collective order, buffer layout, the fallback's row assembly -- runs and is
tested on CPU ranks with ``gloo`` and a stand-in for the kernels.
"""

from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from vinfer_b200 import _lib
from vinfer_b200.sampling import RowParams, TokenHistogram

PARAM_NAMES = ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
               "presence_penalty", "frequency_penalty")


def shard_range(vocab_total: int, world: int, rank: int) -> tuple[int, int]:
    """Ids ``[lo, hi)`` owned by ``rank`` when ``vocab_total`` is split contiguously."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return vocab_total * rank // world, vocab_total * (rank + 1) // world


def select_rows(params: RowParams, uniforms: torch.Tensor, history: TokenHistogram | None,
                idx: torch.Tensor) -> tuple[RowParams, torch.Tensor, TokenHistogram | None]:
    """Parameters, uniforms and histories of the rows ``idx`` (in that order)."""
    sub = RowParams(**{k: getattr(params, k).index_select(0, idx).contiguous()
                       for k in PARAM_NAMES})
    u = uniforms.index_select(0, idx).contiguous()
    if history is None:
        return sub, u, None
    rp = history.row_ptr
    start = rp.index_select(0, idx)
    lens = rp.index_select(0, idx + 1) - start
    ptr = torch.zeros(idx.numel() + 1, dtype=rp.dtype, device=rp.device)
    ptr[1:] = torch.cumsum(lens, 0)
    total = int(ptr[-1])
    pos = torch.arange(total, dtype=rp.dtype, device=rp.device)
    src = torch.repeat_interleave(start, lens, output_size=total) + pos - torch.repeat_interleave(
        ptr[:-1], lens, output_size=total)
    ids = history.ids.index_select(0, src).contiguous()
    counts = history.counts.index_select(0, src).contiguous()
    if total == 0:  # a zero-length array still needs a valid device pointer for the C ABI
        ids, counts = history.ids.new_zeros(1), history.counts.new_zeros(1)
    return sub, u, TokenHistogram(ptr, ids, counts)


class B200ShardKernels:
    """The device steps of a sharded batch, through the sampler's C ABI."""

    def __init__(self, backend) -> None:
        self.backend = backend
        self.lib = backend.lib

    def record_bytes(self, record_cap: int) -> int:
        n = self.lib.vinfer_sample_record_bytes(record_cap)
        if n == 0:
            raise ValueError(f"record_cap {record_cap} is out of range")
        return n

    def _args(self, logits, params, uniforms, history, out, probs_out, voff, vtotal):
        return self.backend.args(logits, params, uniforms, history, out, probs_out,
                                 vocab_offset=voff, vocab_total=vtotal)

    def local(self, logits, params, uniforms, history, voff, vtotal, record_cap, records,
              scratch_ids) -> None:
        a = self._args(logits, params, uniforms, history, scratch_ids, None, voff, vtotal)
        ws = self.backend.workspace(logits.shape[0], logits.shape[1], a.dtype)
        _lib.check(self.lib.vinfer_sample_local(C.byref(a), record_cap, records.data_ptr(),
                                                ws.data_ptr(), ws.numel(),
                                                self.backend._stream()), "vinfer_sample_local")

    def merge(self, logits, params, uniforms, history, voff, vtotal, record_cap, gathered,
              world, out, unresolved, probs_out) -> None:
        a = self._args(logits, params, uniforms, history, out, probs_out, voff, vtotal)
        ws = self.backend.workspace(logits.shape[0], logits.shape[1], a.dtype)
        _lib.check(self.lib.vinfer_sample_merge(C.byref(a), record_cap, gathered.data_ptr(),
                                                world, unresolved.data_ptr(), ws.data_ptr(),
                                                ws.numel(), self.backend._stream()),
                   "vinfer_sample_merge")

    def full(self, logits, params, uniforms, history, out, probs_out) -> None:
        self.backend.sample_batch(logits, params, uniforms, history, out=out,
                                  probs_out=probs_out)

    def check(self) -> None:
        self.backend.check()


class ShardedSampler:
    """Samples rows whose vocabulary is split over the ranks of ``group``.

    ``sample_batch`` must be called by every rank of the group with its own shard and identical
    parameters, uniforms and histories (histories carry global token ids; each rank applies the
    entries that fall in its shard). Every rank gets the same ids.
    """

    def __init__(self, kernels, group=None, record_cap: int = 64) -> None:
        self.kernels = kernels
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.record_cap = record_cap
        self.rec_bytes = kernels.record_bytes(record_cap)
        self._bufs: dict = {}
        self._totals: dict = {}
        self.last_unresolved = 0

    def _buffers(self, B: int, device: torch.device):
        key = (B, str(device))
        b = self._bufs.get(key)
        if b is None:
            n = B * self.rec_bytes
            b = {"local": torch.empty(n, dtype=torch.uint8, device=device),
                 "gathered": torch.empty(self.world * n, dtype=torch.uint8, device=device),
                 "unresolved": torch.zeros(B, dtype=torch.int32, device=device),
                 "scratch_ids": torch.empty(B, dtype=torch.int32, device=device)}
            self._bufs[key] = b
        return b

    def sample_batch(self, logits: torch.Tensor, params: RowParams, uniforms: torch.Tensor,
                     history: TokenHistogram | None, vocab_total: int,
                     out: torch.Tensor | None = None,
                     probs_out: torch.Tensor | None = None) -> torch.Tensor:
        """Sample one global token id per row from this rank's shard ``logits [B, V/w]``.

        ``probs_out`` (optional, ``[B, V/w]`` float32) receives this rank's slice of the final
        probabilities. The device steps (``sample_batch_async``), then one read of the
        unresolved flags and, for the rare unresolved rows, the full-row fallback."""
        out = self.sample_batch_async(logits, params, uniforms, history, vocab_total, out,
                                      probs_out)
        buf = self._buffers(logits.shape[0], logits.device)
        # identical on every rank: all ranks take the fallback for the same rows. One boolean
        # read per step (the count only when some row is unresolved, which is rare).
        n = 0
        if bool(buf["unresolved"].any()):
            n = int(torch.count_nonzero(buf["unresolved"]))
        self.last_unresolved = n
        if n:
            self._resolve(logits, params, uniforms, history, vocab_total, out, probs_out,
                          torch.nonzero(buf["unresolved"]).flatten())
        return out

    def sample_batch_async(self, logits: torch.Tensor, params: RowParams,
                           uniforms: torch.Tensor, history: TokenHistogram | None,
                           vocab_total: int, out: torch.Tensor | None = None,
                           probs_out: torch.Tensor | None = None) -> torch.Tensor:
        """The device steps of ``sample_batch`` alone (local records, all-gather, merge), with
        no host synchronisation, so that they can be captured in a CUDA graph. Rows the records
        cannot decide are left at -1 in ``out`` and counted into ``unresolved_total`` (a device
        tensor; ``pending_unresolved`` reads and clears it): a caller that cannot rule them out
        takes ``sample_batch`` instead."""
        B, Vr = logits.shape
        lo, hi = shard_range(vocab_total, self.world, self.rank)
        if Vr != hi - lo:
            raise ValueError(f"rank {self.rank} holds {Vr} columns; the contiguous split of "
                             f"{vocab_total} over {self.world} ranks gives it {hi - lo}")
        dev = logits.device
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        buf = self._buffers(B, dev)
        self.kernels.local(logits, params, uniforms, history, lo, vocab_total, self.record_cap,
                           buf["local"], buf["scratch_ids"])
        dist.all_gather_into_tensor(buf["gathered"], buf["local"], group=self.group)
        self.kernels.merge(logits, params, uniforms, history, lo, vocab_total, self.record_cap,
                           buf["gathered"], self.world, out, buf["unresolved"], probs_out)
        self._total(dev).add_(buf["unresolved"].sum())
        return out

    def _total(self, device: torch.device) -> torch.Tensor:
        t = self._totals.get(str(device))
        if t is None:
            t = torch.zeros((), dtype=torch.int64, device=device)
            self._totals[str(device)] = t
        return t

    def pending_unresolved(self, device: torch.device) -> int:
        """Rows left unresolved by ``sample_batch_async`` calls since the last read (one
        synchronising read); then zero."""
        t = self._total(device)
        n = int(t.item())
        t.zero_()
        return n

    def _resolve(self, logits, params, uniforms, history, vocab_total, out, probs_out, idx):
        """Assemble the full rows ``idx`` from every rank's shard and sample them unsharded.

        Ends with a status all-reduce that every rank reaches, so that a rank failing here after
        the rows' all-gather makes every rank raise (the ranks would otherwise go on with
        different ids). A rank failing before the all-gather leaves the others in it until the
        process group's timeout ends it with an error."""
        failed = None
        try:
            self._resolve_rows(logits, params, uniforms, history, vocab_total, out, probs_out,
                               idx)
        except Exception as exc:  # noqa: BLE001 -- reported to every rank below, then re-raised
            failed = exc
        status = torch.tensor([0 if failed is None else 1], dtype=torch.int32,
                              device=logits.device)
        dist.all_reduce(status, group=self.group)
        if failed is not None:
            raise failed
        if int(status.item()):
            raise RuntimeError(f"{int(status.item())} rank(s) failed while resolving rows "
                               f"{idx.tolist()} from the full vocabulary")

    def _resolve_rows(self, logits, params, uniforms, history, vocab_total, out, probs_out,
                      idx):
        n, dev = idx.numel(), logits.device
        width = max(hi - lo for lo, hi in
                    (shard_range(vocab_total, self.world, r) for r in range(self.world)))
        mine = torch.zeros(n, width, dtype=logits.dtype, device=dev)
        mine[:, :logits.shape[1]] = logits.index_select(0, idx)
        parts = torch.empty(self.world * n, width, dtype=logits.dtype, device=dev)
        dist.all_gather_into_tensor(parts, mine, group=self.group)
        parts = parts.view(self.world, n, width)
        full = torch.cat([parts[r, :, :hi - lo] for r, (lo, hi) in enumerate(
            shard_range(vocab_total, self.world, r) for r in range(self.world))], dim=1)
        sub_p, sub_u, sub_h = select_rows(params, uniforms, history, idx)
        ids = torch.empty(n, dtype=torch.int32, device=dev)
        full_probs = (torch.empty(n, vocab_total, dtype=torch.float32, device=dev)
                      if probs_out is not None else None)
        self.kernels.full(full.contiguous(), sub_p, sub_u, sub_h, ids, full_probs)
        out.index_copy_(0, idx, ids)
        if probs_out is not None:
            lo, hi = shard_range(vocab_total, self.world, self.rank)
            probs_out.index_copy_(0, idx, full_probs[:, lo:hi])
