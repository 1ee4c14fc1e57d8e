"""The ``b200`` sampler backend: the fused sm_100a kernel behind the C ABI.

Registered with ``devices={"cuda"}``, ``dtypes={bfloat16, float32}`` and a ``supports``
check for compute capability 10.0 and a loadable library, so resolving it anywhere else fails
with the reason (``src/vinfer/kernels/registry.py:84-88``), never by falling back.
"""

from __future__ import annotations

import ctypes as C

import torch

from vinfer_b200 import _lib
from vinfer_b200.kernels.sampler.base import SAMPLER
from vinfer_b200.registry import BackendContext
from vinfer_b200.sampling import (
    RowParams,
    SamplingParams,
    SlotHistogram,
    TokenHistogram,
    position_uniform,
)

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _supports(ctx: BackendContext) -> str | None:
    if not torch.cuda.is_available():
        return "needs a CUDA device (none is available)"
    cc = torch.cuda.get_device_capability(ctx.device)
    if cc != (10, 0):
        return f"needs compute capability 10.0 (B200, sm_100a); device has {cc[0]}.{cc[1]}"
    try:
        _lib.load()
    except (RuntimeError, OSError) as exc:
        return str(exc)
    return None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


@SAMPLER.register("b200", devices={"cuda"}, dtypes={torch.bfloat16, torch.float32},
                  supports=_supports)
class B200Sampler:
    """Fused single-pass sampler. One instance per device; calls on one instance are
    stream-ordered on the current stream and must not overlap (they share a workspace)."""

    def __init__(self, ctx: BackendContext) -> None:
        self.ctx = ctx
        self.device = torch.device(ctx.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.lib = _lib.load()
        self._workspaces: dict[tuple[int, int, int], torch.Tensor] = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    # ---- workspace ---------------------------------------------------------------------------
    def workspace(self, batch: int, vocab: int, dtype: int) -> torch.Tensor:
        key = (batch, vocab, dtype)
        ws = self._workspaces.get(key)
        if ws is None:
            nbytes = self.lib.vinfer_sampler_workspace_bytes(batch, vocab, dtype)
            if nbytes == 0:
                raise ValueError(f"unsupported shape: batch {batch}, vocab {vocab}")
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            _lib.check(self.lib.vinfer_sampler_workspace_init(ws.data_ptr(), nbytes,
                                                              self._stream()), "workspace init")
            self._workspaces[key] = ws
        return ws

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    # ---- argument packing ----------------------------------------------------------------------
    def args(self, logits: torch.Tensor, params: RowParams, uniforms: torch.Tensor | None,
             history: TokenHistogram | None, out: torch.Tensor, probs_out: torch.Tensor | None,
             exact: bool = False, vocab_offset: int = 0,
             vocab_total: int | None = None) -> _lib.SampleArgs:
        if logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("logits must be [batch, vocab] with unit column stride")
        if logits.dtype not in _DTYPES:
            raise ValueError(f"logits dtype {logits.dtype} is not supported (float32, bfloat16)")
        if logits.device != self.device:
            raise ValueError(f"logits are on {logits.device}, backend on {self.device}")
        B, V = logits.shape
        for name in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
                     "presence_penalty", "frequency_penalty"):
            t = getattr(params, name)
            want = torch.int32 if name == "top_k" else torch.float32
            if t.shape != (B,) or t.dtype != want or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"params.{name} must be a contiguous {want} [{B}] on {self.device}")
        if uniforms is not None and (uniforms.shape != (B,) or uniforms.dtype != torch.float32
                                     or uniforms.device != self.device):
            raise ValueError(f"uniforms must be float32 [{B}] on {self.device}")
        if out.shape != (B,) or out.dtype != torch.int32 or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous int32 [{B}]")
        if probs_out is not None and (probs_out.shape != (B, V) or probs_out.dtype != torch.float32
                                      or not probs_out.is_contiguous()):
            raise ValueError(f"probs_out must be a contiguous float32 [{B}, {V}]")
        a = _lib.SampleArgs()
        a.logits = logits.data_ptr()
        a.dtype = _DTYPES[logits.dtype]
        a.flags = _lib.FLAG_EXACT_ALL if exact else 0
        a.batch, a.vocab, a.ld = B, V, logits.stride(0)
        a.vocab_offset = vocab_offset
        a.vocab_total = V if vocab_total is None else vocab_total
        a.temperature = _ptr(params.temperature)
        a.top_k = _ptr(params.top_k)
        a.top_p = _ptr(params.top_p)
        a.min_p = _ptr(params.min_p)
        a.repetition_penalty = _ptr(params.repetition_penalty)
        a.presence_penalty = _ptr(params.presence_penalty)
        a.frequency_penalty = _ptr(params.frequency_penalty)
        if history is not None:
            if history.row_ptr.shape != (B + 1,):
                raise ValueError(f"history.row_ptr must be int64 [{B + 1}]")
            a.hist_row_ptr = _ptr(history.row_ptr)
            a.hist_ids = _ptr(history.ids)
            a.hist_counts = _ptr(history.counts)
        a.uniforms = _ptr(uniforms)
        a.out_ids = out.data_ptr()
        a.out_probs = _ptr(probs_out)
        a.status = self.status.data_ptr()
        return a

    # ---- SamplerBackend ------------------------------------------------------------------------
    def sample_batch(self, logits: torch.Tensor, params: RowParams, uniforms: torch.Tensor,
                     history: TokenHistogram | None = None, out: torch.Tensor | None = None,
                     probs_out: torch.Tensor | None = None, exact: bool = False,
                     logprobs_out: torch.Tensor | None = None) -> torch.Tensor:
        """Sample one id per row into ``out``. ``logprobs_out`` (float32 [B], optional)
        receives each sampled token's log-probability under the row's final distribution
        (0 for greedy rows, NaN for rows without a result)."""
        B, V = logits.shape
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        if logprobs_out is not None and (logprobs_out.shape != (B,) or
                                         logprobs_out.dtype != torch.float32 or
                                         logprobs_out.device != self.device or
                                         not logprobs_out.is_contiguous()):
            raise ValueError(f"logprobs_out must be a contiguous float32 [{B}] on {self.device}")
        a = self.args(logits, params, uniforms, history, out, probs_out, exact)
        ws = self.workspace(B, V, a.dtype)
        _lib.check(self.lib.vinfer_sample(C.byref(a), ws.data_ptr(), ws.numel(), self._stream()),
                   "vinfer_sample")
        if logprobs_out is not None:
            _lib.check(self.lib.vinfer_sample_logprobs(C.byref(a), logprobs_out.data_ptr(),
                                                       ws.data_ptr(), ws.numel(),
                                                       self._stream()), "vinfer_sample_logprobs")
        return out

    def top_logprobs(self, logits: torch.Tensor, params: RowParams, uniforms: torch.Tensor,
                     history: TokenHistogram | None, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The ``n`` most likely tokens of each row's final distribution and their
        log-probabilities (``[B, n]`` int32 ids, float32 log-probabilities; -inf outside the
        kept set, id -1 for an empty slot). Call right after ``sample_batch`` on the same
        inputs: it prices tokens with the row results that call left."""
        B, V = logits.shape
        if not 1 <= n <= _lib.TOP_LOGPROBS_MAX or n >= V:
            raise ValueError(f"n must be in [1, {_lib.TOP_LOGPROBS_MAX}] and below the vocabulary")
        ids = torch.empty(B, n, dtype=torch.int32, device=self.device)
        lp = torch.empty(B, n, dtype=torch.float32, device=self.device)
        scratch = torch.empty(B, dtype=torch.int32, device=self.device)
        a = self.args(logits, params, uniforms, history, scratch, None)
        ws = self.workspace(B, V, a.dtype)
        _lib.check(self.lib.vinfer_sample_top_logprobs(C.byref(a), n, ids.data_ptr(),
                                                       lp.data_ptr(), ws.data_ptr(), ws.numel(),
                                                       self._stream()),
                   "vinfer_sample_top_logprobs")
        return ids, lp

    # ---- batched decode with slotted histories ------------------------------------------------
    def append_tokens(self, slots: SlotHistogram, tokens: torch.Tensor) -> None:
        """Count ``tokens[s]`` once more in slot ``s`` (id order kept; a negative id is no
        token). Stream-ordered on the current stream; a full slot sets a status bit."""
        if tokens.shape != (slots.slots,) or tokens.dtype != torch.int32 or \
                tokens.device != self.device or not tokens.is_contiguous():
            raise ValueError(f"tokens must be a contiguous int32 [{slots.slots}] on {self.device}")
        _lib.check(self.lib.vinfer_hist_append(tokens.data_ptr(), slots.slots,
                                               slots.ids.data_ptr(), slots.counts.data_ptr(),
                                               slots.lens.data_ptr(), slots.cap,
                                               self.status.data_ptr(), self._stream()),
                   "vinfer_hist_append")

    def reset_slots(self, slots: SlotHistogram, which: torch.Tensor) -> None:
        """Empty the listed slots (int32 slot numbers on the device): a request leaving."""
        if which.dtype != torch.int32 or which.device != self.device or which.dim() != 1:
            raise ValueError(f"which must be int32 [n] on {self.device}")
        if which.numel() == 0:
            return
        _lib.check(self.lib.vinfer_hist_reset(which.contiguous().data_ptr(), which.numel(),
                                              slots.slots, slots.ids.data_ptr(),
                                              slots.counts.data_ptr(), slots.lens.data_ptr(),
                                              slots.cap, self._stream()), "vinfer_hist_reset")

    def decode_step(self, logits: torch.Tensor, params: RowParams, uniforms: torch.Tensor,
                    slots: SlotHistogram, out: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step of every slot: sample with the slots' histories (penalties) and count
        the sampled ids into them, in one call (``vinfer_sample_decode``: the finishing kernel
        updates each row's slot once the row is decided). Nothing leaves the device; the ids
        are in ``out``."""
        B, V = logits.shape
        if slots.slots != B:
            raise ValueError(f"{slots.slots} slots for {B} rows")
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        a = self.args(logits, params, uniforms, slots.history, out, None)
        ws = self.workspace(B, V, a.dtype)
        _lib.check(self.lib.vinfer_sample_decode(C.byref(a), slots.lens.data_ptr(), slots.cap,
                                                 ws.data_ptr(), ws.numel(), self._stream()),
                   "vinfer_sample_decode")
        return out

    def sample(self, logits: torch.Tensor, params: SamplingParams, seed: int,
               position: int) -> int:
        row = logits.reshape(1, -1)
        if row.dtype not in _DTYPES:
            row = row.float()
        rp = RowParams.pack([params], self.device)
        u = torch.tensor([position_uniform(seed, position)], dtype=torch.float32,
                         device=self.device)
        ids = self.sample_batch(row, rp, u)
        tok = int(ids[0])
        self.check()
        return tok

    def check(self) -> None:
        """Raise ``RuntimeError`` if a device-side problem was reported (synchronises)."""
        bits = int(self.status[0])
        if bits:
            self.status.zero_()
            raise RuntimeError(f"sampler: {_lib.status_message(bits)}")
