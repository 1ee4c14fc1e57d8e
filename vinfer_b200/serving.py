"""Request fields the B200 sampler serves that vinfer's OpenAI server rejects today.

``src/vinfer/server/protocol.py:129-158`` lists ``presence_penalty``, ``frequency_penalty``,
``repetition_penalty``, ``min_p``, ``logprobs`` and ``top_logprobs`` in ``UNSUPPORTED_DEFAULTS``
(any value but "off" is a 400), and ``src/vinfer/server/app.py:64-83`` (``sampling_params``)
maps a request to ``SamplingParams`` without them. With the ``b200`` sampler selected, the
server drops these names from ``UNSUPPORTED_DEFAULTS`` and passes the request's extra fields
(pydantic's ``model_extra``, where they arrive today) through ``extend_params``; the response
reads the log-probabilities the backend returns (``sample_batch(logprobs_out=)``,
``top_logprobs``). Values are checked here with OpenAI's ranges, and a bad one raises
``ValueError`` naming the field, which the server turns into its 400 ``APIError``.
"""

from __future__ import annotations

import dataclasses
import math
from collections.abc import Mapping
from typing import Any

from vinfer_b200 import _lib
from vinfer_b200.sampling import SamplingParams

# field -> (low, high) inclusive, OpenAI's ranges where it defines them
_RANGES = {
    "presence_penalty": (-2.0, 2.0),
    "frequency_penalty": (-2.0, 2.0),
    "min_p": (0.0, 1.0),
}
SERVED_FIELDS = ("presence_penalty", "frequency_penalty", "repetition_penalty", "min_p",
                 "logprobs", "top_logprobs")


def _number(name: str, v: Any) -> float:
    if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v):
        raise ValueError(f"{name} must be a finite number")
    return float(v)


def sampling_extensions(extra: Mapping[str, Any] | None) -> dict[str, Any]:
    """The served fields present in ``extra`` (a request's ``model_extra``), validated.
    Returns ``SamplingParams`` field values plus ``logprobs`` (bool) and ``top_logprobs``
    (int, 0 = off); a field left out or null keeps its "off" value."""
    extra = extra or {}
    out: dict[str, Any] = {}
    for name, (lo, hi) in _RANGES.items():
        if extra.get(name) is None:
            continue
        v = _number(name, extra[name])
        if not lo <= v <= hi:
            raise ValueError(f"{name} must be in [{lo:g}, {hi:g}], got {v:g}")
        out[name] = v
    if extra.get("repetition_penalty") is not None:
        v = _number("repetition_penalty", extra["repetition_penalty"])
        if not v > 0:
            raise ValueError(f"repetition_penalty must be > 0, got {v:g}")
        out["repetition_penalty"] = v
    lp = extra.get("logprobs")
    if lp is not None and not isinstance(lp, bool):
        raise ValueError("logprobs must be a boolean")
    out["logprobs"] = bool(lp)
    top = extra.get("top_logprobs")
    if top is None:
        top = 0
    if isinstance(top, bool) or not isinstance(top, int):
        raise ValueError("top_logprobs must be an integer")
    if not 0 <= top <= _lib.TOP_LOGPROBS_MAX:
        raise ValueError(f"top_logprobs must be in [0, {_lib.TOP_LOGPROBS_MAX}], got {top}")
    if top and not out["logprobs"]:
        raise ValueError("top_logprobs requires logprobs to be true")
    out["top_logprobs"] = top
    return out


def extend_params(params: Any, extra: Mapping[str, Any] | None) -> tuple[SamplingParams, int, bool]:
    """``params`` (the server's ``SamplingParams``, with the reference's fields) extended with
    the request's served fields: (the sampler's ``SamplingParams``, ``top_logprobs`` n, whether
    ``logprobs`` was asked)."""
    ext = sampling_extensions(extra)
    base = {f.name: getattr(params, f.name) for f in dataclasses.fields(SamplingParams)
            if hasattr(params, f.name)}
    base.update({k: v for k, v in ext.items() if k not in ("logprobs", "top_logprobs")})
    return SamplingParams(**base), ext["top_logprobs"], ext["logprobs"]
