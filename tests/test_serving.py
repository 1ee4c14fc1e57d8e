"""The served request fields on CPU: validation with OpenAI's ranges, the mapping onto the
sampler's SamplingParams, and (where vinfer's sources are present) the reference server's own
request model carrying them in ``model_extra``, where it rejects them today until the server
drops them from ``UNSUPPORTED_DEFAULTS``."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

from vinfer_b200.sampling import SamplingParams
from vinfer_b200.serving import SERVED_FIELDS, extend_params, sampling_extensions

REF_SRC = Path("/root/reference/src")


def test_off_values_and_mapping():
    assert sampling_extensions(None) == {"logprobs": False, "top_logprobs": 0}
    p, top, lp = extend_params(SamplingParams(temperature=0.7, top_k=20, top_p=0.8),
                               {"presence_penalty": 0.5, "frequency_penalty": 0.3,
                                "repetition_penalty": 1.1, "min_p": 0.05, "logprobs": True,
                                "top_logprobs": 5, "unrelated": 1})
    assert (p.temperature, p.top_k, p.top_p) == (0.7, 20, 0.8)
    assert (p.presence_penalty, p.frequency_penalty, p.repetition_penalty, p.min_p) == \
        (0.5, 0.3, 1.1, 0.05)
    assert (top, lp) == (5, True)


@pytest.mark.parametrize("extra,msg", [
    ({"presence_penalty": 2.5}, "presence_penalty"),
    ({"frequency_penalty": "high"}, "frequency_penalty"),
    ({"repetition_penalty": 0}, "repetition_penalty"),
    ({"min_p": 1.5}, "min_p"),
    ({"logprobs": 1}, "logprobs"),
    ({"logprobs": True, "top_logprobs": 33}, "top_logprobs"),
    ({"top_logprobs": 3}, "requires logprobs"),
    ({"min_p": float("nan")}, "min_p"),
])
def test_bad_values_name_the_field(extra, msg):
    with pytest.raises(ValueError, match=msg):
        sampling_extensions(extra)


@pytest.mark.skipif(not REF_SRC.exists(), reason="vinfer's sources are not present")
def test_reference_request_model_carries_the_fields():
    sys.path.insert(0, str(REF_SRC))
    try:
        protocol = pytest.importorskip("vinfer.server.protocol")
    finally:
        sys.path.remove(str(REF_SRC))
    body = {"messages": [{"role": "user", "content": "hi"}], "temperature": 0.7,
            "presence_penalty": 0.5, "min_p": 0.05, "logprobs": True, "top_logprobs": 3}
    req = protocol.ChatCompletionRequest.model_validate(body)
    # today the server rejects them ...
    assert set(protocol.unsupported_fields(req)) >= {"presence_penalty", "min_p", "logprobs",
                                                     "top_logprobs"}
    # ... and they arrive in model_extra, which extend_params reads after the edit
    assert set(SERVED_FIELDS) <= set(protocol.UNSUPPORTED_DEFAULTS)
    p, top, lp = extend_params(SamplingParams(temperature=0.7), req.model_extra)
    assert (p.presence_penalty, p.min_p, top, lp) == (0.5, 0.05, 3, True)
