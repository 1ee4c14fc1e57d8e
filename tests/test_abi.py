"""The C ABI library on CPU: it loads, exports every symbol the header declares, and answers
host-only queries; no call here reaches the GPU."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from vinfer_b200 import _lib
from vinfer_b200.build import build

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def declared_symbols() -> set[str]:
    out = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        out |= set(re.findall(r"^\s*(?:int|size_t)\s+(vinfer_\w+)\s*\(", text, re.M))
    return out


def test_every_declared_symbol_is_exported(lib):
    syms = declared_symbols()
    assert syms >= set(_lib.EXPORTS)
    for name in syms:
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.vinfer_sampler_abi_version() == _lib.ABI_VERSION


def test_struct_layout_matches_the_header():
    # pointer, 2 x int32, 5 x int64, 14 pointers
    assert C.sizeof(_lib.SampleArgs) == 8 + 8 + 5 * 8 + 14 * 8


def test_workspace_sizes(lib):
    a = lib.vinfer_sampler_workspace_bytes(256, 151936, _lib.DTYPE_BF16)
    b = lib.vinfer_sampler_workspace_bytes(256, 151936, _lib.DTYPE_F32)
    assert 0 < a <= b < 256 << 20
    big = lib.vinfer_sampler_workspace_bytes(4096, 151936, _lib.DTYPE_F32)
    assert b < big < 4 << 30
    assert lib.vinfer_sampler_workspace_bytes(0, 100, _lib.DTYPE_F32) == 0
    assert lib.vinfer_sampler_workspace_bytes(1, _lib.MAX_VOCAB + 1, _lib.DTYPE_F32) == 0
    assert lib.vinfer_sampler_workspace_bytes(1, 100, 7) == 0
    assert lib.vinfer_sample_record_bytes(64) == 32 + 64 * 8
    assert lib.vinfer_sample_record_bytes(0) == 0


def test_bad_arguments_are_rejected_before_any_launch(lib):
    assert lib.vinfer_sample(None, None, 0, None) == _lib.E_ARG
    a = _lib.SampleArgs()
    a.logits = 16
    a.out_ids = 16
    a.dtype = 5
    a.batch, a.vocab, a.ld = 1, 10, 10
    assert lib.vinfer_sample(C.byref(a), None, 0, None) == _lib.E_ARG
    a.dtype = _lib.DTYPE_F32
    a.vocab = a.ld = _lib.MAX_VOCAB + 1
    a.vocab_total = a.vocab
    assert lib.vinfer_sample(C.byref(a), None, 0, None) == _lib.E_LIMIT
    a.vocab = a.ld = a.vocab_total = 10
    assert lib.vinfer_sample(C.byref(a), None, 0, None) == _lib.E_ARG  # no workspace
    assert lib.vinfer_sample(C.byref(a), 16, 1, None) == _lib.E_LIMIT  # workspace too small
