"""ctypes binding of the sampler's C ABI (``include/vinfer_sampler.h``).

The shared library is built in-tree (``vinfer_b200/libvinfer_sampler.so``). There is no
fallback: if it is missing or cannot be loaded, ``load()`` raises, and so does every backend
constructed on top of it.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvinfer_sampler.so"
ABI_VERSION = 1

DTYPE_F32 = 0
DTYPE_BF16 = 1
OK, E_ARG, E_LIMIT, E_CUDA = 0, 1, 2, 3
ST_BAD_PARAM, ST_NONFINITE, ST_HIST_FULL, ST_INTERNAL = 1, 2, 4, 8
FLAG_EXACT_ALL = 1
MAX_VOCAB = 262144
MAX_BATCH = 65535
STATIC_SCRATCH_BYTES = 32 << 20
HIST_PAD_ID = 0x7FFFFFFF
TOP_LOGPROBS_MAX = 32
HIST_MAX_CAP = 1 << 20

EXPORTS = (
    "vinfer_sampler_abi_version",
    "vinfer_sampler_workspace_bytes",
    "vinfer_sampler_workspace_init",
    "vinfer_sample",
    "vinfer_sample_record_bytes",
    "vinfer_sample_local",
    "vinfer_sample_merge",
    "vinfer_sample_static",
    "vinfer_sample_logprobs",
    "vinfer_sample_top_logprobs",
    "vinfer_hist_append",
    "vinfer_hist_reset",
    "vinfer_sample_decode",
)

_ERRORS = {E_ARG: "invalid argument", E_LIMIT: "limit exceeded", E_CUDA: "CUDA error"}


class SampleArgs(C.Structure):
    """Mirror of ``VinferSampleArgs``."""

    _fields_ = [
        ("logits", C.c_void_p),
        ("dtype", C.c_int32),
        ("flags", C.c_uint32),
        ("batch", C.c_int64),
        ("vocab", C.c_int64),
        ("ld", C.c_int64),
        ("vocab_offset", C.c_int64),
        ("vocab_total", C.c_int64),
        ("temperature", C.c_void_p),
        ("top_k", C.c_void_p),
        ("top_p", C.c_void_p),
        ("min_p", C.c_void_p),
        ("repetition_penalty", C.c_void_p),
        ("presence_penalty", C.c_void_p),
        ("frequency_penalty", C.c_void_p),
        ("hist_row_ptr", C.c_void_p),
        ("hist_ids", C.c_void_p),
        ("hist_counts", C.c_void_p),
        ("uniforms", C.c_void_p),
        ("out_ids", C.c_void_p),
        ("out_probs", C.c_void_p),
        ("status", C.c_void_p),
    ]


_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load the library (once). Raises ``RuntimeError`` if it is absent or mismatched."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("VINFER_SAMPLER_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"the B200 sampler library is missing ({path}); build it with "
            "`python -m vinfer_b200.build` (there is no CPU fallback)"
        )
    lib = C.CDLL(str(path))
    lib.vinfer_sampler_abi_version.restype = C.c_int
    lib.vinfer_sampler_workspace_bytes.restype = C.c_size_t
    lib.vinfer_sampler_workspace_bytes.argtypes = [C.c_int64, C.c_int64, C.c_int32]
    lib.vinfer_sampler_workspace_init.restype = C.c_int
    lib.vinfer_sampler_workspace_init.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p]
    lib.vinfer_sample.restype = C.c_int
    lib.vinfer_sample.argtypes = [C.POINTER(SampleArgs), C.c_void_p, C.c_size_t, C.c_void_p]
    lib.vinfer_sample_record_bytes.restype = C.c_size_t
    lib.vinfer_sample_record_bytes.argtypes = [C.c_int32]
    lib.vinfer_sample_local.restype = C.c_int
    lib.vinfer_sample_local.argtypes = [C.POINTER(SampleArgs), C.c_int32, C.c_void_p, C.c_void_p,
                                        C.c_size_t, C.c_void_p]
    lib.vinfer_sample_merge.restype = C.c_int
    lib.vinfer_sample_merge.argtypes = [C.POINTER(SampleArgs), C.c_int32, C.c_void_p, C.c_int32,
                                        C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
    lib.vinfer_sample_static.restype = C.c_int
    lib.vinfer_sample_static.argtypes = [C.POINTER(SampleArgs), C.c_void_p]
    lib.vinfer_sample_logprobs.restype = C.c_int
    lib.vinfer_sample_logprobs.argtypes = [C.POINTER(SampleArgs), C.c_void_p, C.c_void_p,
                                           C.c_size_t, C.c_void_p]
    lib.vinfer_sample_top_logprobs.restype = C.c_int
    lib.vinfer_sample_top_logprobs.argtypes = [C.POINTER(SampleArgs), C.c_int32, C.c_void_p,
                                               C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
    lib.vinfer_hist_append.restype = C.c_int
    lib.vinfer_hist_append.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_int32, C.c_void_p, C.c_void_p]
    lib.vinfer_sample_decode.restype = C.c_int
    lib.vinfer_sample_decode.argtypes = [C.POINTER(SampleArgs), C.c_void_p, C.c_int32, C.c_void_p,
                                         C.c_size_t, C.c_void_p]
    lib.vinfer_hist_reset.restype = C.c_int
    lib.vinfer_hist_reset.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_int32, C.c_void_p]
    version = lib.vinfer_sampler_abi_version()
    if version != ABI_VERSION:
        raise RuntimeError(f"sampler library ABI {version}, expected {ABI_VERSION}")
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != OK:
        raise RuntimeError(f"{what} failed: {_ERRORS.get(rc, rc)}")


def status_message(bits: int) -> str:
    names = []
    if bits & ST_BAD_PARAM:
        names.append("invalid sampling parameters in a row")
    if bits & ST_NONFINITE:
        names.append("a row has no finite logit")
    if bits & ST_HIST_FULL:
        names.append("a history slot was full (a token was not counted)")
    if bits & ST_INTERNAL:
        names.append("internal consistency check failed")
    return ", ".join(names) or "ok"
