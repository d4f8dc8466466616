"""ctypes binding of ``include/lsampler.h`` (the library ``_lib/liblss.so``).

Loading fails loudly: there is no CPU fallback behind this module.
"""
from __future__ import annotations

import ctypes
import os
import re
from ctypes import c_char_p, c_int, c_int64, c_size_t, c_uint32, c_void_p

from . import build as _build

LSS_OK = 0
DTYPES = {"f32": 0, "bf16": 1, "f16": 2}
PATHS = {1: "greedy", 2: "special", 3: "gather", 4: "dense", 5: "slow_gather"}

_lib = None


class SamplerError(RuntimeError):
    """A non-zero status from the native library."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} (status {status})")


def _declare(lib: ctypes.CDLL) -> None:
    P = c_void_p
    lib.lss_version.restype = c_int
    lib.lss_version.argtypes = []
    lib.lss_status_string.restype = c_char_p
    lib.lss_status_string.argtypes = [c_int]
    lib.lss_max_vocab.restype = c_int
    lib.lss_max_vocab.argtypes = []
    lib.lss_workspace_bytes.restype = c_size_t
    lib.lss_workspace_bytes.argtypes = [c_int, c_int, c_int64]
    lib.lss_sample.restype = c_int
    lib.lss_sample.argtypes = [P, c_int, c_int, c_int, c_int64, P, P, P, P, P, P, P, P, P, c_int64,
                               P, P, P, P, P, c_size_t, P]
    lib.lss_sample_prepare.restype = c_int
    lib.lss_sample_prepare.argtypes = [c_int, c_int, P, P, P, P, P, P, P, P, c_int64, P, c_size_t, P]
    lib.lss_sample_rows.restype = c_int
    lib.lss_sample_rows.argtypes = [P, c_int, c_int, c_int, c_int64, P, P, P, P, P, P, P, P, P, c_int64,
                                    P, P, P, P, P, c_size_t, P]
    lib.lss_scan_pass.restype = c_int
    lib.lss_scan_pass.argtypes = [P, c_int, c_int, c_int, c_int64, P, P, P, P, P, P, P, P, P, c_int64,
                                  P, P, P, c_size_t, P]
    lib.lss_shard_record_bytes.restype = c_size_t
    lib.lss_shard_record_bytes.argtypes = [c_int]
    lib.lss_shard_merge_workspace_bytes.restype = c_size_t
    lib.lss_shard_merge_workspace_bytes.argtypes = [c_int]
    lib.lss_shard_topk.restype = c_int
    lib.lss_shard_topk.argtypes = [P, c_int, c_int, c_int, c_int64, c_int64, P, c_int, P, P]
    lib.lss_shard_merge.restype = c_int
    lib.lss_shard_merge.argtypes = [P, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, c_size_t, P]
    lib.lss_noalloc_read_status.restype = c_int
    lib.lss_noalloc_read_status.argtypes = [P, P]
    lib.lss_sample_noalloc.restype = c_int
    lib.lss_sample_noalloc.argtypes = [P, c_int, c_int, c_int, c_int64, P, P, P, P, P, P, P, P, P,
                                       c_int64, P, P, P, P, P]
    lib.lss_argmax.restype = c_int
    lib.lss_argmax.argtypes = [P, c_int, c_int, c_int, c_int64, P, P]
    lib.lss_stop_check.restype = c_int
    lib.lss_stop_check.argtypes = [P, c_int, P, P, P, P, P]
    lib.lss_read_status.restype = c_int
    lib.lss_read_status.argtypes = [P, ctypes.POINTER(c_uint32), P]
    lib.lss_read_row_paths.restype = c_int
    lib.lss_read_row_paths.argtypes = [P, c_int, P, P]


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """The loaded library (built first when missing and ``build_if_missing``)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    if not os.path.exists(path):
        if not build_if_missing:
            raise RuntimeError(f"native sampler library missing: {path}")
        _build.build()
    lib = ctypes.CDLL(path)
    _declare(lib)
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().lss_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != LSS_OK:
        raise SamplerError(fn, status)


def header_functions() -> list:
    """Function names declared in include/lsampler.h (for the export test)."""
    hdr = os.path.join(_build.INCLUDE, "lsampler.h")
    text = open(hdr).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\*]+\s+)+\**(lss_\w+)\s*\(", text, re.M)))
