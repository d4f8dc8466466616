"""CPU-only checks of the C ABI library and the host-side logic (no GPU calls)."""
import ctypes
import dataclasses

import numpy as np
import pytest

from localstrm_b200 import _lib
from localstrm_b200 import sampling as S


def test_library_loads_and_exports_every_header_symbol():
    lib = _lib.load()
    names = _lib.header_functions()
    assert len(names) >= 8, names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/lsampler.h but not exported"


def test_version_status_and_limits():
    lib = _lib.load()
    assert lib.lss_version() >= (0 << 16) | (1 << 8)
    assert _lib.status_string(0) == "ok"
    assert "invalid" in _lib.status_string(1)
    assert _lib.status_string(999) == "unknown status"
    assert lib.lss_max_vocab() >= 256_000


def test_workspace_bytes_grows_with_history():
    lib = _lib.load()
    a = lib.lss_workspace_bytes(256, 151_936, 0)
    b = lib.lss_workspace_bytes(256, 151_936, 256 * 2048)
    assert 0 < a < b
    assert b % 256 == 0
    assert lib.lss_workspace_bytes(-1, 10, 0) == 0


def _call(lib, **kw):
    args = dict(logits=1, dtype=0, B=1, V=8, stride=8, t=1, k=1, p=1, mp=1, rp=1, fp=1, pp=1,
                hoff=None, hids=None, htot=0, u=1, tok=1, kept=None, probs=None, ws=256, wsb=1 << 20,
                stream=None)
    args.update(kw)
    return lib.lss_sample(args["logits"], args["dtype"], args["B"], args["V"], args["stride"],
                          args["t"], args["k"], args["p"], args["mp"], args["rp"], args["fp"],
                          args["pp"], args["hoff"], args["hids"], args["htot"], args["u"],
                          args["tok"], args["kept"], args["probs"], args["ws"], args["wsb"],
                          args["stream"])


def test_invalid_arguments_are_rejected_before_any_device_work():
    lib = _lib.load()
    assert _call(lib, B=-1) == 1
    assert _call(lib, V=0) == 1
    assert _call(lib, stride=4) == 1
    assert _call(lib, dtype=7) == 1
    assert _call(lib, V=lib.lss_max_vocab() + 1, stride=lib.lss_max_vocab() + 1) == 4
    assert _call(lib, B=0) == 0                    # empty batch: nothing to do
    assert _call(lib, logits=None) == 1
    assert _call(lib, u=None) == 1
    assert _call(lib, htot=5) == 1                 # history without offsets / ids
    assert _call(lib, ws=None) == 2
    assert _call(lib, wsb=16) == 2
    assert _call(lib, ws=257) == 2                 # misaligned workspace
    assert lib.lss_argmax(None, 0, 1, 8, 8, 1, None) == 1
    assert lib.lss_argmax(1, 0, 0, 8, 8, 1, None) == 0


def test_sampling_params_mirror_reference_fields():
    f = {x.name: x.default for x in dataclasses.fields(S.SamplingParams)
         if x.default is not dataclasses.MISSING}
    assert f == {"temperature": 0.7, "top_p": 1.0, "top_k": -1, "min_p": 0.0,
                 "repetition_penalty": 1.0, "frequency_penalty": 0.0, "presence_penalty": 0.0}
    assert S.SamplingParams.greedy().temperature == 0.0


def test_history_csr():
    offs, ids = S.build_history_csr([[1, 2, 2], None, [], [-1, 0]], 4, 10)
    assert offs.tolist() == [0, 3, 3, 3, 5]
    assert ids.tolist() == [1, 2, 2, 9, 0]
    offs, ids = S.build_history_csr(None, 3, 10)
    assert offs.tolist() == [0, 0, 0, 0] and ids.size == 0
    with pytest.raises(IndexError):
        S.build_history_csr([[10]], 1, 10)
    with pytest.raises(IndexError):
        S.build_history_csr([[-11]], 1, 10)
    with pytest.raises(ValueError):
        S.build_history_csr([[1]], 2, 10)


def test_cpu_tensors_fail_loudly():
    import torch
    with pytest.raises(RuntimeError):
        S.sample_next_token(torch.zeros(4), S.SamplingParams.greedy())
    with pytest.raises(RuntimeError):
        S.sample_batch(torch.zeros(2, 4), [S.SamplingParams()] * 2)


def test_noalloc_rejects_requests_beyond_its_fixed_scratch():
    lib = _lib.load()
    limit = 32 << 20
    B, V = 256, 151_936
    H = 1
    while lib.lss_workspace_bytes(B, V, H) <= limit:
        H *= 2
    args = [1, 0, B, V, V] + [1] * 7 + [1, 1, H, 1, 1, None, None, None]
    assert lib.lss_sample_noalloc(*args) == 6            # LSS_ERR_SCRATCH_LIMIT, nothing launched
    assert "scratch" in _lib.status_string(6)
    assert lib.lss_workspace_bytes(256, V, 256 * 2048) <= limit   # the headline fits
    assert lib.lss_sample_noalloc(*([1, 0, 0, V, V] + [1] * 7 + [1, 1, 0, 1, 1, None, None, None])) == 0


def test_history_csr_dtype_and_shape_are_checked_on_the_host():
    """An int64 CSR (torch's default for Python ints) or a wrong-sized one is refused before
    anything reaches the library, which reads int32 arrays."""
    import torch
    s = S.BatchSampler.__new__(S.BatchSampler)  # no device needed: the checks run first
    s.device = torch.device("cpu")
    s.lib = _lib.load()
    s._ws = None
    s._ws_bytes = 0
    s._last_ws = None
    B, V = 2, 16
    x = torch.zeros(B, V)
    prm = S.RowParams.from_arrays("cpu", temperature=[1, 1], top_k=[5, 5], top_p=[1, 1], min_p=[0, 0],
                                  repetition_penalty=[1.1, 1.1], frequency_penalty=[0, 0],
                                  presence_penalty=[0, 0])
    u = torch.zeros(B)
    good_off = torch.tensor([0, 2, 3], dtype=torch.int32)
    good_ids = torch.tensor([1, 2, 3], dtype=torch.int32)
    for off, ids in ((good_off.long(), good_ids), (good_off, good_ids.long()),
                     (good_off[:2], good_ids), (None, good_ids)):
        with pytest.raises(ValueError):
            s.sample(x, prm, off, ids, u)


def test_noalloc_status_reader_is_exported():
    lib = _lib.load()
    assert hasattr(lib, "lss_noalloc_read_status")
    assert lib.lss_noalloc_read_status(None, None) == 1   # NULL output: rejected without device work
