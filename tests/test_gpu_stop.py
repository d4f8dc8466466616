"""Device stop check (lss_stop_check) against the restated check_stop_criteria token part."""
import os

import numpy as np
import pytest
import torch

from localstrm_b200 import sampling as S
from oracle import restated as R

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _golden():
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "stop_check.npz"))
    lists = [g["ids"][g["offsets"][i]:g["offsets"][i + 1]].tolist() for i in range(len(g["tokens"]))]
    return g, lists


@needs_cuda
def test_stop_check_golden():
    g, lists = _golden()
    dev = torch.device("cuda", 0)
    tok = torch.from_numpy(g["tokens"]).to(dev)
    eos = [None if e < 0 else int(e) for e in g["eos"]]
    codes = S.check_stop_batch(tok, eos, lists).cpu().numpy()
    assert np.array_equal(codes, g["codes"])
    reasons = S.stop_reasons(codes, g["tokens"])
    for i, (stop, why) in enumerate(reasons):
        assert stop == (g["codes"][i] != 0)
        if g["codes"][i] == 2:
            assert why == f"stop_token_{int(g['tokens'][i])}"


@needs_cuda
def test_stop_check_shapes_and_defaults():
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(5)
    B = 4099
    t = rng.integers(0, 151936, size=B).astype(np.int32)
    lists = [rng.integers(0, 151936, size=int(rng.integers(0, 4))).tolist() for _ in range(B)]
    for r in range(0, B, 13):
        lists[r].append(int(t[r]))
    tok = torch.from_numpy(t).to(dev)
    # one EOS id for every row, per-row stop lists
    got = S.check_stop_batch(tok, 151643, lists).cpu().numpy()
    want = np.array([R.stop_code(int(t[r]), 151643, lists[r]) for r in range(B)], np.int32)
    assert np.array_equal(got, want)
    # no EOS id, one stop list shared by every row
    shared = [int(t[0]), int(t[1])]
    got = S.check_stop_batch(tok, None, shared).cpu().numpy()
    want = np.array([R.stop_code(int(t[r]), None, shared) for r in range(B)], np.int32)
    assert np.array_equal(got, want)
    # neither: every row continues
    assert int(S.check_stop_batch(tok).abs().sum().item()) == 0
    # empty batch
    assert S.check_stop_batch(tok[:0], 1, [[]] * 0).numel() == 0
