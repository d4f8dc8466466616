"""The CPU oracles against golden vectors produced by the reference's own sampler.

``oracle.restated`` (numpy, supplied uniform) must reproduce the reference's greedy and
NaN-guard tokens exactly and its kept sets and probabilities under the parity rules;
``oracle.torch_port`` (the timed CPU baseline) must reproduce the reference bit for bit,
including its ``torch.multinomial`` draws under the same seed.
"""
import numpy as np
import pytest
import torch

from oracle import restated as R
from oracle import torch_port as TP
from tests import parity as P
from tests.golden.make_golden import row_seed
from tests.golden.sets import golden_sets

SETS = golden_sets()


@pytest.mark.parametrize("name", list(SETS))
def test_restated_matches_reference(name):
    w = SETS[name]
    g = P.load_golden(name)
    worst = 0.0
    for r in range(w.B):
        res = R.sample_batch(w, want_detail=True, rows=[r])[0]
        kind = int(g["kind"][r])
        if kind == 1:
            assert res.special == "greedy" and res.token == g["tokens"][r], (name, r)
            continue
        if kind == 2:
            assert res.special == "nan_inf" and res.token == g["tokens"][r], (name, r)
            continue
        assert res.special == "", (name, r, res.special)
        kept_ref, probs_ref = P.kept_from_golden(g, r, w.V)
        if kept_ref is None:
            # Long kept list: the fixture keeps its size and smallest kept value only.
            y = R.scaled_row(w.logits[r], float(w.temperature[r]), float(w.repetition_penalty[r]),
                             float(w.frequency_penalty[r]), float(w.presence_penalty[r]),
                             w.history(r))
            n = int(res.kept.sum())
            band = len(P.boundary_tokens(w, r, res, P.reference_topp_band(w, r, res)))
            assert abs(n - int(g["kept_count"][r])) <= band, (name, r, n, g["kept_count"][r])
            if n == int(g["kept_count"][r]):
                assert np.float32(y[res.kept].min()) == g["kept_min"][r], (name, r)
            continue
        msg = P.compare_kept(w, r, res.kept, kept_ref, res, P.reference_topp_band(w, r, res))
        assert msg == "", f"{name}: {msg}"
        both = res.kept & kept_ref
        worst = max(worst, P.probs_close(res.probs, probs_ref, both))
    assert worst <= P.PROB_RTOL, (name, worst)


@pytest.mark.parametrize("name", list(SETS))
def test_torch_port_bit_exact(name):
    w = SETS[name]
    g = P.load_golden(name)
    for r in range(w.B):
        torch.manual_seed(row_seed(w.name, r))
        tok = TP.sample_workload_rows(w, [r])[0]
        assert tok == int(g["tokens"][r]), (name, r, tok, int(g["tokens"][r]))


def test_reference_suite_vectors():
    """tests/test_all_features.py:236-248 of the reference, restated."""
    x = np.array([1.0, 2.0, 5.0, 0.5], np.float32)
    assert R.sample_row(x, 0.0).token == 2
    z = R.apply_penalties(x.copy(), [2], 10.0, 0.0, 0.0)
    assert R.sample_row(z, 0.0).token == 1


def test_ordered_key_is_monotone():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 100,
                        np.array([-np.inf, np.inf, 0.0, -0.0, 1e-45, -1e-45], np.float32)])
    k = R.ordered_key(v)
    order_v = np.argsort(v, kind="stable")
    assert np.all(np.diff(k[order_v].astype(np.int64)) >= 0)
    assert R.ordered_key(np.float32(-0.0)) == R.ordered_key(np.float32(0.0))


def _stop_cases():
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "stop_check.npz"))
    lists = [g["ids"][g["offsets"][i]:g["offsets"][i + 1]] for i in range(len(g["tokens"]))]
    return g, lists


def test_stop_code_matches_reference():
    """The restated token-id stop check against check_stop_criteria's own results."""
    g, lists = _stop_cases()
    for i, t in enumerate(g["tokens"]):
        eos = None if g["eos"][i] < 0 else int(g["eos"][i])
        assert R.stop_code(int(t), eos, [int(v) for v in lists[i]]) == int(g["codes"][i]), i
