"""Hand-made edge-case rows (small vocabularies) for the golden vectors and parity tests.

Covers what the reference's own sampling test checks (``tests/test_all_features.py:236-248``:
greedy on ``[1, 2, 5, 0.5]`` gives 2; a repetition penalty of 10 on token 2 flips greedy to 1)
plus the corners of ``sample_next_token``: NaN / +inf / all -inf rows, +0/-0 and exact ties,
top-k >= V, tiny and huge temperatures, duplicate histories, negative logits under the
multiplicative penalty, V = 1, and vocabularies that are not a multiple of the vector width.
"""
from __future__ import annotations

import numpy as np

from localstrm_b200.workloads import Workload, _csr, _zipf_ids

NAN = np.float32("nan")
INF = np.float32("inf")


def _w(name, rows, params, hists=None, uniforms=None) -> Workload:
    x = np.asarray(rows, dtype=np.float32)
    B = x.shape[0]
    cols = {k: [] for k in ("t", "k", "p", "mp", "rep", "freq", "pres")}
    for prm in params:
        for key, default in (("t", 0.7), ("k", -1), ("p", 1.0), ("mp", 0.0), ("rep", 1.0),
                             ("freq", 0.0), ("pres", 0.0)):
            cols[key].append(prm.get(key, default))
    hists = hists or [[] for _ in range(B)]
    offs, ids = _csr([np.asarray(h, np.int32) for h in hists])
    u = np.asarray(uniforms if uniforms is not None else [0.5] * B, np.float32)
    return Workload(name, x, "f32", np.asarray(cols["t"], np.float32),
                    np.asarray(cols["k"], np.int32), np.asarray(cols["p"], np.float32),
                    np.asarray(cols["mp"], np.float32), np.asarray(cols["rep"], np.float32),
                    np.asarray(cols["freq"], np.float32), np.asarray(cols["pres"], np.float32),
                    offs, ids, u)


def _random(name, V, B, seed) -> Workload:
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((B, V)) * 2.0).astype(np.float32)
    t = rng.choice(np.array([0.0, 0.3, 0.7, 1.0, 1.5], np.float32), size=B)
    k = rng.choice(np.array([-1, 0, 1, 3, 50, 10 ** 6], np.int32), size=B)
    p = rng.choice(np.array([1.0, 0.95, 0.5, 0.1], np.float32), size=B)
    mp = rng.choice(np.array([0.0, 0.05, 0.3], np.float32), size=B)
    rep = rng.choice(np.array([1.0, 1.1, 2.0], np.float32), size=B)
    freq = rng.choice(np.array([0.0, 0.3, -0.5], np.float32), size=B)
    pres = rng.choice(np.array([0.0, 0.2], np.float32), size=B)
    hists = [_zipf_ids(rng, 1.3, int(rng.integers(0, 3 * V + 2)), V) for _ in range(B)]
    offs, ids = _csr(hists)
    u = rng.random(B, dtype=np.float32)
    return Workload(name, x, "f32", t, k, p, mp, rep, freq, pres, offs, ids, u, seed)


def edge_workloads() -> dict:
    out = {}
    # The reference's own golden vectors (tests/test_all_features.py:238-248), as rows.
    out["edge_ref_suite"] = _w(
        "edge_ref_suite",
        [[1.0, 2.0, 5.0, 0.5],            # greedy -> 2
         [1.0, 2.0, 0.5, 0.5],            # the penalised row of the test, greedy -> 1
         [1.0, 2.0, 5.0, 0.5],            # same penalty applied by the sampler, T tiny -> 1
         [1.0, 2.0, 5.0, 0.5]],
        [dict(t=0.0), dict(t=0.0), dict(t=1e-3, rep=10.0), dict(t=1.0, k=2)],
        hists=[[], [], [2], [2, 2, 0]], uniforms=[0.5, 0.5, 0.5, 0.99])
    out["edge_special"] = _w(
        "edge_special",
        [[1.0, NAN, 2.0, INF, 0.0],       # NaN row: NaN guard -> first NaN
         [1.0, INF, 2.0, INF, 0.0],       # +inf row -> first +inf
         [-INF] * 5,                      # all -inf -> 0
         [-0.0, 0.0, -1.0, -INF, -2.0],   # greedy +0/-0 tie -> 0
         [1.0, NAN, 2.0, 3.0, 0.0],       # greedy with NaN -> 1
         [3.0, 5.0, 5.0, 5.0, 1.0],       # exact max ties, top-p tiny
         [3.0, 5.0, 5.0, 5.0, 1.0],       # exact max ties, greedy -> 1
         [1e30, 3e38, 2e38, 0.0, 1.0],    # tiny temperature overflows to +inf
         [-INF, 2.0, -INF, 2.0, 1.0],     # partial -inf, ties at top-k threshold
         [0.5, -1.5, 2.5, -3.0, 1.0]],    # negative logits under the multiplicative penalty
        [dict(t=0.7, p=0.9), dict(t=0.7, p=0.9), dict(t=0.7, k=2, p=0.9, mp=0.1), dict(t=0.0),
         dict(t=0.0), dict(t=1.0, p=0.01), dict(t=0.0), dict(t=1e-3), dict(t=1.0, k=1),
         dict(t=0.9, rep=1.5, freq=0.25, pres=0.5)],
        hists=[[], [], [], [], [], [], [], [], [], [1, 1, 3, 3, 3, 4]],
        uniforms=[0.5, 0.5, 0.5, 0.5, 0.5, 0.7, 0.5, 0.5, 0.9, 0.3])
    out["edge_v1"] = _w("edge_v1", [[0.25], [-INF], [3.0]],
                        [dict(t=0.8, k=5, p=0.5, mp=0.5), dict(t=0.8), dict(t=0.0)],
                        hists=[[0, 0], [], []])
    out["edge_v7"] = _random("edge_v7", 7, 24, 11)
    out["edge_v33"] = _random("edge_v33", 33, 24, 12)
    out["edge_v4099"] = _random("edge_v4099", 4099, 24, 13)
    return out
