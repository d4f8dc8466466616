"""Comparison rules shared by the parity tests.

* greedy and NaN-guard tokens: bit-exact;
* kept set: bit-exact, except (a) which members of a tie group at the boundary value survive
  (same count, same multiset of kept values), and (b) tokens on a filter boundary: top-p
  tokens whose cumulative mass before them lies within ``BAND`` of ``top_p``, min-p tokens
  whose ``exp(y - max) / min_p`` lies within ``BAND`` of 1;
* probabilities of kept tokens: within ``PROB_RTOL`` relative (float32 accumulation);
* drawn token for the same uniform: exact unless the uniform lies within ``BAND`` of a CDF
  boundary of the oracle's final distribution.
"""
from __future__ import annotations

import os

import numpy as np

from oracle import restated as R

BAND = 1e-6
PROB_RTOL = 1e-5
GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as f:
        return {k: f[k] for k in f.files}


def boundary_tokens(w, r: int, res: "R.RowResult", band_topp: float = BAND,
                    band_minp: float = BAND) -> np.ndarray:
    """Vocabulary indices of row r that sit within the band of a min-p or top-p boundary."""
    h = w.hist_ids[w.hist_offsets[r]:w.hist_offsets[r + 1]]
    y = R.scaled_row(w.logits[r], float(w.temperature[r]), float(w.repetition_penalty[r]),
                     float(w.frequency_penalty[r]), float(w.presence_penalty[r]), h)
    band = np.zeros(w.V, dtype=bool)
    mp = float(w.min_p[r])
    finite = np.isfinite(y)
    if 0.0 < mp < 1.0:
        e = np.exp((y[finite] - np.float32(res.y_max)).astype(np.float32)).astype(np.float64)
        band[np.nonzero(finite)[0]] |= np.abs(e / mp - 1.0) <= band_minp
    tp = float(w.top_p[r])
    if 0.0 < tp < 1.0 and res.cum_before is not None:
        cb = res.cum_before
        ok = ~np.isnan(cb)
        band[ok] |= np.abs(cb[ok].astype(np.float64) - tp) <= band_topp
    return np.nonzero(band)[0]


def compare_kept(w, r: int, kept_test: np.ndarray, kept_ref: np.ndarray,
                 res: "R.RowResult", band_topp: float = BAND, band_minp: float = BAND) -> str:
    """'' when the kept sets agree under the rules above, else a description of the mismatch."""
    kt = np.asarray(kept_test, dtype=bool)
    kr = np.asarray(kept_ref, dtype=bool)
    if np.array_equal(kt, kr):
        return ""
    h = w.hist_ids[w.hist_offsets[r]:w.hist_offsets[r + 1]]
    y = R.scaled_row(w.logits[r], float(w.temperature[r]), float(w.repetition_penalty[r]),
                     float(w.frequency_penalty[r]), float(w.presence_penalty[r]), h)
    if R.kept_equal_modulo_ties(kt, kr, y):
        return ""
    diff = np.nonzero(kt != kr)[0]
    allowed = set(boundary_tokens(w, r, res, band_topp, band_minp).tolist())
    # Members of the tie group of a boundary token are interchangeable as well.
    if allowed:
        keys = R.ordered_key(y)
        bkeys = set(keys[list(allowed)].tolist())
        allowed |= set(np.nonzero(np.isin(keys, list(bkeys)))[0].tolist())
    bad = [int(i) for i in diff if int(i) not in allowed]
    if bad:
        return (f"row {r}: {len(bad)} kept-set mismatches outside the band "
                f"(e.g. {bad[:5]}, test={kt[bad[:5]].tolist()}, y={y[bad[:5]].tolist()})")
    return ""


def reference_topp_band(w, r: int, res: "R.RowResult") -> float:
    """Top-p band for comparisons against the reference itself.

    The reference's CPU ``F.softmax`` accumulates its normaliser in float32; on long rows its
    probabilities are off by a common factor (measured up to about 1.2e-5 for 151,936
    entries), which moves every cumulative value at the top-p boundary by that much.  The
    band is twice that row's measured ``|sum(softmax) - 1|`` (never below ``BAND``).
    """
    import torch
    import torch.nn.functional as F

    tp = float(w.top_p[r])
    if not (0.0 < tp < 1.0) or res.cum_before is None:
        return BAND
    h = w.hist_ids[w.hist_offsets[r]:w.hist_offsets[r + 1]]
    y = R.scaled_row(w.logits[r], float(w.temperature[r]), float(w.repetition_penalty[r]),
                     float(w.frequency_penalty[r]), float(w.presence_penalty[r]), h)
    pre = np.where(~np.isnan(res.cum_before), y, -np.inf).astype(np.float32)
    s = float(F.softmax(torch.from_numpy(np.sort(pre)[::-1].copy()), dim=-1).double().sum())
    return max(BAND, 2.0 * abs(s - 1.0))


def kept_from_golden(g: dict, r: int, V: int):
    a, b = int(g["kept_ptr"][r]), int(g["kept_ptr"][r + 1])
    if b - a == 0 and g["kept_count"][r] > 0:
        return None, None
    kept = np.zeros(V, dtype=bool)
    kept[g["kept_idx"][a:b]] = True
    probs = np.zeros(V, dtype=np.float32)
    probs[g["kept_idx"][a:b]] = g["kept_prob"][a:b]
    return kept, probs


def probs_close(p_test: np.ndarray, p_ref: np.ndarray, mask: np.ndarray) -> float:
    """Largest relative difference over the masked entries (0 when they all agree)."""
    a = p_test[mask].astype(np.float64)
    b = p_ref[mask].astype(np.float64)
    if a.size == 0:
        return 0.0
    den = np.maximum(np.abs(b), 1e-30)
    return float(np.max(np.abs(a - b) / den))


def draw_is_boundary(probs: np.ndarray, u: float) -> bool:
    """True when u lies within BAND of a CDF boundary of the final distribution."""
    c = np.cumsum(probs.astype(np.float64))
    if c[-1] <= 0:
        return False
    c = c / c[-1]
    return bool(np.any(np.abs(c - u) <= BAND))
