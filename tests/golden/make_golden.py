"""Generate golden vectors from LocalStrm's own sampler (run in a container that has the reference).

Usage:  python tests/golden/make_golden.py /path/to/localstrm

Imports ``src.engine.sampling`` from the given reference checkout and runs its functions on
the seeded workloads of ``localstrm_b200.workloads`` (inputs upcast to float32, which is the
parity contract).  For every row it records what the reference computes:

* ``token``: ``sample_next_token`` with ``torch.manual_seed(row_seed(name, r))`` set first, so
  its ``torch.multinomial`` draw is reproducible (greedy and NaN-guard rows are deterministic);
* the kept set after ``apply_repetition_penalties`` -> ``/ temperature`` ->
  ``apply_top_k_top_p_min_p`` (entries that are not -inf), as a sorted index list with the
  reference's ``softmax`` probabilities at those indices (lists longer than ``MAX_LIST`` are
  summarised by count and minimum kept value only).

The inputs are not stored: the tests regenerate them from the same seeds.  The fixtures are
small ``.npz`` files committed next to this script.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.sets import golden_sets  # noqa: E402

MAX_LIST = 8192


def row_seed(name: str, r: int) -> int:
    return (sum(ord(c) for c in name) * 1_000_003 + r * 7919) % (2 ** 31)


def golden_for(w, sampling) -> dict:
    SP = sampling.SamplingParams
    B, V = w.B, w.V
    tokens = np.zeros(B, np.int64)
    kind = np.zeros(B, np.int8)          # 0 draw, 1 greedy, 2 NaN guard
    kept_count = np.zeros(B, np.int64)
    kept_min = np.full(B, np.nan, np.float32)
    ptr = [0]
    idx_all, prob_all = [], []
    for r in range(B):
        x = torch.from_numpy(w.logits[r].copy())
        hist = w.hist_ids[w.hist_offsets[r]:w.hist_offsets[r + 1]].tolist()
        p = SP(temperature=float(w.temperature[r]), top_p=float(w.top_p[r]),
               top_k=int(w.top_k[r]), min_p=float(w.min_p[r]),
               repetition_penalty=float(w.repetition_penalty[r]),
               frequency_penalty=float(w.frequency_penalty[r]),
               presence_penalty=float(w.presence_penalty[r]))
        torch.manual_seed(row_seed(w.name, r))
        tokens[r] = sampling.sample_next_token(x.unsqueeze(0), p, past_token_ids=hist)
        if p.temperature <= 0.0:
            kind[r] = 1
            ptr.append(ptr[-1])
            continue
        row = x.clone()
        if hist:
            row = sampling.apply_repetition_penalties(row, hist, p.repetition_penalty,
                                                      p.frequency_penalty, p.presence_penalty)
        row = row / p.temperature
        filt = sampling.apply_top_k_top_p_min_p(row, top_k=p.top_k, top_p=p.top_p, min_p=p.min_p)
        probs = F.softmax(filt, dim=-1)
        if torch.isnan(probs).any() or probs.sum() == 0:
            kind[r] = 2
            ptr.append(ptr[-1])
            continue
        kept = torch.nonzero(filt > float("-inf")).flatten().numpy()
        kept_count[r] = len(kept)
        kept_min[r] = float(filt[kept].min())
        if len(kept) <= MAX_LIST:
            idx_all.append(kept.astype(np.int32))
            prob_all.append(probs[kept].numpy().astype(np.float32))
            ptr.append(ptr[-1] + len(kept))
        else:
            ptr.append(ptr[-1])
    return dict(tokens=tokens, kind=kind, kept_count=kept_count, kept_min=kept_min,
                kept_ptr=np.asarray(ptr, np.int64),
                kept_idx=np.concatenate(idx_all) if idx_all else np.zeros(0, np.int32),
                kept_prob=np.concatenate(prob_all) if prob_all else np.zeros(0, np.float32))


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from src.engine import sampling  # the reference module
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    sets = golden_sets()
    for name, w in sets.items():
        g = golden_for(w, sampling)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **g)
        print(f"{name}: B={w.B} V={w.V} kept={int(g['kept_count'].sum())} "
              f"listed={len(g['kept_idx'])}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/localstrm")
    main(sys.argv[1])
