"""PyTorch-CPU restatement of LocalStrm's per-row sampler.  TEST INFRASTRUCTURE ONLY.

This is the CPU baseline that ``bench.py --impl reference`` and the ``cpu_baseline`` field
time on the GPU box's host cores (the reference tree itself does not travel there).  It
issues the same PyTorch operations, in the same order and on the same dtypes, as
``sample_next_token`` (``src/engine/sampling.py:118-163``), so it keeps the reference's cost
profile (a full-vocabulary sort for top-p, ``torch.multinomial`` for the draw) and, fed the
same ``torch.Generator`` state, draws the same tokens as the reference; ``tests/golden``
pins that bit for bit.  Only ``tests/``, ``smoke()`` and ``bench.py``'s CPU legs may use it.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn.functional as F

NEG_INF = float("-inf")


def _penalise(row: torch.Tensor, hist: Sequence[int], rep: float, freq: float,
              pres: float) -> torch.Tensor:
    # sampling.py:48-68: unique ids with counts, sign-dependent multiplicative penalty,
    # then additive frequency/presence penalty.
    if len(hist) == 0:
        return row
    ids, counts = torch.unique(torch.as_tensor(list(hist), dtype=torch.int64), return_counts=True)
    if rep != 1.0:
        cur = row[ids]
        row[ids] = torch.where(cur > 0, cur / rep, cur * rep)
    if freq != 0.0 or pres != 0.0:
        row[ids] -= freq * counts.float() + pres
    return row


def _filter(row: torch.Tensor, top_k: int, top_p: float, min_p: float) -> torch.Tensor:
    # sampling.py:71-115 with min_tokens_to_keep == 1.
    V = row.shape[-1]
    if top_k > 0:
        kth = torch.topk(row, min(max(top_k, 1), V))[0][..., -1, None]
        row = row.masked_fill(row < kth, NEG_INF)
    if 0.0 < min_p < 1.0:
        p = F.softmax(row, dim=-1)
        row = row.masked_fill(p < min_p * p.max(dim=-1, keepdim=True)[0], NEG_INF)
    if 0.0 < top_p < 1.0:
        vals, order = torch.sort(row, descending=True)
        cum = torch.cumsum(F.softmax(vals, dim=-1), dim=-1)
        drop = cum > top_p
        drop[..., 1:] = drop[..., :-1].clone()
        drop[..., 0] = False
        row = row.masked_fill(drop.scatter(-1, order, drop), NEG_INF)
    return row


def sample_next_token_cpu(logits: torch.Tensor, temperature: float, top_k: int = -1,
                          top_p: float = 1.0, min_p: float = 0.0, rep: float = 1.0,
                          freq: float = 0.0, pres: float = 0.0, hist: Sequence[int] = (),
                          generator: Optional[torch.Generator] = None) -> int:
    """One token for one row, as ``sample_next_token`` computes it (``sampling.py:118-163``)."""
    row = (logits[-1] if logits.ndim > 1 else logits).clone()
    if temperature <= 0.0:
        return int(torch.argmax(row, dim=-1).item())
    row = _penalise(row, hist, rep, freq, pres)
    row = row / temperature
    row = _filter(row, top_k, top_p, min_p)
    probs = F.softmax(row, dim=-1)
    if torch.isnan(probs).any() or probs.sum() == 0:
        return int(torch.argmax(row, dim=-1).item())
    return int(torch.multinomial(probs, 1, generator=generator).item())


def filtered_row(logits: torch.Tensor, temperature: float, top_k: int = -1, top_p: float = 1.0,
                 min_p: float = 0.0, rep: float = 1.0, freq: float = 0.0, pres: float = 0.0,
                 hist: Sequence[int] = ()) -> torch.Tensor:
    """The masked, scaled row that ``sample_next_token`` feeds to its final softmax."""
    row = (logits[-1] if logits.ndim > 1 else logits).clone()
    row = _penalise(row, hist, rep, freq, pres)
    return _filter(row / temperature, top_k, top_p, min_p)


def sample_workload_rows(w, rows, generator: Optional[torch.Generator] = None) -> list:
    """Per-row loop over a ``Workload`` on float32 CPU tensors (the engine's per-row seam)."""
    out = []
    for r in rows:
        x = torch.from_numpy(w.logits[r])
        h = w.hist_ids[w.hist_offsets[r]:w.hist_offsets[r + 1]].tolist()
        out.append(sample_next_token_cpu(x, float(w.temperature[r]), int(w.top_k[r]),
                                         float(w.top_p[r]), float(w.min_p[r]),
                                         float(w.repetition_penalty[r]),
                                         float(w.frequency_penalty[r]),
                                         float(w.presence_penalty[r]), h, generator))
    return out
