"""Seeded synthetic workloads for the batched sampler.

The reference publishes no sampling benchmark and no dataset; these generators
produce the five input shapes and value distributions that the benchmark plan
names (logit distribution, per-row sampling parameters, token histories), from
fixed seeds, with numpy's PCG64 so that the same arrays come out on every
machine with this image.  All outputs are plain numpy arrays on the host; the
caller moves them to the device.

Row parameters use the reference's conventions (``SamplingParams`` in
``src/engine/sampling.py:20-35``): ``temperature <= 0`` is greedy, ``top_k <= 0``
disables top-k, ``top_p`` outside ``(0, 1)`` disables top-p, ``min_p`` outside
``(0, 1)`` disables min-p.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

QWEN_VOCAB = 151_936
LLAMA3_VOCAB = 128_256


@dataclass
class Workload:
    """A batch of rows: logits, per-row parameters (SoA), CSR histories, uniforms."""

    name: str
    logits: np.ndarray                 # [B, V] float32 (values exactly representable in `dtype`)
    dtype: str                         # "f32" | "bf16" | "f16": the dtype the logits arrive in
    temperature: np.ndarray            # [B] float32
    top_k: np.ndarray                  # [B] int32
    top_p: np.ndarray                  # [B] float32
    min_p: np.ndarray                  # [B] float32
    repetition_penalty: np.ndarray     # [B] float32
    frequency_penalty: np.ndarray      # [B] float32
    presence_penalty: np.ndarray       # [B] float32
    hist_offsets: np.ndarray           # [B+1] int32 CSR offsets into hist_ids
    hist_ids: np.ndarray               # [N] int32
    uniforms: np.ndarray               # [B] float32 in [0, 1)
    seed: int = 0
    notes: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return int(self.logits.shape[0])

    @property
    def V(self) -> int:
        return int(self.logits.shape[1])

    def history(self, r: int) -> List[int]:
        return self.hist_ids[self.hist_offsets[r]:self.hist_offsets[r + 1]].tolist()

    def rows(self, idx) -> "Workload":
        """A sub-batch made of the given row indices (histories re-packed)."""
        idx = np.asarray(idx, dtype=np.int64)
        hs = [self.hist_ids[self.hist_offsets[r]:self.hist_offsets[r + 1]] for r in idx]
        offs = np.zeros(len(idx) + 1, dtype=np.int32)
        offs[1:] = np.cumsum([len(h) for h in hs])
        ids = np.concatenate(hs).astype(np.int32) if len(hs) and offs[-1] > 0 else np.zeros(0, np.int32)
        return Workload(self.name, self.logits[idx].copy(), self.dtype,
                        self.temperature[idx].copy(), self.top_k[idx].copy(), self.top_p[idx].copy(),
                        self.min_p[idx].copy(), self.repetition_penalty[idx].copy(),
                        self.frequency_penalty[idx].copy(), self.presence_penalty[idx].copy(),
                        offs, ids, self.uniforms[idx].copy(), self.seed, self.notes, dict(self.extra))


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to bf16/f16 (round-to-nearest-even) and return them as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        rounding = ((u >> 16) & 1) + 0x7FFF
        r = ((u + rounding) >> 16) << 16
        out = r.astype(np.uint32).view(np.float32).copy()
        out[nan] = np.float32("nan")
        return out
    raise ValueError(f"unknown dtype {dtype!r}")


def _zipf_ids(rng: np.random.Generator, a: float, n: int, V: int) -> np.ndarray:
    z = rng.zipf(a, size=n)
    return np.minimum(z - 1, V - 1).astype(np.int32)


def _csr(hists: List[np.ndarray]) -> tuple:
    offs = np.zeros(len(hists) + 1, dtype=np.int32)
    offs[1:] = np.cumsum([len(h) for h in hists])
    ids = np.concatenate(hists).astype(np.int32) if offs[-1] > 0 else np.zeros(0, np.int32)
    return offs, ids


def _uniforms(seed: int, B: int) -> np.ndarray:
    u = np.random.default_rng(seed + 1).random(B, dtype=np.float32)
    return np.minimum(u, np.float32(1.0) - np.float32(2.0 ** -24)).astype(np.float32)


def config1(seed: int = 0, V: int = QWEN_VOCAB) -> Workload:
    """B=8, fp32 N(0, 2^2) plus 3 spike tokens per row raised by +8.

    Rows 0-1 greedy; rows 2-7 temperature 0.8, top-k 50, top-p 0.9, min-p 0; no penalties.
    """
    B = 8
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)).astype(np.float32)
    for r in range(B):
        spikes = rng.choice(V, size=min(3, V), replace=False)
        x[r, spikes] += np.float32(8.0)
    temp = np.full(B, 0.8, np.float32)
    temp[:2] = 0.0
    offs, ids = _csr([np.zeros(0, np.int32)] * B)
    return Workload("cfg1", x, "f32", temp, np.full(B, 50, np.int32), np.full(B, 0.9, np.float32),
                    np.zeros(B, np.float32), np.ones(B, np.float32), np.zeros(B, np.float32),
                    np.zeros(B, np.float32), offs, ids, _uniforms(seed, B), seed)


def config2(seed: int = 0, B: int = 64, V: int = QWEN_VOCAB, H: int = 512,
            all_features: bool = False) -> Workload:
    """bf16 N(0, 2.5^2) with a per-row shift U(-5, 5); mixed per-row parameters.

    temperature U(0.3, 1.3); top-k from {0, 20, 100, 1000} (0 disables it); top-p U(0.5, 1.0);
    min-p from {0, 0.05}; repetition penalty 1.1 over H ids ~ Zipf(1.2) clipped to V.
    With ``all_features`` (the row-sharded sweep) top-k is drawn from {20, 100, 1000}, min-p is
    0.05 and frequency/presence penalties 0.3/0.2 are on as well.
    """
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.5)
    x += rng.uniform(-5.0, 5.0, size=(B, 1)).astype(np.float32)
    x = round_to_dtype(x, "bf16")
    temp = rng.uniform(0.3, 1.3, size=B).astype(np.float32)
    if all_features:
        top_k = rng.choice(np.array([20, 100, 1000], np.int32), size=B).astype(np.int32)
        min_p = np.full(B, 0.05, np.float32)
        freq = np.full(B, 0.3, np.float32)
        pres = np.full(B, 0.2, np.float32)
    else:
        top_k = rng.choice(np.array([0, 20, 100, 1000], np.int32), size=B).astype(np.int32)
        min_p = rng.choice(np.array([0.0, 0.05], np.float32), size=B).astype(np.float32)
        freq = np.zeros(B, np.float32)
        pres = np.zeros(B, np.float32)
    top_p = rng.uniform(0.5, 1.0, size=B).astype(np.float32)
    rep = np.full(B, 1.1, np.float32)
    hists = [_zipf_ids(rng, 1.2, H, V) for _ in range(B)]
    offs, ids = _csr(hists)
    return Workload("cfg4" if all_features else "cfg2", x, "bf16", temp, top_k, top_p, min_p, rep,
                    freq, pres, offs, ids, _uniforms(seed, B), seed)


def config3(seed: int = 0, B: int = 256, V: int = LLAMA3_VOCAB, H: int = 2048) -> Workload:
    """fp32 Gumbel(0, 1) background plus a Zipf-ranked head of 32 tokens.

    Head token of rank r in 1..32 (distinct random ids) gets +4*ln(32/r) on top of its Gumbel
    draw, so head logits fall off as a Zipf law of exponent 4 and the last head token merges
    into the background.  Temperature 0.7, top-p 0.95, min-p 0.05, repetition 1.1, frequency
    0.3, presence 0.2, history of H ids ~ Zipf(1.1).  Edge rows: every 10th row (r % 10 == 0)
    has 5% of its entries set to -inf; every 50th row (r % 50 == 1) has its maximum copied to
    two more random positions (exact max ties).
    """
    rng = np.random.default_rng(seed)
    x = rng.gumbel(0.0, 1.0, size=(B, V)).astype(np.float32)
    ranks = np.arange(1, 33, dtype=np.float64)
    boost = (4.0 * np.log(32.0 / ranks)).astype(np.float32)
    for r in range(B):
        head = rng.choice(V, size=min(32, V), replace=False)
        x[r, head] += boost[:len(head)]
    for r in range(B):
        if r % 10 == 0:
            n = max(1, V // 20)
            x[r, rng.choice(V, size=n, replace=False)] = -np.inf
        if r % 50 == 1 and V >= 3:
            j = int(np.argmax(x[r]))
            others = rng.choice(np.delete(np.arange(V), j), size=2, replace=False)
            x[r, others] = x[r, j]
    hists = [_zipf_ids(rng, 1.1, H, V) for _ in range(B)]
    offs, ids = _csr(hists)
    return Workload("cfg3", x, "f32", np.full(B, 0.7, np.float32), np.zeros(B, np.int32),
                    np.full(B, 0.95, np.float32), np.full(B, 0.05, np.float32),
                    np.full(B, 1.1, np.float32), np.full(B, 0.3, np.float32),
                    np.full(B, 0.2, np.float32), offs, ids, _uniforms(seed, B), seed)


def config4(seed: int = 0, B: int = 1024, V: int = QWEN_VOCAB) -> Workload:
    """Row-sharded sweep: B=1,024, bf16 as config 2 with every sampling feature on."""
    return config2(seed=seed, B=B, V=V, all_features=True)


def config5(seed: int = 0, B: int = 128, V: int = 256_000) -> Workload:
    """Vocab-sharded head: fp32 N(0, 3^2) plus 5 spikes (+8) per row; T 1.0, top-k 64, top-p 0.9."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(3.0)).astype(np.float32)
    for r in range(B):
        x[r, rng.choice(V, size=min(5, V), replace=False)] += np.float32(8.0)
    offs, ids = _csr([np.zeros(0, np.int32)] * B)
    return Workload("cfg5", x, "f32", np.ones(B, np.float32), np.full(B, 64, np.int32),
                    np.full(B, 0.9, np.float32), np.zeros(B, np.float32), np.ones(B, np.float32),
                    np.zeros(B, np.float32), np.zeros(B, np.float32), offs, ids,
                    _uniforms(seed, B), seed)


def headline(seed: int = 0, B: int = 256, V: int = QWEN_VOCAB) -> Workload:
    """The metric point: B=256, V=151,936 fp32 with config 3's distribution and parameters."""
    w = config3(seed=seed, B=B, V=V)
    w.name = "headline"
    return w


def history_on_top(seed: int = 0, B: int = 32, V: int = QWEN_VOCAB, dtype: str = "f32") -> Workload:
    """Rows whose largest raw logits are history tokens, as in repetitive decoding.

    N(0, 2^2) background; per row 24 head tokens raised by +6 .. +11 (distinct random ids), of
    which the 12 largest are in the row's history (1 to 6 times each) together with 400 ids ~
    Zipf(1.1).  Repetition 1.6, frequency 0.6, presence 0.4 push those tokens below the others.
    Parameters cycle over four kinds of row: min-p 0.05; top-k 20; top-k 50 with min-p 0.02;
    top-k 100 with top-p 0.9.  Temperature 0.8.
    """
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)).astype(np.float32)
    hists = []
    for r in range(B):
        head = rng.choice(V, size=min(24, V), replace=False)
        boost = np.sort(rng.uniform(6.0, 11.0, size=len(head)).astype(np.float32))[::-1]
        x[r, head] += boost
        top = head[:12]
        reps = [np.full(int(rng.integers(1, 7)), t, np.int32) for t in top]
        h = np.concatenate(reps + [_zipf_ids(rng, 1.1, 400, V)])
        rng.shuffle(h)
        hists.append(h.astype(np.int32))
    x = round_to_dtype(x, dtype)
    offs, ids = _csr(hists)
    kind = np.arange(B) % 4
    top_k = np.select([kind == 1, kind == 2, kind == 3], [20, 50, 100], 0).astype(np.int32)
    min_p = np.select([kind == 0, kind == 2], [0.05, 0.02], 0.0).astype(np.float32)
    top_p = np.where(kind == 3, 0.9, 1.0).astype(np.float32)
    return Workload("hist_on_top", x, dtype, np.full(B, 0.8, np.float32), top_k, top_p, min_p,
                    np.full(B, 1.6, np.float32), np.full(B, 0.6, np.float32),
                    np.full(B, 0.4, np.float32), offs, ids, _uniforms(seed, B), seed)


def by_name(name: str, **kw) -> Workload:
    return {"cfg1": config1, "cfg2": config2, "cfg3": config3, "cfg4": config4,
            "cfg5": config5, "headline": headline}[name](**kw)
