"""Test infrastructure only: the vocabulary-sharded mode restated on the CPU.

``shard_records`` writes the same bytes as the native per-shard step (``lss_shard_topk``): per
row, the shard's K largest values of ``y = z / T`` as u64 codes ``key(y) << 32 | ~global_index``
(value descending, index ascending; a greedy row uses the raw values), then f32 max of y, f32
sum of ``exp(y - max)``, u32 flags, u32 code count.  ``merge_records`` follows the reference on
the union of the shards' candidates: ``sample_next_token`` (``sampling.py:118-163``) with
``top_k = K``, the row's ``top_p``, no min-p and no penalties, which is the reference on the
whole row because the union holds the row's K largest values.  Only ``tests/`` use this module.
"""
from __future__ import annotations

import numpy as np

from . import restated as R

F32 = np.float32


def record_bytes(K: int) -> int:
    return 8 * K + 16


def _code(y: np.ndarray, idx: np.ndarray) -> np.ndarray:
    return (R.ordered_key(y).astype(np.uint64) << np.uint64(32)) | (~idx.astype(np.uint32)).astype(np.uint64)


def shard_records(z: np.ndarray, offset: int, temperature: np.ndarray, K: int) -> np.ndarray:
    """Records of every row of one shard (``z``: [B, Vs] float32) as a flat uint8 array."""
    z = np.asarray(z, dtype=F32)
    B, Vs = z.shape
    out = np.zeros((B, record_bytes(K)), dtype=np.uint8)
    for b in range(B):
        T = float(temperature[b])
        y = z[b] if T <= 0.0 else (z[b] / F32(T)).astype(F32)
        idx = np.arange(Vs, dtype=np.int64) + offset
        codes = np.zeros(K, dtype=np.uint64)
        fin = np.isfinite(y)
        if np.isnan(y).any() or np.isposinf(y).any() or not fin.any():
            # special shard: its argmax only (NaN first, lowest index)
            j = R.argmax_nan_first(y)
            key = np.uint64(0xFFFFFFFF) if np.isnan(y[j]) else np.uint64(R.ordered_key(y[j:j + 1])[0])
            codes[0] = (key << np.uint64(32)) | np.uint64(~np.uint32(idx[j]) & np.uint32(0xFFFFFFFF))
            my = F32(np.nan) if np.isnan(y).any() else (F32(np.inf) if np.isposinf(y).any() else F32(-np.inf))
            flags = 0 if my == -np.inf else 2
            tail = np.array([my.view(np.uint32), F32(0.0 if my == -np.inf else np.nan).view(np.uint32),
                             np.uint32(flags), np.uint32(1)], dtype=np.uint32)
        else:
            sel = np.where(fin)[0]
            c = _code(y[sel], idx[sel])
            c = np.sort(c)[::-1][:K]
            codes[:len(c)] = c
            my = F32(y[fin].max())
            se = np.exp((y[fin] - my).astype(np.float64)).sum()
            tail = np.array([my.view(np.uint32), F32(se).view(np.uint32), np.uint32(0), np.uint32(len(c))],
                            dtype=np.uint32)
        out[b, :8 * K] = codes.view(np.uint8)
        out[b, 8 * K:] = tail.view(np.uint8)
    return out.reshape(-1)


def merge_records(recs: np.ndarray, nshards: int, B: int, K: int, V: int, temperature, top_p, uniforms):
    """Tokens and per-row results (``restated.RowResult``) from shard-major records."""
    recs = np.asarray(recs, dtype=np.uint8).reshape(nshards, B, record_bytes(K))
    toks, results = [], []
    for b in range(B):
        codes = np.concatenate([recs[s, b, :8 * K].view(np.uint64) for s in range(nshards)])
        tails = np.stack([recs[s, b, 8 * K:].view(np.uint32) for s in range(nshards)])
        codes = codes[codes != 0]
        maxes = tails[:, 0].view(F32)
        T = float(temperature[b])
        special = bool((tails[:, 2] & 2).any()) or np.isnan(maxes).any() or not np.isfinite(maxes).any()
        if T <= 0.0 or special:
            best = int(codes.max())
            toks.append(int(~np.uint32(best & 0xFFFFFFFF) & np.uint32(0xFFFFFFFF)))
            results.append(None)
            continue
        keys = (codes >> np.uint64(32)).astype(np.uint32)
        idx = (~(codes & np.uint64(0xFFFFFFFF)).astype(np.uint32)).astype(np.int64)
        vals = np.where(keys & np.uint32(0x80000000), keys & np.uint32(0x7FFFFFFF), ~keys).astype(np.uint32).view(F32)
        keep = vals > -np.inf
        row = np.full(V, -np.inf, dtype=F32)
        row[idx[keep]] = vals[keep]
        res = R.sample_row(row, 1.0, top_k=K, top_p=float(top_p[b]), u=float(uniforms[b]))
        toks.append(res.token)
        results.append(res)
    return np.array(toks, dtype=np.int32), results
