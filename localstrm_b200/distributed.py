"""Multi-GPU sampling, one process per GPU over ``torch.distributed``.

Two ways to split a batch:

* **Rows** (``RowShardSampler``): rows are independent, so each rank samples a contiguous block
  of rows with the single-GPU sampler and one all-gather hands every rank all token ids.  No
  collective touches the data path.
* **Vocabulary** (``VocabShardSampler``): each rank holds the columns ``[offset, offset + Vs)``
  of every row.  Each rank writes one record per row (the shard's K largest values of
  ``y = z / T``, its max and its sum of ``exp(y - max)``, ``lss_shard_topk``); one all-gather
  of the records is the exchange step; every rank then merges them and draws
  (``lss_shard_merge``: the reference's top-k with ``k = K``, top-p and the inverse-CDF draw of
  ``sampling.py:82-113,157-162`` over the union of the shards' candidates).

The per-rank compute steps are arguments with the native library as the default, so that the
exchange logic can be exercised with any backend of the same contract.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib


def shard_rows(B: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous block ``[start, stop)`` of rank ``rank``; the first ``B % world`` ranks get one
    row more."""
    if world < 1 or not 0 <= rank < world or B < 0:
        raise ValueError(f"bad split: B={B} world={world} rank={rank}")
    base, extra = divmod(B, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_vocab(V: int, world: int, rank: int) -> Tuple[int, int]:
    """Vocabulary columns ``[offset, offset + Vs)`` of rank ``rank`` (same split as rows)."""
    return shard_rows(V, world, rank)


def _world(group) -> Tuple[int, int]:
    return dist.get_world_size(group), dist.get_rank(group)


class RowShardSampler:
    """Each rank samples its own rows; ``sample`` returns all ``B_total`` token ids on every rank.

    ``sample_local(logits, params, hist_off, hist_ids, uniforms) -> int32 tokens`` samples the
    rank's rows; the default is the native ``BatchSampler``.
    """

    def __init__(self, device, group=None, sample_local: Optional[Callable] = None):
        self.group = group
        self.device = torch.device(device)
        if sample_local is None:
            from .sampling import BatchSampler
            sampler = BatchSampler(self.device)
            sample_local = sampler.sample
        self.sample_local = sample_local

    def sample(self, logits, params, hist_off, hist_ids, uniforms, B_total: int) -> torch.Tensor:
        world, rank = _world(self.group)
        start, stop = shard_rows(B_total, world, rank)
        n = stop - start
        if logits.shape[0] != n:
            raise ValueError(f"rank {rank} holds {logits.shape[0]} rows, its block has {n}")
        tok = self.sample_local(logits, params, hist_off, hist_ids, uniforms).to(torch.int32)
        per = -(-B_total // world)  # blocks padded to the largest one
        buf = torch.full((per,), -1, dtype=torch.int32, device=tok.device)
        buf[:n] = tok
        out = torch.empty(world * per, dtype=torch.int32, device=tok.device)
        dist.all_gather_into_tensor(out, buf, group=self.group)
        parts = [out[r * per: r * per + (shard_rows(B_total, world, r)[1] - shard_rows(B_total, world, r)[0])]
                 for r in range(world)]
        return torch.cat(parts)


class VocabShardSampler:
    """Vocabulary split across ranks: per-shard records, one all-gather, merge and draw.

    ``records(logits, offset, temperature, K) -> uint8 [B * record_bytes]`` and
    ``merge(gathered, nshards, B, K, V_total, temperature, top_p, uniforms) -> int32 tokens``
    default to the native kernels.
    """

    def __init__(self, device, K: int = 64, group=None, records: Optional[Callable] = None,
                 merge: Optional[Callable] = None, record_bytes: Optional[int] = None):
        self.group = group
        self.device = torch.device(device)
        self.K = int(K)
        self._lib = None
        if records is None or merge is None:
            self._lib = _lib.load()
        self.rec_bytes = int(record_bytes if record_bytes is not None else self._lib.lss_shard_record_bytes(self.K))
        if self.rec_bytes <= 0:
            raise ValueError(f"unsupported K={K}")
        self._records = records or self._native_records
        self._merge = merge or self._native_merge
        self._ws = None

    # ---- native steps
    def _native_records(self, logits, offset, temperature, K):
        B, Vs = logits.shape
        if not logits.is_cuda:
            raise RuntimeError("the native shard step needs CUDA tensors")
        dt = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[logits.dtype]
        rec = torch.empty(B * self.rec_bytes, dtype=torch.uint8, device=logits.device)
        stream = torch.cuda.current_stream(logits.device).cuda_stream
        _lib.check("lss_shard_topk", self._lib.lss_shard_topk(
            logits.data_ptr(), dt, B, Vs, logits.stride(0), int(offset), temperature.data_ptr(), K,
            rec.data_ptr(), stream))
        return rec

    def _native_merge(self, gathered, nshards, B, K, V_total, temperature, top_p, uniforms,
                      kept=None, probs=None):
        dev = gathered.device
        need = int(self._lib.lss_shard_merge_workspace_bytes(B))
        if self._ws is None or self._ws.numel() < need or self._ws.device != dev:
            self._ws = torch.empty(need, dtype=torch.uint8, device=dev)
        tokens = torch.empty(B, dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check("lss_shard_merge", self._lib.lss_shard_merge(
            gathered.data_ptr(), nshards, B, K, V_total, temperature.data_ptr(), top_p.data_ptr(),
            uniforms.data_ptr(), tokens.data_ptr(), kept.data_ptr() if kept is not None else None,
            probs.data_ptr() if probs is not None else None, self._ws.data_ptr(), self._ws.numel(), stream))
        return tokens

    def check_params(self, top_k=None, min_p=None, repetition_penalty=None, frequency_penalty=None,
                     presence_penalty=None) -> None:
        """Raises ``ValueError`` unless every row's reference parameters mean what this mode
        computes: top-k with ``k = K``, no min-p and no penalties (``sampling.py:38-115``).
        Arguments are the rows' values (sequences or tensors; ``None`` skips a field)."""
        def vals(x):
            if x is None:
                return None
            return (x.detach().cpu().tolist() if isinstance(x, torch.Tensor) else list(x))
        k = vals(top_k)
        if k is not None and any(int(v) != self.K for v in k):
            raise ValueError(f"vocabulary-sharded mode applies top-k with k={self.K}; rows with another "
                             "top_k (or top-k disabled) must be sampled in row mode")
        mp = vals(min_p)
        if mp is not None and any(0.0 < float(v) < 1.0 for v in mp):
            raise ValueError("vocabulary-sharded mode does not apply min-p; sample such rows in row mode")
        for name, x, neutral in (("repetition_penalty", repetition_penalty, 1.0),
                                 ("frequency_penalty", frequency_penalty, 0.0),
                                 ("presence_penalty", presence_penalty, 0.0)):
            v = vals(x)
            if v is not None and any(float(e) != neutral for e in v):
                raise ValueError(f"vocabulary-sharded mode does not apply {name}; sample such rows in row mode")

    # ---- the step
    def sample(self, logits, offset: int, V_total: int, temperature, top_p, uniforms,
               **row_params) -> torch.Tensor:
        """One token per row.  ``row_params`` (``top_k``, ``min_p``, ``repetition_penalty``,
        ``frequency_penalty``, ``presence_penalty``) are checked with ``check_params`` first
        when given."""
        if row_params:
            self.check_params(**row_params)
        world, _ = _world(self.group)
        B = logits.shape[0]
        rec = self._records(logits, offset, temperature, self.K)
        gathered = torch.empty(world * B * self.rec_bytes, dtype=torch.uint8, device=rec.device)
        dist.all_gather_into_tensor(gathered, rec, group=self.group)
        return self._merge(gathered, world, B, self.K, V_total, temperature, top_p, uniforms)
