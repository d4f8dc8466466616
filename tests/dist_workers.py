"""Rank bodies for the multi-process tests (spawned; gloo on CPU or NCCL on GPUs)."""
from __future__ import annotations

import json
import os

import numpy as np
import torch
import torch.distributed as dist


def _oracle_rows(w, rows):
    from oracle import restated as R
    return [r.token for r in R.sample_batch(w, want_detail=False, rows=list(rows))]


def host_exchange(rank: int, world: int, port: int, outdir: str) -> None:
    """Row and vocabulary exchange logic over gloo, with the oracle as the per-rank step."""
    from localstrm_b200 import workloads as wl
    from localstrm_b200.distributed import RowShardSampler, VocabShardSampler, shard_rows, shard_vocab
    from oracle import restated as R
    from oracle import sharded as OS

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    out = {}
    try:
        # rows: an odd batch, penalties on
        w = wl.config3(seed=5, B=7, V=3000, H=40)
        start, stop = shard_rows(w.B, world, rank)

        def local(logits, params, hist_off, hist_ids, uniforms):
            return torch.tensor(_oracle_rows(w, range(start, stop)), dtype=torch.int32)

        rs = RowShardSampler("cpu", sample_local=local)
        tok = rs.sample(torch.zeros(stop - start, w.V), None, None, None, None, w.B)
        out["rows"] = tok.tolist()
        out["rows_ref"] = _oracle_rows(w, range(w.B))

        # vocabulary: config 5 split into `world` column blocks
        K = 16
        w5 = wl.config5(seed=2, B=6, V=4001)
        off, stop_v = shard_vocab(w5.V, world, rank)

        def records(logits, offset, temperature, K_):
            return torch.from_numpy(OS.shard_records(logits.numpy(), offset, temperature.numpy(), K_))

        def merge(gathered, nshards, B, K_, V, temperature, top_p, uniforms):
            toks, _ = OS.merge_records(gathered.numpy(), nshards, B, K_, V, temperature.numpy(),
                                       top_p.numpy(), uniforms.numpy())
            return torch.from_numpy(toks)

        vs = VocabShardSampler("cpu", K=K, records=records, merge=merge, record_bytes=OS.record_bytes(K))
        logits = torch.from_numpy(np.ascontiguousarray(w5.logits[:, off:stop_v]))
        tok5 = vs.sample(logits, off, w5.V, torch.from_numpy(w5.temperature), torch.from_numpy(w5.top_p),
                         torch.from_numpy(w5.uniforms))
        out["vocab"] = tok5.tolist()
        out["vocab_ref"] = [R.sample_row(w5.logits[b], float(w5.temperature[b]), top_k=K,
                                         top_p=float(w5.top_p[b]), u=float(w5.uniforms[b])).token
                            for b in range(w5.B)]
    finally:
        dist.destroy_process_group()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(out, f)
