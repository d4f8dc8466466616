"""Run under torch.distributed.run with one rank per GPU (NCCL): row mode and vocabulary mode
against the oracle.  Exits non-zero on a mismatch."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from localstrm_b200 import workloads as wl  # noqa: E402
from localstrm_b200.distributed import RowShardSampler, VocabShardSampler, shard_rows, shard_vocab  # noqa: E402
from localstrm_b200.sampling import RowParams  # noqa: E402
from oracle import restated as R  # noqa: E402
from tests import parity as P  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    bad = 0
    try:
        # rows
        w = wl.config3(seed=11, B=37, V=151_936, H=256)
        a, b = shard_rows(w.B, world, rank)
        x = torch.from_numpy(w.logits[a:b]).to(dev)
        prm = RowParams.from_arrays(dev, temperature=w.temperature[a:b], top_k=w.top_k[a:b], top_p=w.top_p[a:b],
                                    min_p=w.min_p[a:b], repetition_penalty=w.repetition_penalty[a:b],
                                    frequency_penalty=w.frequency_penalty[a:b],
                                    presence_penalty=w.presence_penalty[a:b])
        offs = w.hist_offsets[a:b + 1] - w.hist_offsets[a]
        ids = w.hist_ids[w.hist_offsets[a]:w.hist_offsets[b]]
        ho = torch.from_numpy(offs.astype(np.int32)).to(dev)
        hi = torch.from_numpy(ids.astype(np.int32)).to(dev)
        u = torch.from_numpy(w.uniforms[a:b]).to(dev)
        tok = RowShardSampler(dev).sample(x, prm, ho, hi, u, w.B).cpu().numpy()
        res = R.sample_batch(w, want_detail=True)
        ref = np.array([r.token for r in res])
        # a draw may differ only where the uniform sits within 1e-6 of a CDF boundary
        bad += sum(1 for i in np.nonzero(tok != ref)[0]
                   if res[i].special or not P.draw_is_boundary(res[i].probs, float(w.uniforms[i])))
        # vocabulary
        K = 64
        w5 = wl.config5(seed=3, B=32, V=256_000)
        off, stop = shard_vocab(w5.V, world, rank)
        x5 = torch.from_numpy(np.ascontiguousarray(w5.logits[:, off:stop])).to(dev)
        tok5 = VocabShardSampler(dev, K=K).sample(
            x5, off, w5.V, torch.from_numpy(w5.temperature).to(dev), torch.from_numpy(w5.top_p).to(dev),
            torch.from_numpy(w5.uniforms).to(dev)).cpu().numpy()
        res5 = [R.sample_row(w5.logits[i], float(w5.temperature[i]), top_k=K, top_p=float(w5.top_p[i]),
                             u=float(w5.uniforms[i])) for i in range(w5.B)]
        ref5 = np.array([r.token for r in res5])
        bad += sum(1 for i in np.nonzero(tok5 != ref5)[0]
                   if res5[i].special or not P.draw_is_boundary(res5[i].probs, float(w5.uniforms[i])))
        print(f"rank {rank}: row mismatches {(tok != ref).sum()}, vocab mismatches {(tok5 != ref5).sum()}",
              flush=True)
    finally:
        dist.destroy_process_group()
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
