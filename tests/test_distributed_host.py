"""Host logic of the multi-GPU modes on CPU: block splits, and the row / vocabulary exchange
over gloo with world size 2 (the oracle stands in for the per-rank GPU step)."""
import json
import os
import socket

import pytest
import torch.multiprocessing as mp

from localstrm_b200.distributed import shard_rows, shard_vocab


@pytest.mark.parametrize("B,world", [(0, 1), (1, 2), (7, 2), (256, 3), (1024, 8), (5, 8)])
def test_shard_rows_cover_the_batch_once(B, world):
    blocks = [shard_rows(B, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == B
    for (a, b), (c, d) in zip(blocks, blocks[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1
    assert shard_vocab(B, world, world - 1) == blocks[-1]


def test_shard_rows_rejects_bad_splits():
    with pytest.raises(ValueError):
        shard_rows(4, 0, 0)
    with pytest.raises(ValueError):
        shard_rows(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_and_vocab_exchange_gloo_world2(tmp_path):
    from tests.dist_workers import host_exchange
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=host_exchange, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [json.load(open(os.path.join(tmp_path, f"rank{r}.json"))) for r in range(2)]
    for r in res:
        assert r["rows"] == r["rows_ref"]
        assert r["vocab"] == r["vocab_ref"]
    assert res[0]["vocab"] == res[1]["vocab"]


def test_vocab_mode_rejects_rows_it_cannot_serve():
    import torch
    from localstrm_b200.distributed import VocabShardSampler
    s = VocabShardSampler("cpu", K=64, records=lambda *a: None, merge=lambda *a: None, record_bytes=528)
    s.check_params(top_k=[64, 64], min_p=[0.0, 1.0], repetition_penalty=[1.0, 1.0],
                   frequency_penalty=torch.zeros(2), presence_penalty=[0.0, 0.0])
    for bad in (dict(top_k=[64, 20]), dict(top_k=[-1, 64]), dict(min_p=[0.0, 0.05]),
                dict(repetition_penalty=[1.0, 1.1]), dict(frequency_penalty=[0.0, 0.3]),
                dict(presence_penalty=torch.tensor([0.2, 0.0]))):
        with pytest.raises(ValueError):
            s.check_params(**bad)
