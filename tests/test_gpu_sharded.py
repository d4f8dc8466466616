"""Vocabulary-sharded mode on the GPU.  The shards of a row are column blocks of one logits
buffer (each launch of the shard step sees its block through the row stride), so one device
checks the kernels for any shard count; the records are compared with the oracle's byte for
byte, the merged draw and kept set with the oracle on the whole row (top-k = K, top-p)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from localstrm_b200 import _lib
from localstrm_b200 import workloads as wl
from localstrm_b200.distributed import shard_vocab
from oracle import restated as R
from oracle import sharded as OS
from tests import parity as P

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


DT_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _gpu_records(lib, x, w, n, K):
    rb = lib.lss_shard_record_bytes(K)
    T = torch.from_numpy(w.temperature).cuda()
    recs = []
    for s in range(n):
        off, stop = shard_vocab(w.V, n, s)
        rec = torch.empty(w.B * rb, dtype=torch.uint8, device="cuda")
        view = x[:, off:stop]
        _lib.check("lss_shard_topk", lib.lss_shard_topk(view.data_ptr(), DT_CODE[x.dtype], w.B, stop - off,
                                                         view.stride(0), off, T.data_ptr(), K, rec.data_ptr(),
                                                         None))
        recs.append(rec)
    return torch.cat(recs), T


def _merge(lib, gathered, w, n, K, T, detail=True):
    tp = torch.from_numpy(w.top_p).cuda()
    u = torch.from_numpy(w.uniforms).cuda()
    tok = torch.empty(w.B, dtype=torch.int32, device="cuda")
    kept = torch.empty((w.B, w.V), dtype=torch.uint8, device="cuda") if detail else None
    probs = torch.empty((w.B, w.V), dtype=torch.float32, device="cuda") if detail else None
    ws = torch.empty(lib.lss_shard_merge_workspace_bytes(w.B), dtype=torch.uint8, device="cuda")
    _lib.check("lss_shard_merge", lib.lss_shard_merge(
        gathered.data_ptr(), n, w.B, K, w.V, T.data_ptr(), tp.data_ptr(), u.data_ptr(), tok.data_ptr(),
        kept.data_ptr() if detail else None, probs.data_ptr() if detail else None, ws.data_ptr(), ws.numel(), None))
    torch.cuda.synchronize()
    return tok.cpu().numpy(), (kept.cpu().numpy().astype(bool) if detail else None), \
        (probs.cpu().numpy() if detail else None)


@needs_cuda
@pytest.mark.parametrize("n", [1, 2, 8])
def test_vocab_shards_match_oracle(n):
    lib = _lib.load()
    K = 64
    w = wl.config5(seed=9, B=16, V=64_000)
    x = torch.from_numpy(w.logits).cuda()
    gathered, T = _gpu_records(lib, x, w, n, K)
    rb = lib.lss_shard_record_bytes(K)
    g = gathered.cpu().numpy().reshape(n, w.B, rb)
    for s in range(n):
        off, stop = shard_vocab(w.V, n, s)
        ref = OS.shard_records(w.logits[:, off:stop], off, w.temperature, K).reshape(w.B, rb)
        assert np.array_equal(g[s, :, :8 * K], ref[:, :8 * K]), s          # codes
        assert np.array_equal(g[s, :, 8 * K:8 * K + 4], ref[:, 8 * K:8 * K + 4])  # max
        se, se_ref = g[s, :, 8 * K + 4:8 * K + 8].view(np.float32), ref[:, 8 * K + 4:8 * K + 8].view(np.float32)
        assert np.allclose(se, se_ref, rtol=1e-5)
    tok, kept, probs = _merge(lib, gathered, w, n, K, T)
    for b in range(w.B):
        res = R.sample_row(w.logits[b], float(w.temperature[b]), top_k=K, top_p=float(w.top_p[b]),
                           u=float(w.uniforms[b]))
        assert P.compare_kept(w, b, kept[b], res.kept, res) == ""
        both = kept[b] & res.kept
        assert P.probs_close(probs[b], res.probs, both) <= P.PROB_RTOL
        if int(tok[b]) != res.token:
            assert P.draw_is_boundary(res.probs, float(w.uniforms[b])), (b, int(tok[b]), res.token)


@needs_cuda
@pytest.mark.parametrize("n", [2, 4, 8])
def test_config5_full_size_emulated_shards(n):
    """Config 5 at its stated size (B=128, V=256,000, top-k 64, top-p 0.9) split into n column
    shards of one buffer: every record byte for byte against the oracle, then the merged kept
    set, probabilities and draw of every row against the oracle on the whole row."""
    lib = _lib.load()
    K = 64
    w = wl.config5(seed=0)
    assert (w.B, w.V) == (128, 256_000)
    x = torch.from_numpy(w.logits).cuda()
    gathered, T = _gpu_records(lib, x, w, n, K)
    rb = lib.lss_shard_record_bytes(K)
    g = gathered.cpu().numpy().reshape(n, w.B, rb)
    for s in range(n):
        off, stop = shard_vocab(w.V, n, s)
        ref = OS.shard_records(w.logits[:, off:stop], off, w.temperature, K).reshape(w.B, rb)
        assert np.array_equal(g[s, :, :8 * K + 4], ref[:, :8 * K + 4]), s          # codes, max
        assert np.array_equal(g[s, :, 8 * K + 8:], ref[:, 8 * K + 8:]), s          # flags, count
        se, se_ref = g[s, :, 8 * K + 4:8 * K + 8].view(np.float32), ref[:, 8 * K + 4:8 * K + 8].view(np.float32)
        assert np.allclose(se, se_ref, rtol=1e-5), s
    tok, kept, probs = _merge(lib, gathered, w, n, K, T)
    for b in range(w.B):
        res = R.sample_row(w.logits[b], float(w.temperature[b]), top_k=K, top_p=float(w.top_p[b]),
                           u=float(w.uniforms[b]))
        assert P.compare_kept(w, b, kept[b], res.kept, res) == "", b
        assert kept[b][int(tok[b])], b
        both = kept[b] & res.kept
        assert P.probs_close(probs[b], res.probs, both) <= P.PROB_RTOL, b
        own = R.draw_inverse_cdf(kept[b], np.where(kept[b], probs[b], 0).astype(np.float32), float(w.uniforms[b]))
        assert int(tok[b]) == own or P.draw_is_boundary(np.where(kept[b], probs[b], 0), float(w.uniforms[b])), b
        if int(tok[b]) != res.token:
            assert P.draw_is_boundary(res.probs, float(w.uniforms[b])), (b, int(tok[b]), res.token)


@needs_cuda
@pytest.mark.parametrize("dtype,V,n,K", [("bf16", 64_000, 2, 64), ("f16", 64_000, 8, 64), ("f32", 64_001, 2, 64),
                                         ("f32", 300_000, 1, 256), ("bf16", 40_000, 4, 16)])
def test_vocab_shard_records_dtypes_and_layouts(dtype, V, n, K):
    """Shard records of 16-bit logits (compared with the oracle on the widened values), of
    shards that start off a 16-byte boundary (V odd), of a long shard row with K = 256 and of
    a small K: codes, max, flags and count byte for byte, the sum within 1e-5."""
    lib = _lib.load()
    w = wl.config5(seed=13, B=12, V=V)
    w.logits = wl.round_to_dtype(w.logits, dtype)
    w.temperature[3] = 0.0  # a greedy row: codes of the raw values
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    x = torch.from_numpy(w.logits).to(tdt).cuda()
    gathered, T = _gpu_records(lib, x, w, n, K)
    rb = lib.lss_shard_record_bytes(K)
    g = gathered.cpu().numpy().reshape(n, w.B, rb)
    for s in range(n):
        off, stop = shard_vocab(w.V, n, s)
        ref = OS.shard_records(w.logits[:, off:stop], off, w.temperature, K).reshape(w.B, rb)
        assert np.array_equal(g[s, :, :8 * K + 4], ref[:, :8 * K + 4]), s          # codes, max
        assert np.array_equal(g[s, :, 8 * K + 8:], ref[:, 8 * K + 8:]), s          # flags, count
        se, se_ref = g[s, :, 8 * K + 4:8 * K + 8].view(np.float32), ref[:, 8 * K + 4:8 * K + 8].view(np.float32)
        assert np.allclose(se, se_ref, rtol=1e-5), s


@needs_cuda
def test_vocab_shards_special_rows():
    lib = _lib.load()
    K, n = 32, 4
    w = wl.config5(seed=4, B=6, V=8_192)
    w.logits[0, 5000] = np.nan                  # NaN in shard 2
    w.logits[1, 100] = np.inf                   # +inf in shard 0
    w.logits[2, :2048] = -np.inf                # shard 0 all -inf, the rest finite
    w.logits[3, :] = -np.inf                    # the whole row -inf
    w.temperature[4] = 0.0                      # greedy row
    w.logits[4, 7000] = w.logits[4].max() + 1.0
    x = torch.from_numpy(w.logits).cuda()
    gathered, T = _gpu_records(lib, x, w, n, K)
    tok, _, _ = _merge(lib, gathered, w, n, K, T, detail=False)
    ref, _ = OS.merge_records(gathered.cpu().numpy(), n, w.B, K, w.V, w.temperature, w.top_p, w.uniforms)
    for b in range(w.B):
        full = R.sample_row(w.logits[b], float(w.temperature[b]), top_k=K, top_p=float(w.top_p[b]),
                            u=float(w.uniforms[b]))
        assert int(tok[b]) == full.token == int(ref[b]), (b, int(tok[b]), full.token, int(ref[b]))


@needs_cuda
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_nccl_row_and_vocab_modes():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29631", os.path.join(root, "tests", "mgpu_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
