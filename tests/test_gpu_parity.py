"""Native sampler (through the C ABI) against the CPU oracle on the same seeded inputs.

Bars (``tests/parity.py``): greedy / NaN-guard tokens bit-exact; kept set bit-exact up to
tie groups and the 1e-6 boundary band; probabilities within 1e-5 relative; drawn token
exact unless the uniform lies within 1e-6 of a CDF boundary.
"""
import numpy as np
import pytest
import torch

from localstrm_b200 import workloads as wl
from oracle import restated as R
from tests import gpu_util as G
from tests import parity as P
from tests.golden.sets import golden_sets

pytestmark = pytest.mark.gpu

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def check_workload(w, out, rows=None, detail=True):
    """Assert parity of a GPU result against the oracle; returns per-path row counts.

    With ``detail`` (kept sets and probabilities read back) every sampled row must satisfy:
    the kept set matches the oracle's under the tie/band rules; the probabilities agree within
    ``PROB_RTOL``; the drawn token is kept by the GPU and is the inverse-CDF draw of the
    row's uniform over the GPU's own kept set and probabilities (unless the uniform sits
    within ``BAND`` of one of that distribution's CDF boundaries); and when the kept sets are
    identical, the token is the oracle's own draw (same boundary exception).  Without
    ``detail`` only the tokens are known: greedy / NaN-guard rows must be exact and every
    other token must be the oracle's draw unless the uniform is on a boundary."""
    rows = range(w.B) if rows is None else rows
    worst = 0.0
    stats = {}
    for r in rows:
        res = R.sample_batch(w, want_detail=True, rows=[r])[0]
        path = int(out["paths"][r])
        stats[path] = stats.get(path, 0) + 1
        tok = int(out["tokens"][r])
        u = float(w.uniforms[r])
        if res.special in ("greedy", "nan_inf"):
            assert tok == res.token, (w.name, r, res.special, tok, res.token)
            continue
        if detail:
            kept_g = out["kept"][r]
            probs_g = np.where(kept_g, out["probs"][r], np.float32(0.0)).astype(np.float32)
            assert kept_g[tok], (w.name, r, "drawn token not in the GPU's kept set", tok)
            msg = P.compare_kept(w, r, kept_g, res.kept, res)
            assert msg == "", f"{w.name}: {msg}"
            both = kept_g & res.kept
            worst = max(worst, P.probs_close(out["probs"][r], res.probs, both))
            own = R.draw_inverse_cdf(kept_g, probs_g, u)
            assert tok == own or P.draw_is_boundary(probs_g, u), \
                (w.name, r, "token is not the draw over the GPU's own distribution", tok, own, u)
            if np.array_equal(kept_g, res.kept) and tok != res.token:
                assert P.draw_is_boundary(res.probs, u), (w.name, r, tok, res.token, u)
        else:
            assert tok == res.token or P.draw_is_boundary(res.probs, u), (w.name, r, tok, res.token, u)
    assert worst <= P.PROB_RTOL, (w.name, worst)
    return stats


@needs_cuda
@pytest.mark.parametrize("name", list(golden_sets()))
def test_golden_sets(name):
    w = golden_sets()[name]
    out = G.run(w)
    assert out["flags"] == 0
    check_workload(w, out)


@needs_cuda
def test_config3_full():
    w = wl.config3(seed=0)
    out = G.run(w)
    assert out["flags"] == 0
    stats = check_workload(w, out)
    assert set(stats) <= {2, 3, 4, 5}


@needs_cuda
def test_headline_full():
    w = wl.headline(seed=1)
    out = G.run(w)
    assert out["flags"] == 0
    check_workload(w, out)


@needs_cuda
def test_config2_bf16():
    w = wl.config2(seed=3)
    out = G.run(w)
    assert out["flags"] == 0
    stats = check_workload(w, out)
    assert stats.get(3, 0) + stats.get(4, 0) + stats.get(5, 0) == w.B


@needs_cuda
@pytest.mark.parametrize("dtype,V,pad", [("f32", wl.QWEN_VOCAB, 0), ("bf16", wl.QWEN_VOCAB, 0),
                                         ("f32", 40_001, 0), ("f32", 40_001, 3), ("bf16", 40_001, 1)])
def test_history_on_top_tokens(dtype, V, pad):
    """The rows' largest raw logits are history tokens that the penalties push down: the
    streaming pass counts them with their raw values, so its thresholds lie above the exact
    cut, and the resolve kernel must re-read chunks of those slices (16-byte loads, or one by
    one for rows that start off a 16-byte boundary; ragged row ends).  Parity on every row,
    and the rows stay in the resolve kernel (path 3) instead of going to the second kernel."""
    w = wl.history_on_top(seed=11, V=V, dtype=dtype)
    out = G.run(w, dtype=dtype, row_stride=(V + pad) if pad else None)
    assert out["flags"] == 0
    stats = check_workload(w, out)
    assert stats.get(3, 0) == w.B, stats


@needs_cuda
@pytest.mark.parametrize("name,rows", [
    ("cfg1", [0]), ("cfg1", [2, 3]), ("cfg1", [1, 4, 5, 6]),            # greedy; top-k 50 + top-p
    ("cfg2", [0]), ("cfg2", [1, 2, 3, 4]), ("cfg2", [5, 6]),           # bf16, mixed parameters, history
    ("cfg3", [0]), ("cfg3", [1, 2, 10, 51]),                           # -inf rows, exact max ties
    ("hist_on_top", [0, 1, 2, 3]),                                     # history on the largest logits
    ("headline", [7])])
def test_latency_path_small_batches(name, rows):
    """Batches of up to four rows take the single-kernel latency path (one cluster per row;
    rows it cannot bound go to the deferred-row kernel).  Parity on every row, and the greedy
    and gathered rows stay in that kernel."""
    w = {"cfg1": lambda: wl.config1(seed=2), "cfg2": lambda: wl.config2(seed=6),
         "cfg3": lambda: wl.config3(seed=8, B=64), "hist_on_top": lambda: wl.history_on_top(seed=4),
         "headline": lambda: wl.headline(seed=3, B=16)}[name]().rows(rows)
    out = G.run(w)
    assert out["flags"] == 0
    stats = check_workload(w, out)
    assert sum(stats.values()) == w.B


@needs_cuda
@pytest.mark.parametrize("V,pad,dtype", [(4099, 3, "f32"), (40_001, 1, "bf16"), (777, 0, "f32"), (151_936, 0, "f16")])
def test_latency_path_layouts(V, pad, dtype):
    """The latency path on small and ragged vocabularies, rows that start off a 16-byte
    boundary, and 16-bit logits."""
    w = wl.config3(seed=12, B=3, V=V, H=96)
    w.logits = wl.round_to_dtype(w.logits, dtype)
    w.top_k[1] = 40
    w.min_p[2] = 0.0
    w.temperature[0] = 0.0
    out = G.run(w, dtype=dtype, row_stride=(V + pad) if pad else None)
    assert out["flags"] == 0
    check_workload(w, out)


@needs_cuda
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_half_dtypes_match_upcast(dtype):
    w = wl.config1(seed=5)
    w.logits = wl.round_to_dtype(w.logits, dtype)
    out = G.run(w, dtype=dtype)
    check_workload(w, out)


@needs_cuda
@pytest.mark.parametrize("stride_extra", [1, 3, 16])
def test_row_stride_and_alignment(stride_extra):
    w = wl.config3(seed=7, B=6, V=4099 + stride_extra, H=64)
    out = G.run(w, row_stride=w.V + stride_extra)
    check_workload(w, out)


@needs_cuda
def test_dense_paths_top_p_only_flat():
    # Flat rows with top-p only: the nucleus has tens of thousands of tokens (dense path).
    w = wl.config2(seed=4, B=8)
    w.top_k[:] = 0
    w.min_p[:] = 0.0
    w.top_p[:] = np.array([0.9, 0.99, 0.5, 0.7, 0.95, 0.999, 0.3, 0.8], np.float32)
    w.temperature[:] = 1.3
    out = G.run(w)
    stats = check_workload(w, out)
    assert stats.get(4, 0) >= 1


@needs_cuda
def test_dense_top_k_large_and_no_filter():
    w = wl.config2(seed=6, B=6)
    w.min_p[:] = 0.0
    w.top_k[:] = np.array([5000, 20000, 0, 0, 100000, 4097], np.int32)
    w.top_p[:] = np.array([1.0, 0.9, 1.0, 0.6, 0.97, 1.0], np.float32)
    out = G.run(w)
    stats = check_workload(w, out)
    assert stats.get(4, 0) >= 3


@needs_cuda
def test_long_histories_global_hash():
    w = wl.config3(seed=8, B=4, V=32000, H=6000)
    out = G.run(w)
    check_workload(w, out)


@needs_cuda
def test_large_vocab_one_cta_per_sm():
    w = wl.config5(seed=9, B=4, V=256_000)
    out = G.run(w)
    check_workload(w, out)


@needs_cuda
def test_greedy_seam_matches_torch_argmax():
    from localstrm_b200.sampling import greedy_batch
    torch.manual_seed(0)
    for V in (1, 7, 4099, 151_936):
        x = torch.randn(37, V, device="cuda") * 3
        x[3, V // 2] = float("nan")
        x[5, :] = float("-inf")
        if V > 2:
            x[6, 1] = x[6].max() + 1
            x[6, 2] = x[6, 1]
        for dt in (torch.float32, torch.bfloat16, torch.float16):
            y = x.to(dt)
            got = greedy_batch(y).long().cpu()
            ref = torch.tensor([R.argmax_nan_first(r) for r in y.float().cpu().numpy()])
            assert torch.equal(got, ref), (V, dt)


@needs_cuda
def test_drop_in_sample_next_token():
    from localstrm_b200 import SamplingParams, sample_next_token
    x = torch.tensor([[1.0, 2.0, 5.0, 0.5]], device="cuda")
    assert sample_next_token(x, SamplingParams.greedy()) == 2
    assert sample_next_token(x, SamplingParams(temperature=1e-3, repetition_penalty=10.0),
                             past_token_ids=[2]) == 1
    with pytest.raises(RuntimeError):
        sample_next_token(x.cpu(), SamplingParams.greedy())


@needs_cuda
def test_bad_history_offsets_raise_a_flag_and_stay_in_bounds():
    """Offsets that decrease or point past hist_total: the row's history is ignored and
    LSS_FLAG_BAD_HISTORY is raised; the other rows are sampled with their histories."""
    from localstrm_b200.sampling import BatchSampler
    w = wl.config3(seed=31, B=4, V=4096, H=20)
    good = w.hist_offsets.copy()
    for bad in (np.array([0, 20, 10, 60, 80], np.int32),      # row 1 decreasing
                np.array([0, 20, 40, 60, 1000], np.int32)):   # row 3 past the end
        x, prm, ho, hi, u = G.device_inputs(w)
        ho.copy_(torch.from_numpy(bad))
        s = BatchSampler("cuda")
        tok = s.sample(x, prm, ho, hi, u)
        torch.cuda.synchronize()
        assert s.status() & 0x2, bad
        got = tok.cpu().numpy()
        assert ((got >= 0) & (got < w.V)).all()
        H = w.hist_ids.size
        valid = [r for r in range(w.B) if 0 <= bad[r] <= bad[r + 1] <= H]
        # Rows whose ranges overlap another row's are unreliable by contract: skip them.
        alone = [r for r in valid if not any(q != r and max(bad[r], bad[q]) < min(bad[r + 1], bad[q + 1])
                                             for q in valid)]
        assert alone
        for r in alone:
            ww = w.rows([r])
            ww.hist_ids = w.hist_ids[bad[r]:bad[r + 1]].copy()
            ww.hist_offsets = np.array([0, bad[r + 1] - bad[r]], np.int32)
            res = R.sample_batch(ww, want_detail=True)[0]
            assert int(got[r]) == res.token or P.draw_is_boundary(res.probs, float(w.uniforms[r])), (r, bad)
    assert np.array_equal(w.hist_offsets, good)


@needs_cuda
def test_empty_batch_and_native_library_loaded():
    from localstrm_b200 import sampling as S
    s = S.BatchSampler("cuda")
    x = torch.empty((0, 10), device="cuda")
    prm = S.RowParams.from_params([], "cuda")
    tok = s.sample(x, prm, None, None, torch.empty(0, device="cuda"))
    assert tok.numel() == 0
    maps = open("/proc/self/maps").read()
    assert "liblss.so" in maps


def _chi_square_row(w, r, B, calls):
    """2^20-ish draws of row r of workload w (the row tiled B times, history included, ``calls``
    calls with fresh uniforms): the token histogram against the oracle's final probabilities
    (``scipy.stats.chisquare``, bins with an expected count below 5 merged)."""
    from scipy.stats import chisquare
    from localstrm_b200.sampling import BatchSampler, RowParams
    res = R.sample_batch(w, want_detail=True, rows=[r])[0]
    assert res.special == ""
    V = w.V
    s = BatchSampler("cuda")
    logits = torch.from_numpy(w.logits[r]).to(G.TORCH_DT[w.dtype]).cuda().reshape(1, V).expand(B, V).contiguous()
    rep = lambda a: np.full(B, a[r])
    prm = RowParams.from_arrays("cuda", temperature=rep(w.temperature), top_k=rep(w.top_k),
                                top_p=rep(w.top_p), min_p=rep(w.min_p),
                                repetition_penalty=rep(w.repetition_penalty),
                                frequency_penalty=rep(w.frequency_penalty),
                                presence_penalty=rep(w.presence_penalty))
    h = w.hist_ids[w.hist_offsets[r]:w.hist_offsets[r + 1]].astype(np.int32)
    h_off = h_ids = None
    if h.size:
        h_off = torch.arange(B + 1, dtype=torch.int32, device="cuda") * int(h.size)
        h_ids = torch.from_numpy(np.tile(h, B)).cuda()
    gen = torch.Generator(device="cuda").manual_seed(123 + r)
    counts = torch.zeros(V, dtype=torch.int64, device="cuda")
    for _ in range(calls):
        u = torch.rand(B, device="cuda", generator=gen)
        tok = s.sample(logits, prm, h_off, h_ids, u)
        counts += torch.bincount(tok.long(), minlength=V)
    counts = counts.cpu().numpy()
    assert counts.sum() == B * calls
    assert counts[~res.kept].sum() == 0
    exp = res.probs.astype(np.float64) * B * calls
    keep = res.kept
    obs, ex = counts[keep].astype(np.float64), exp[keep]
    big = ex >= 5
    o2 = np.append(obs[big], obs[~big].sum())
    e2 = np.append(ex[big], ex[~big].sum())
    if e2[-1] == 0:
        o2, e2 = o2[:-1], e2[:-1]
    e2 *= o2.sum() / e2.sum()
    if o2.size < 2:  # a single bin: every draw landed on the one token the oracle keeps
        return
    assert chisquare(o2, e2).pvalue > 1e-4, (w.name, r, o2[:10], e2[:10])


@needs_cuda
def test_chi_square_distribution():
    """2^20 draws of a synthetic row (V=1,000, k200/p0.9/mp0.01) against the oracle."""
    V = 1000
    rng = np.random.default_rng(11)
    w = wl.config1(seed=0, V=V)
    w.logits[2] = (rng.standard_normal(V) * 1.5).astype(np.float32)
    w.temperature[2], w.top_k[2], w.top_p[2], w.min_p[2] = 0.9, 200, 0.9, 0.01
    _chi_square_row(w, 2, B=65536, calls=16)


@needs_cuda
@pytest.mark.parametrize("cfg,row", [("cfg1", 3), ("cfg3", 45)])
def test_chi_square_config_rows_full_vocab(cfg, row):
    """2^20 draws of one BASELINE config row at its full vocabulary: config 1 row 3
    (V=151,936, T0.8 k50 p0.9, 40 kept tokens) and config 3 row 45 (V=128,256, T0.7 p0.95
    mp0.05 with repetition/frequency/presence penalties over its 2,048-id history)."""
    w = wl.config1(seed=0) if cfg == "cfg1" else wl.config3(seed=0)
    _chi_square_row(w, row, B=4096, calls=256)


@needs_cuda
def test_config4_bf16_all_features():
    """Config 4 (B=1,024 bf16, every feature on): kept set, probabilities and draw of every
    row against the oracle."""
    w = wl.config4(seed=2)
    out = G.run(w)
    assert out["flags"] == 0
    check_workload(w, out)


@needs_cuda
def test_cuda_graph_capture_and_replay():
    """prepare + rows captured once in a CUDA graph and replayed on new contents of the same
    buffers (the decode-loop use), against the oracle for both workloads."""
    from localstrm_b200 import _lib
    from localstrm_b200.sampling import BatchSampler
    w1 = wl.config3(seed=21, B=24, V=32_000, H=300)
    w2 = wl.config3(seed=22, B=24, V=32_000, H=300)
    w2.top_k[:] = np.array([0, 5, 50] * 8, np.int32)
    assert w1.hist_ids.size == w2.hist_ids.size
    s = BatchSampler("cuda")
    lib = _lib.load()
    x, prm, ho, hi, u = G.device_inputs(w1, s.device)
    tok = torch.empty(w1.B, dtype=torch.int32, device=s.device)
    H = int(hi.numel())
    ws = s.workspace(w1.B, w1.V, H)
    P_ = lambda t: t.data_ptr()

    def step(stream):
        _lib.check("prepare", lib.lss_sample_prepare(
            w1.B, w1.V, P_(prm.temperature), P_(prm.top_k), P_(prm.min_p), P_(prm.repetition_penalty),
            P_(prm.frequency_penalty), P_(prm.presence_penalty), P_(ho), P_(hi), H, P_(ws), ws.numel(), stream))
        _lib.check("rows", lib.lss_sample_rows(
            P_(x), 0, w1.B, w1.V, x.stride(0), P_(prm.temperature), P_(prm.top_k), P_(prm.top_p), P_(prm.min_p),
            P_(prm.repetition_penalty), P_(prm.frequency_penalty), P_(prm.presence_penalty), P_(ho), P_(hi), H,
            P_(u), P_(tok), None, None, P_(ws), ws.numel(), stream))

    step(torch.cuda.current_stream().cuda_stream)  # warm-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(torch.cuda.current_stream().cuda_stream)
    for w in (w1, w2, w1):
        x2, prm2, ho2, hi2, u2 = G.device_inputs(w, s.device)
        x.copy_(x2)
        ho.copy_(ho2)
        hi.copy_(hi2)
        u.copy_(u2)
        for name in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty", "frequency_penalty",
                     "presence_penalty"):
            getattr(prm, name).copy_(getattr(prm2, name))
        g.replay()
        torch.cuda.synchronize()
        got = tok.cpu().numpy()
        for r in range(w.B):
            res = R.sample_batch(w, want_detail=True, rows=[r])[0]
            if int(got[r]) != res.token:
                assert res.special == "" and P.draw_is_boundary(res.probs, float(w.uniforms[r])), (r, got[r])
