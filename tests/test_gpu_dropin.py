"""The reference's entry points as its callers use them, on the GPU, against the oracle and the
reference's own golden vectors.

* ``apply_top_k_top_p_min_p(logits, top_k, top_p, min_p)`` (reference ``sampling.py:71-115``)
  on ``[V]`` and ``[B, V]`` tensors: the mask and the surviving values against the kept sets
  the reference itself produced (``tests/golden/cfg1.npz``, ``cfg5.npz``);
* ``sample_next_token(logits, params, past_token_ids)`` (``sampling.py:118-163``) on config-1
  rows with a history, the call's uniform reproduced from torch's CUDA generator so that the
  token can be compared exactly;
* ``sample_batch(logits, [SamplingParams...], [history lists...])``: a mixed batch of greedy
  and sampled rows with Python history lists;
* the engine's batched decode seam (``llm_engine.py:1129-1153``): several decode steps of a
  64-request batch with growing ``output_token_ids``, ``check_stop_batch`` / ``stop_reasons``
  for the token-id part of ``check_stop_criteria`` (``sampling.py:182-185``), finished
  requests leaving the batch.
"""
import numpy as np
import pytest
import torch

from localstrm_b200 import workloads as wl
from oracle import restated as R
from tests import parity as P
from tests.test_gpu_parity import check_workload

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _workload_from_batch(name, logits_f32, params, histories, uniforms):
    """A ``Workload`` holding exactly what a ``sample_batch`` call was given."""
    from localstrm_b200.sampling import build_history_csr
    B, V = logits_f32.shape
    offs, ids = build_history_csr(histories, B, V)
    f = lambda k: np.array([float(getattr(p, k)) for p in params], np.float32)
    return wl.Workload(name, np.ascontiguousarray(logits_f32, np.float32), "f32", f("temperature"),
                       np.array([int(p.top_k) for p in params], np.int32), f("top_p"), f("min_p"),
                       f("repetition_penalty"), f("frequency_penalty"), f("presence_penalty"),
                       offs, ids, np.asarray(uniforms, np.float32))


def _check_filter_against_golden(name, w, out, rows, scaled):
    """``out`` (the filtered rows) against the reference's kept sets for ``rows`` of ``w``."""
    g = P.load_golden(name)
    out = out.float().cpu().numpy()
    for i, r in enumerate(rows):
        kept_ref, _ = P.kept_from_golden(g, r, w.V)
        assert kept_ref is not None
        res = R.sample_batch(w, want_detail=True, rows=[r])[0]
        kept = out[i] > -np.inf
        msg = P.compare_kept(w, r, kept, kept_ref, res, P.reference_topp_band(w, r, res))
        assert msg == "", f"{name}: {msg}"
        # The surviving entries keep their input values; everything else is -inf.
        assert np.array_equal(out[i][kept], scaled[i][kept]), (name, r)
        assert np.all(np.isneginf(out[i][~kept])), (name, r)


def test_apply_top_k_top_p_min_p_rows_and_batch():
    from localstrm_b200.sampling import apply_top_k_top_p_min_p
    # Config 1, sampled rows 2-7 (T 0.8, top-k 50, top-p 0.9): the reference filtered x / T.
    w = wl.config1(seed=0)
    rows = list(range(2, 8))
    x = torch.from_numpy(w.logits[rows]).cuda() / torch.tensor(0.8, device="cuda")
    scaled = x.cpu().numpy()
    batch = apply_top_k_top_p_min_p(x, top_k=50, top_p=0.9, min_p=0.0)
    assert batch.shape == x.shape and batch.dtype == x.dtype
    _check_filter_against_golden("cfg1", w, batch, rows, scaled)
    one = apply_top_k_top_p_min_p(x[3], top_k=50, top_p=0.9, min_p=0.0)  # a [V] tensor
    assert one.shape == x[3].shape
    _check_filter_against_golden("cfg1", w, one.reshape(1, -1), [rows[3]], scaled[3:4])
    # Config 5 rows (T 1.0, top-k 64, top-p 0.9) straight from the logits.
    w5 = wl.config5(seed=0, B=16)
    x5 = torch.from_numpy(w5.logits).cuda()
    out5 = apply_top_k_top_p_min_p(x5, top_k=64, top_p=0.9)
    _check_filter_against_golden("cfg5", w5, out5, list(range(16)), w5.logits)


def test_apply_filter_min_p_and_no_filter():
    """min-p alone and no active filter: against the oracle (no golden row has these)."""
    from localstrm_b200.sampling import apply_top_k_top_p_min_p
    rng = np.random.default_rng(3)
    V = 50_000
    x = (rng.standard_normal((4, V)) * 2.0).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    out = apply_top_k_top_p_min_p(xt, min_p=0.05).cpu().numpy()
    for r in range(4):
        res = R.sample_row(x[r], 1.0, min_p=0.05)
        assert np.array_equal(out[r] > -np.inf, res.kept), r
    same = apply_top_k_top_p_min_p(xt).cpu().numpy()
    assert np.array_equal(same, x)


def test_sample_next_token_config1_with_history():
    from localstrm_b200 import SamplingParams, sample_next_token
    w = wl.config1(seed=0)
    rng = np.random.default_rng(5)
    hists = [wl._zipf_ids(rng, 1.2, 512, w.V).tolist() for _ in range(w.B)]
    for r in range(w.B):
        p = SamplingParams(temperature=float(w.temperature[r]), top_k=int(w.top_k[r]),
                           top_p=float(w.top_p[r]), repetition_penalty=1.1,
                           frequency_penalty=0.2 if r % 2 else 0.0, presence_penalty=0.1)
        # The call's first use of the CUDA generator is its uniform: reproduce it.
        torch.cuda.manual_seed(1000 + r)
        u = float(torch.rand(1, device="cuda").item())
        torch.cuda.manual_seed(1000 + r)
        shape = [(1, w.V), (w.V,), (3, w.V)][r % 3]
        x = torch.from_numpy(w.logits[r]).cuda()
        logits = x.reshape(1, -1).expand(*shape).contiguous() if len(shape) == 2 else x.clone()
        tok = sample_next_token(logits, p, past_token_ids=hists[r])
        assert isinstance(tok, int)
        res = R.sample_row(w.logits[r], p.temperature, p.top_k, p.top_p, p.min_p, p.repetition_penalty,
                           p.frequency_penalty, p.presence_penalty, hists[r], u)
        if res.special:
            assert tok == res.token, (r, tok, res.token)
        else:
            assert tok == res.token or P.draw_is_boundary(res.probs, u), (r, tok, res.token, u)
    # The input is not modified (the reference clones first, sampling.py:129).
    x = torch.from_numpy(w.logits[2]).cuda()
    before = x.clone()
    sample_next_token(x, SamplingParams(repetition_penalty=2.0), past_token_ids=[0, 1, 1])
    assert torch.equal(x, before)


def _mixed_params(B, rng):
    from localstrm_b200 import SamplingParams
    out = []
    for r in range(B):
        kind = r % 6
        if kind == 0:
            out.append(SamplingParams.greedy())
        elif kind == 1:
            out.append(SamplingParams())  # the reference's defaults: T 0.7, no filter
        elif kind == 2:
            out.append(SamplingParams(temperature=0.8, top_k=50, top_p=0.9))
        elif kind == 3:
            out.append(SamplingParams(temperature=float(rng.uniform(0.3, 1.3)), min_p=0.05,
                                      repetition_penalty=1.1))
        elif kind == 4:
            out.append(SamplingParams(temperature=1.0, top_k=int(rng.choice([20, 100, 1000])),
                                      top_p=float(rng.uniform(0.5, 1.0)), min_p=0.05,
                                      repetition_penalty=1.1, frequency_penalty=0.3,
                                      presence_penalty=0.2))
        else:
            out.append(SamplingParams(temperature=0.7, top_p=0.95, min_p=0.05,
                                      repetition_penalty=1.3, stop_token_ids=[1, 2]))
    return out


def test_sample_batch_mixed_rows_python_lists():
    from localstrm_b200 import sampling as S
    rng = np.random.default_rng(7)
    B, V = 36, 151_936
    x = (rng.standard_normal((B, V)) * 2.5).astype(np.float32)
    x += rng.uniform(-5, 5, size=(B, 1)).astype(np.float32)
    params = _mixed_params(B, rng)
    hists = []
    for r in range(B):
        n = [0, 1, 37, 512, 2048, 3000][r % 6]
        h = wl._zipf_ids(rng, 1.1, n, V).tolist()
        hists.append(None if r % 12 == 7 else h)
    u = rng.random(B, dtype=np.float32)
    tok, kept, probs = S.sample_batch(torch.from_numpy(x).cuda(), params, hists,
                                      uniforms=torch.from_numpy(u).cuda(), return_kept=True)
    assert tok.dtype == torch.int32 and tok.shape == (B,)
    w = _workload_from_batch("mixed", x, params, hists, u)
    out = dict(tokens=tok.cpu().numpy(), kept=kept.cpu().numpy().astype(bool), probs=probs.cpu().numpy(),
               paths=S._sampler(tok.device).row_paths(B))
    check_workload(w, out)


def test_engine_decode_seam_with_stop_checks():
    """Three decode steps of a 64-request batch through the INTEGRATION.md seam: one
    ``sample_batch`` per step with each request's ``output_token_ids`` as its history, the
    token-id stop check on the device, finished requests dropped before the next step."""
    from localstrm_b200 import sampling as S
    rng = np.random.default_rng(11)
    V = 32_000
    nreq = 64
    params = _mixed_params(nreq, rng)
    outputs = [wl._zipf_ids(rng, 1.2, int(rng.integers(0, 300)), V).tolist() for _ in range(nreq)]
    live = list(range(nreq))
    stopped = 0
    for step in range(3):
        B = len(live)
        x = rng.standard_normal((B, V)).astype(np.float32) * np.float32(3.0)
        xh = torch.from_numpy(x).to(torch.float16)  # the engine's fp16 logits
        x32 = xh.float().numpy()
        u = rng.random(B, dtype=np.float32)
        p = [params[i] for i in live]
        hist = [outputs[i] for i in live]
        w = _workload_from_batch(f"seam{step}", x32, p, hist, u)
        expect = [res.token for res in R.sample_batch(w, want_detail=False)]
        # EOS id and stop ids chosen so that some rows stop on each rule.
        eos = int(expect[0])
        stop_lists = []
        for b, i in enumerate(live):
            extra = [int(expect[b])] if b % 5 == 2 else []
            stop_lists.append(list(p[b].stop_token_ids) + extra)
        tok = S.sample_batch(xh.cuda(), p, hist, uniforms=torch.from_numpy(u).cuda())
        codes = S.check_stop_batch(tok, eos, stop_lists)
        sampled, verdicts = tok.tolist(), S.stop_reasons(codes, tok)  # the step's one read-back
        paths = S._sampler(tok.device).row_paths(B)
        full = R.sample_batch(w, want_detail=True)
        nxt = []
        for b, i in enumerate(live):
            res = full[b]
            t = sampled[b]
            if res.special:
                assert t == res.token, (step, b, t, res.token, int(paths[b]))
            else:
                assert t == res.token or P.draw_is_boundary(res.probs, float(u[b])), (step, b, t, res.token)
            outputs[i].append(t)
            code = R.stop_code(t, eos, stop_lists[b])
            want = {R.STOP_EOS: (True, "eos_token"), R.STOP_TOKEN: (True, f"stop_token_{t}"),
                    R.STOP_NONE: (False, None)}[code]
            assert verdicts[b] == want, (step, b, verdicts[b], want)
            if verdicts[b][0]:
                stopped += 1
            else:
                nxt.append(i)
        live = nxt
    assert stopped > 0 and live
