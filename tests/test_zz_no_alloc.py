"""The allocation-free entry point against the regular one, through the C ABI.

``lss_sample_noalloc`` serves callers that must not allocate device memory mid-decode (an
engine that reserved the GPU for its KV cache up front); it runs on one fixed device array
inside the library instead of a caller workspace.  Two calls in a row must give exactly the
tokens, kept sets and probabilities of ``lss_sample`` on the same inputs, the second call
with different inputs so that anything left over from the first would show.

Named so that pytest collects it last.
"""
import numpy as np
import pytest
import torch

from localstrm_b200 import _lib
from localstrm_b200 import workloads as wl
from localstrm_b200.sampling import BatchSampler
from tests import gpu_util as G

pytestmark = pytest.mark.gpu


def _call(lib, fn, w, inputs, ws=None):
    logits, prm, h_off, h_ids, u = inputs
    B, V = w.B, w.V
    tok = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    kept = torch.empty((B, V), dtype=torch.uint8, device="cuda")
    probs = torch.empty((B, V), dtype=torch.float32, device="cuda")
    H = 0 if h_ids is None else int(h_ids.numel())
    P = lambda t: None if t is None else t.data_ptr()
    args = [P(logits), _lib.DTYPES[w.dtype], B, V, logits.stride(0), P(prm.temperature),
            P(prm.top_k), P(prm.top_p), P(prm.min_p), P(prm.repetition_penalty),
            P(prm.frequency_penalty), P(prm.presence_penalty), P(h_off), P(h_ids), H, P(u),
            P(tok), P(kept), P(probs)]
    stream = torch.cuda.current_stream().cuda_stream
    if fn == "lss_sample":
        st = lib.lss_sample(*args, P(ws), ws.numel(), stream)
    else:
        st = lib.lss_sample_noalloc(*args, stream)
    assert st == 0, _lib.status_string(st)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), kept.cpu().numpy(), probs.cpu().numpy()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_noalloc_matches_workspace_entry_point_twice():
    lib = _lib.load()
    s = BatchSampler("cuda")
    first = wl.config3(seed=21, B=48, V=50_000, H=512)
    second = wl.config2(seed=22, B=40, V=60_000, H=300)   # bf16, other params and shapes
    for w in (first, second):
        inputs = G.device_inputs(w)
        ws = s.workspace(w.B, w.V, int(w.hist_ids.size))
        ref = _call(lib, "lss_sample", w, inputs, ws)
        got = _call(lib, "lss_sample_noalloc", w, inputs)
        assert np.array_equal(got[0], ref[0]), (w.name, np.nonzero(got[0] != ref[0]))
        assert np.array_equal(got[1], ref[1]), w.name
        assert np.array_equal(got[2], ref[2]), w.name
        assert (got[0] >= 0).all() and (got[0] < w.V).all()
        # The device status of the call (error flags in the fixed scratch) reads clean.
        import ctypes
        flags = ctypes.c_uint32(0xdead)
        st = lib.lss_noalloc_read_status(ctypes.byref(flags), torch.cuda.current_stream().cuda_stream)
        assert st == 0 and flags.value == 0, (w.name, st, flags.value)
