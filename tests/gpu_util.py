"""Helpers that run a ``Workload`` through the native sampler (C ABI via ctypes)."""
from __future__ import annotations

import numpy as np
import torch

from localstrm_b200.sampling import BatchSampler, RowParams

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def device_inputs(w, device="cuda", dtype=None, row_stride=None):
    dt = TORCH_DT[dtype or w.dtype]
    x = torch.from_numpy(w.logits)
    if row_stride is not None and row_stride != w.V:
        buf = torch.full((w.B, row_stride), float("nan"), dtype=torch.float32)
        buf[:, :w.V] = x
        logits = buf.to(dt).to(device)[:, :w.V]
    else:
        logits = x.to(dt).to(device)
    prm = RowParams.from_arrays(device, temperature=w.temperature, top_k=w.top_k, top_p=w.top_p,
                                min_p=w.min_p, repetition_penalty=w.repetition_penalty,
                                frequency_penalty=w.frequency_penalty,
                                presence_penalty=w.presence_penalty)
    if w.hist_ids.size:
        h_off = torch.from_numpy(w.hist_offsets.astype(np.int32)).to(device)
        h_ids = torch.from_numpy(w.hist_ids.astype(np.int32)).to(device)
    else:
        h_off = h_ids = None
    u = torch.from_numpy(w.uniforms.astype(np.float32)).to(device)
    return logits, prm, h_off, h_ids, u


def run(w, sampler: BatchSampler = None, detail=True, dtype=None, row_stride=None):
    """Tokens (and kept / probs when ``detail``) for every row, plus the per-row path codes."""
    s = sampler or BatchSampler("cuda")
    logits, prm, h_off, h_ids, u = device_inputs(w, s.device, dtype, row_stride)
    kept = probs = None
    if detail:
        kept = torch.empty((w.B, w.V), dtype=torch.uint8, device=s.device)
        probs = torch.empty((w.B, w.V), dtype=torch.float32, device=s.device)
    tok = s.sample(logits, prm, h_off, h_ids, u, kept_out=kept, probs_out=probs)
    torch.cuda.synchronize()
    paths = s.row_paths(w.B)
    flags = s.status()
    out = dict(tokens=tok.cpu().numpy(), paths=paths, flags=flags)
    if detail:
        out["kept"] = kept.cpu().numpy().astype(bool)
        out["probs"] = probs.cpu().numpy()
    return out
