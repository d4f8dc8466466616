"""Drop-in replacement for LocalStrm's sampler (``src/engine/sampling.py``) on B200.

Same names, arguments and defaults as the reference:

* ``SamplingParams``                                   (``sampling.py:20-35``)
* ``sample_next_token(logits, params, past_token_ids)``  (``sampling.py:118-163``)
* ``apply_top_k_top_p_min_p(logits, top_k, top_p, min_p)`` (``sampling.py:71-115``)

plus the batched seam the engine loop needs (``llm_engine.py:1129-1153``):
``sample_batch`` / ``BatchSampler`` (one ``[B, V]`` call instead of B row calls) and
``greedy_batch`` (the all-greedy ``argmax``).  Everything runs in the native library
``_lib/liblss.so`` on the logits' CUDA device; a CPU tensor or a missing library raises.

Parity contract: inputs of any dtype are widened to float32 on load (the reference is
compared on ``logits.float()``).  The draw is an inverse CDF in vocabulary order driven by
one uniform per row; ``sample_next_token`` draws that uniform from torch's CUDA generator,
``sample_batch`` accepts caller-supplied uniforms.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from . import _lib

__all__ = ["SamplingParams", "sample_next_token", "sample_batch", "greedy_batch",
           "apply_top_k_top_p_min_p", "BatchSampler", "RowParams", "SamplerError"]

SamplerError = _lib.SamplerError
_DT = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


@dataclass
class SamplingParams:
    """Per-request sampling knobs, field for field as the reference's ``SamplingParams``."""
    temperature: float = 0.7
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    stop_token_ids: List[int] = field(default_factory=list)
    stop_strings: List[str] = field(default_factory=list)

    @classmethod
    def greedy(cls) -> "SamplingParams":
        return cls(temperature=0.0)


@dataclass
class RowParams:
    """Structure-of-arrays per-row parameters as device tensors (the C ABI's layout)."""
    temperature: torch.Tensor
    top_k: torch.Tensor
    top_p: torch.Tensor
    min_p: torch.Tensor
    repetition_penalty: torch.Tensor
    frequency_penalty: torch.Tensor
    presence_penalty: torch.Tensor

    @classmethod
    def from_params(cls, params: Sequence[SamplingParams], device) -> "RowParams":
        f = lambda name: torch.tensor([float(getattr(p, name)) for p in params], dtype=torch.float32)
        host = dict(temperature=f("temperature"),
                    top_k=torch.tensor([_clamp_k(p.top_k) for p in params], dtype=torch.int32),
                    top_p=f("top_p"), min_p=f("min_p"), repetition_penalty=f("repetition_penalty"),
                    frequency_penalty=f("frequency_penalty"), presence_penalty=f("presence_penalty"))
        return cls(**{k: v.to(device, non_blocking=True) for k, v in host.items()})

    @classmethod
    def from_arrays(cls, device, **arrays) -> "RowParams":
        conv = {}
        for k in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
                  "frequency_penalty", "presence_penalty"):
            dt = torch.int32 if k == "top_k" else torch.float32
            conv[k] = torch.as_tensor(np.asarray(arrays[k]), dtype=dt).to(device)
        return cls(**conv)

    def check(self, B: int, device) -> None:
        for k, v in self.__dict__.items():
            want = torch.int32 if k == "top_k" else torch.float32
            if v.dtype != want or v.numel() != B or v.device != device or not v.is_contiguous():
                raise ValueError(f"row parameter {k}: expected contiguous {want} [{B}] on {device}")


def _clamp_k(k) -> int:
    k = int(k)
    return max(min(k, 2 ** 31 - 1), -(2 ** 31))


def build_history_csr(histories: Optional[Sequence[Optional[Sequence[int]]]], B: int, V: int):
    """CSR (offsets[B+1], ids) int32 host arrays from per-row id lists.

    Ids follow torch indexing as the reference applies it (``logits[..., ids]``,
    ``sampling.py:56``): values in [-V, V) are accepted and negatives count from the end;
    anything else raises IndexError.
    """
    offs = np.zeros(B + 1, dtype=np.int64)
    chunks = []
    if histories is not None:
        if len(histories) != B:
            raise ValueError(f"expected {B} histories, got {len(histories)}")
        for r, h in enumerate(histories):
            a = np.asarray(h if h is not None else [], dtype=np.int64).reshape(-1)
            if a.size:
                if a.min() < -V or a.max() >= V:
                    bad = a[(a < -V) | (a >= V)][0]
                    raise IndexError(f"history id {int(bad)} out of range for vocabulary {V}")
                a = np.where(a < 0, a + V, a)
            chunks.append(a)
            offs[r + 1] = offs[r] + a.size
    if offs[-1] >= 2 ** 31:
        raise ValueError("total history length must stay below 2**31")
    ids = np.concatenate(chunks).astype(np.int32) if chunks and offs[-1] else np.zeros(0, np.int32)
    return offs.astype(np.int32), ids


class BatchSampler:
    """Reusable device state for batched sampling on one CUDA device.

    Holds the workspace (grown on demand) so that steady-state calls allocate nothing
    but their outputs; every call is stream-ordered on torch's current stream.
    """

    def __init__(self, device: Union[int, str, torch.device, None] = None):
        self.lib = _lib.load()
        dev = torch.device("cuda") if device is None else torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("BatchSampler needs a CUDA device (there is no CPU path)")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self._ws = None
        self._ws_bytes = 0
        self._last_ws = None

    def workspace(self, B: int, V: int, hist_total: int) -> torch.Tensor:
        need = int(self.lib.lss_workspace_bytes(B, V, hist_total))
        if self._ws is None or self._ws_bytes < need:
            self._ws = torch.empty(need + 256, dtype=torch.uint8, device=self.device)
            self._ws_bytes = need
        base = self._ws.data_ptr()
        off = (-base) % 256
        self._last_ws = self._ws[off:off + need]
        return self._last_ws

    def sample(self, logits: torch.Tensor, params: RowParams, hist_offsets: Optional[torch.Tensor],
               hist_ids: Optional[torch.Tensor], uniforms: torch.Tensor,
               tokens_out: Optional[torch.Tensor] = None, kept_out: Optional[torch.Tensor] = None,
               probs_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One token per row of ``logits [B, V]`` (all tensors already on this device)."""
        if logits.device != self.device:
            raise ValueError(f"logits on {logits.device}, sampler on {self.device}")
        if logits.dim() != 2:
            raise ValueError("logits must be [B, V]")
        if logits.dtype not in _DT:
            raise TypeError(f"unsupported logits dtype {logits.dtype}")
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        B, V = logits.shape
        params.check(B, self.device)
        if uniforms.dtype != torch.float32 or uniforms.numel() != B or uniforms.device != self.device:
            raise ValueError(f"uniforms: expected float32 [{B}] on {self.device}")
        hist_total = 0
        if hist_ids is not None and hist_ids.numel() > 0:
            hist_total = int(hist_ids.numel())
            # The library reads these as int32 device arrays: an int64 CSR would be read as
            # pairs of int32 words.  Offsets' values are checked on the device (a bad row sets
            # LSS_FLAG_BAD_HISTORY and its history is ignored).
            for name, t, n in (("hist_offsets", hist_offsets, B + 1), ("hist_ids", hist_ids, hist_total)):
                if t is None or t.dtype != torch.int32 or t.numel() != n or t.device != self.device \
                        or not t.is_contiguous():
                    raise ValueError(f"{name}: expected a contiguous int32 tensor of {n} entries on {self.device}")
        if tokens_out is None:
            tokens_out = torch.empty(B, dtype=torch.int32, device=self.device)
        ws = self.workspace(B, V, hist_total)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        ptr = lambda t: t.data_ptr() if t is not None else None
        st = self.lib.lss_sample(
            logits.data_ptr(), _lib.DTYPES[_DT[logits.dtype]], B, V, logits.stride(0),
            ptr(params.temperature), ptr(params.top_k), ptr(params.top_p), ptr(params.min_p),
            ptr(params.repetition_penalty), ptr(params.frequency_penalty),
            ptr(params.presence_penalty),
            ptr(hist_offsets) if hist_total else None, ptr(hist_ids) if hist_total else None,
            hist_total, uniforms.data_ptr(), tokens_out.data_ptr(), ptr(kept_out), ptr(probs_out),
            ws.data_ptr(), ws.numel(), stream)
        _lib.check("lss_sample", st)
        return tokens_out

    def row_paths(self, B: int) -> np.ndarray:
        """Path codes of the last call (synchronises the stream)."""
        if self._last_ws is None:
            raise RuntimeError("no call has been made on this sampler yet")
        out = np.zeros(B, dtype=np.int32)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check("lss_read_row_paths", self.lib.lss_read_row_paths(
            self._last_ws.data_ptr(), B, out.ctypes.data_as(ctypes.c_void_p), stream))
        return out

    def status(self) -> int:
        """Device error flags of the last call (synchronises the stream)."""
        if self._last_ws is None:
            raise RuntimeError("no call has been made on this sampler yet")
        f = ctypes.c_uint32(0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.lib.lss_read_status(self._last_ws.data_ptr(), ctypes.byref(f), stream)
        return int(f.value)

    def argmax(self, logits: torch.Tensor, tokens_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if logits.dim() != 2 or logits.dtype not in _DT or logits.device != self.device:
            raise ValueError("argmax: expected [B, V] f32/bf16/f16 logits on the sampler's device")
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        B, V = logits.shape
        if tokens_out is None:
            tokens_out = torch.empty(B, dtype=torch.int32, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check("lss_argmax", self.lib.lss_argmax(logits.data_ptr(), _lib.DTYPES[_DT[logits.dtype]],
                                                     B, V, logits.stride(0), tokens_out.data_ptr(),
                                                     stream))
        return tokens_out


_SAMPLERS = {}


def _sampler(device: torch.device) -> BatchSampler:
    key = (device.type, device.index)
    s = _SAMPLERS.get(key)
    if s is None:
        s = _SAMPLERS[key] = BatchSampler(device)
    return s


def _require_cuda(logits: torch.Tensor) -> None:
    if not isinstance(logits, torch.Tensor) or not logits.is_cuda:
        raise RuntimeError("localstrm_b200 samples on CUDA tensors only (no CPU fallback)")


def sample_batch(logits: torch.Tensor, params: Union[Sequence[SamplingParams], RowParams],
                 past_token_ids: Optional[Sequence[Optional[Sequence[int]]]] = None,
                 uniforms: Optional[torch.Tensor] = None, return_kept: bool = False):
    """Tokens for every row of ``logits [B, V]`` in one native call (int32 CUDA tensor)."""
    _require_cuda(logits)
    if logits.dim() != 2:
        raise ValueError("logits must be [B, V]")
    B, V = logits.shape
    dev = logits.device
    s = _sampler(dev)
    rp = params if isinstance(params, RowParams) else RowParams.from_params(list(params), dev)
    offs, ids = build_history_csr(past_token_ids, B, V)
    h_off = torch.from_numpy(offs).to(dev, non_blocking=True) if ids.size else None
    h_ids = torch.from_numpy(ids).to(dev, non_blocking=True) if ids.size else None
    if uniforms is None:
        uniforms = torch.rand(B, device=dev, dtype=torch.float32)
    kept = probs = None
    if return_kept:
        kept = torch.empty((B, V), dtype=torch.uint8, device=dev)
        probs = torch.empty((B, V), dtype=torch.float32, device=dev)
    tok = s.sample(logits, rp, h_off, h_ids, uniforms.to(dev, torch.float32), kept_out=kept,
                   probs_out=probs)
    return (tok, kept, probs) if return_kept else tok


def greedy_batch(logits: torch.Tensor) -> torch.Tensor:
    """``torch.argmax(logits, dim=-1)`` for a CUDA ``[B, V]`` batch (int32 result)."""
    _require_cuda(logits)
    return _sampler(logits.device).argmax(logits)


def sample_next_token(logits: torch.Tensor, params: SamplingParams,
                      past_token_ids: Optional[List[int]] = None) -> int:
    """Selects the next token for the last row of ``logits`` (``[V]`` or ``[..., V]``)."""
    _require_cuda(logits)
    row = logits[-1] if logits.ndim > 1 else logits
    row = row.reshape(1, -1)
    hist = [past_token_ids] if past_token_ids else None
    tok = sample_batch(row, [params], hist)
    return int(tok.item())


STOP_NONE, STOP_EOS, STOP_TOKEN = 0, 1, 2


def check_stop_batch(tokens: torch.Tensor, eos_token_id=None,
                     stop_token_ids: Optional[Sequence] = None) -> torch.Tensor:
    """Token-id part of ``check_stop_criteria`` (``sampling.py:182-185``) for a CUDA batch of
    freshly sampled ids, on the device: an int32 code per row, ``STOP_EOS`` when the token is
    the row's EOS id, else ``STOP_TOKEN`` when it is one of the row's stop ids, else
    ``STOP_NONE``.

    ``eos_token_id``: one id for every row, a per-row sequence (``None`` or a negative id: no
    EOS id), or ``None``.  ``stop_token_ids``: one list for every row or one list per row.
    The stop-string part (``sampling.py:188-194``) needs the tokenizer and stays on the host.
    """
    if not isinstance(tokens, torch.Tensor) or not tokens.is_cuda or tokens.dim() != 1:
        raise ValueError("tokens must be a 1-D CUDA tensor")
    dev = tokens.device
    tok = tokens.to(torch.int32).contiguous()
    B = tok.numel()
    out = torch.empty(B, dtype=torch.int32, device=dev)
    eos = None
    if eos_token_id is not None:
        if isinstance(eos_token_id, (int, np.integer)):
            e = np.full(B, int(eos_token_id), dtype=np.int32)
        else:
            vals = list(eos_token_id)
            if len(vals) != B:
                raise ValueError(f"expected {B} EOS ids, got {len(vals)}")
            e = np.array([-1 if v is None else int(v) for v in vals], dtype=np.int32)
        eos = torch.from_numpy(e).to(dev)
    offs = ids = None
    if stop_token_ids is not None:
        lists = list(stop_token_ids)
        if lists and not isinstance(lists[0], (list, tuple, np.ndarray)):
            lists = [lists] * B  # one list for every row
        if len(lists) != B:
            raise ValueError(f"expected {B} stop-id lists, got {len(lists)}")
        o = np.zeros(B + 1, dtype=np.int32)
        for r, l in enumerate(lists):
            o[r + 1] = o[r] + len(l)
        flat = np.array([int(i) for l in lists for i in l], dtype=np.int32)
        offs = torch.from_numpy(o).to(dev)
        ids = torch.from_numpy(flat if flat.size else np.zeros(1, np.int32)).to(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    P = lambda t: t.data_ptr() if t is not None else None
    _lib.check("lss_stop_check", lib.lss_stop_check(tok.data_ptr(), B, P(eos), P(offs), P(ids),
                                                    out.data_ptr(), stream))
    return out


def stop_reasons(codes, tokens) -> List[Tuple[bool, Optional[str]]]:
    """The reference's ``(should_stop, reason)`` per row (``sampling.py:182-185``) from the
    codes of ``check_stop_batch``; rows with ``STOP_NONE`` still owe the host stop-string
    check."""
    c = codes.tolist() if isinstance(codes, torch.Tensor) else list(codes)
    t = tokens.tolist() if isinstance(tokens, torch.Tensor) else list(tokens)
    out = []
    for code, tk in zip(c, t):
        if code == STOP_EOS:
            out.append((True, "eos_token"))
        elif code == STOP_TOKEN:
            out.append((True, f"stop_token_{tk}"))
        else:
            out.append((False, None))
    return out


def apply_top_k_top_p_min_p(logits: torch.Tensor, top_k: int = -1, top_p: float = 1.0,
                            min_p: float = 0.0, min_tokens_to_keep: int = 1) -> torch.Tensor:
    """The reference's filter (``sampling.py:71-115``): non-surviving entries set to -inf.

    Runs the native kernel with temperature 1 and no penalties on each row of ``logits``
    (``[V]`` or ``[B, V]``) and masks with its kept set; ``min_tokens_to_keep`` must be 1,
    the only value the reference's sampler uses.
    """
    _require_cuda(logits)
    if min_tokens_to_keep != 1:
        raise NotImplementedError("min_tokens_to_keep != 1 is not supported")
    x = logits.reshape(1, -1) if logits.ndim == 1 else logits.reshape(-1, logits.shape[-1])
    B = x.shape[0]
    prm = [SamplingParams(temperature=1.0, top_k=top_k, top_p=top_p, min_p=min_p)] * B
    _, kept, _ = sample_batch(x, prm, None, torch.zeros(B, device=x.device), return_kept=True)
    out = x.float().masked_fill(kept == 0, float("-inf")).to(logits.dtype)
    return out.reshape(logits.shape)
