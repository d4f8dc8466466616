"""Generate the stop-check golden cases from LocalStrm's own ``check_stop_criteria``.

Usage:  python tests/golden/make_stop_golden.py /path/to/localstrm

Seeded cases (last token, EOS id or None, stop-id list) are run through the reference's
``check_stop_criteria`` (``src/engine/sampling.py:166-196``) with a stand-in tokenizer that
only carries ``eos_token_id`` and no stop strings, so only its token-id part
(``:182-185``) decides.  The result is stored as a code (0 none, 1 EOS, 2 stop id) next to the
inputs in ``stop_check.npz``.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class _Tok:
    def __init__(self, eos):
        self.eos_token_id = eos

    def decode(self, ids, skip_special_tokens=False):  # not reached without stop strings
        return ""


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from src.engine.sampling import check_stop_criteria
    rng = np.random.default_rng(2026)
    n = 512
    tokens = rng.integers(0, 64, size=n).astype(np.int32)
    eos = rng.integers(-1, 64, size=n).astype(np.int32)  # -1: the tokenizer has no EOS id
    offs = np.zeros(n + 1, np.int32)
    lists = []
    for i in range(n):
        k = int(rng.integers(0, 6))
        l = rng.integers(0, 64, size=k).astype(np.int32)
        if i % 7 == 0 and k:
            l[0] = tokens[i]  # make the stop id hit
        if i % 11 == 0:
            eos[i] = tokens[i]  # make the EOS id hit (also when a stop id hits)
        lists.append(l)
        offs[i + 1] = offs[i] + k
    ids = np.concatenate(lists).astype(np.int32)
    codes = np.zeros(n, np.int32)
    for i in range(n):
        stop, reason = check_stop_criteria([int(tokens[i])], _Tok(None if eos[i] < 0 else int(eos[i])),
                                           [int(v) for v in lists[i]], [])
        codes[i] = 0 if not stop else (1 if reason == "eos_token" else 2)
        if stop and reason not in ("eos_token", f"stop_token_{int(tokens[i])}"):
            raise AssertionError(reason)
    np.savez_compressed(os.path.join(HERE, "stop_check.npz"), tokens=tokens, eos=eos, offsets=offs,
                        ids=ids, codes=codes)
    print("stop_check.npz:", n, "cases,", int((codes == 1).sum()), "EOS,", int((codes == 2).sum()), "stop id")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_stop_golden.py /path/to/localstrm")
    main(sys.argv[1])
