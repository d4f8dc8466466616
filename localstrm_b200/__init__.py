"""B200-native (sm_100a) batched token sampler with LocalStrm's sampling semantics.

The hot path is one native library (``_lib/liblss.so``, built from ``csrc/``) behind the
C ABI in ``include/lsampler.h``; ``sampling`` is the drop-in for the reference's
``src/engine/sampling.py`` and ``distributed`` holds the row- and vocabulary-sharded modes.
"""
from .sampling import (BatchSampler, RowParams, SamplerError, SamplingParams,  # noqa: F401
                       STOP_EOS, STOP_NONE, STOP_TOKEN, apply_top_k_top_p_min_p, check_stop_batch,
                       greedy_batch, sample_batch, sample_next_token, stop_reasons)

__version__ = "0.1.0"
