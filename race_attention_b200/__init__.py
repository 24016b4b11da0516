"""B200-native causal RACE attention (drop-in for sahiljoshi515/RACE_Attention's
``scaling/race_common.py`` + ``scaling/race_causal_cuda.py`` operator surface).

Every operator runs on hand-written sm_100a CUDA in ``librace_b200.so``; there
is no CPU fallback.
"""
from . import ops  # noqa: F401
from .decode import RaceDecodeState, prefill_with_state  # noqa: F401
from .ext import load_ext  # noqa: F401
from .race_causal_cuda import (RaceBTHDFn, RaceCausalCuda, RaceCausalFn, RaceQKVFn, fwd_chunk,  # noqa: F401
                               nanochat_race_attention, race_causal, race_causal_bthd, race_cuda_fused)
from .race_common import build_planes_protos, soft_hash_probs  # noqa: F401
from .noncausal import BatchedACE, RaceNonCausalFn, race_noncausal  # noqa: F401
from .sharded import race_causal_sharded  # noqa: F401

__all__ = [
    "build_planes_protos", "soft_hash_probs", "fwd_chunk", "RaceCausalFn", "race_cuda_fused", "RaceCausalCuda",
    "RaceQKVFn", "race_causal", "race_noncausal", "RaceNonCausalFn", "BatchedACE", "RaceBTHDFn", "race_causal_bthd", "nanochat_race_attention", "RaceDecodeState", "prefill_with_state", "race_causal_sharded", "load_ext", "ops",
]
