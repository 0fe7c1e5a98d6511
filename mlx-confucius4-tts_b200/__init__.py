"""c4s -- B200-native T2S sampling stage for Confucius4-TTS (host side).

The package directory is `mlx-confucius4-tts_b200/`; it is imported under the
name `c4s`. CUDA kernels and the C ABI live in csrc/ (built into
lib/libc4s.so); this module is the Python mirror of the reference's
c4::t2s::sampling interface on top of that ABI.
"""
from . import decode, sharding, vocab_shard, workloads  # noqa: F401
from .sampling import (  # noqa: F401
    C4SError, SamplingContext, argmax, default_context, library, params_tensor,
    repetition_penalty, temperature, top_k, top_p, STAGE_ALL, STAGE_PENALTY,
    STAGE_TEMPERATURE, STAGE_TOP_K, STAGE_TOP_P, DEBUG_FORCE_BINS, DEBUG_FORCE_EXACT,
)
