"""B200-native (sm_100a) draft step of Domino speculative decoding.

``DraftCorrectionGraphRunner`` is a drop-in for the reference runner of the
same name (code/kernel/domino.py:229-508); the compute runs in the
hand-written CUDA kernels of ``libdomino_draft.so`` (C ABI:
include/domino_draft.h), loaded through ``domino_b200._lib``.
"""
from .runner import DominoDraftError, DraftCorrectionGraphRunner, unwrap_correction_mlp

__all__ = ["DraftCorrectionGraphRunner", "DominoDraftError", "unwrap_correction_mlp"]
__version__ = "0.1.0"
