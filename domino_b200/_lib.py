"""ctypes binding of libdomino_draft.so (declared in include/domino_draft.h).

The shared library is built in-tree by ``domino_b200.build`` (``nvcc`` for
sm_100a).  There is no fallback: if the library is missing, or the device is
not an sm_100 GPU, the calls below raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdomino_draft.so")

DD_OK = 0
DD_EINVAL = -1
DD_ECUDA = -2
DD_EDEVICE = -3
DD_EUNSUPPORTED = -4
DD_BF16 = 0
DD_FP16 = 1
DD_F32 = 2
DD_STATUS_TIMEOUT = 1
DD_STATUS_BAD_TOKEN = 2
DD_STATUS_NO_ARGMAX = 4
# dd_set_middle kinds (include/domino_draft.h)
DD_MIDDLE_SILU, DD_MIDDLE_IDENTITY, DD_MIDDLE_RELU, DD_MIDDLE_GELU = 0, 1, 2, 3
DD_MIDDLE_GELU_TANH, DD_MIDDLE_TANH, DD_MIDDLE_SIGMOID, DD_MIDDLE_SILU_ROUNDED = 4, 5, 6, 7

EXPORTS = (
    "dd_create", "dd_set_weights", "dd_build_table", "dd_rollout", "dd_draft_block",
    "dd_accept", "dd_get_status", "dd_last_error", "dd_version", "dd_destroy",
    "dd_set_timing", "dd_read_timing", "dd_rollout_noalloc", "dd_noalloc_status",
    "dd_get_exchange_buffer", "dd_ipc_export", "dd_ipc_open", "dd_ipc_close", "dd_set_vocab_shard",
    "dd_set_exchange_timeout", "dd_verify_accept", "dd_set_weight_layout", "dd_set_rollout_mode",
    "dd_set_trace", "dd_set_middle",
)
PHASES = {1: "z", 2: "zlm", 3: "gh", 4: "sgh", 5: "fc2", 6: "table", 7: "cell", 8: "gather", 9: "rollout"}


class DDConfig(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("steps", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("gru_hidden", ctypes.c_int32),
        ("emb_dim", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("prefix_tokens", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class DDWeights(ctypes.Structure):
    _fields_ = [
        ("fc1", ctypes.c_void_p), ("fc1_ld", ctypes.c_int64),
        ("fc1_bias", ctypes.c_void_p),
        ("fc2", ctypes.c_void_p), ("fc2_ld", ctypes.c_int64),
        ("fc2_bias", ctypes.c_void_p),
        ("w_hh", ctypes.c_void_p), ("w_hh_ld", ctypes.c_int64),
        ("b_hh", ctypes.c_void_p),
        ("table", ctypes.c_void_p), ("table_ld", ctypes.c_int64),
        ("lm_head", ctypes.c_void_p), ("lm_head_ld", ctypes.c_int64),
    ]


class DDTrace(ctypes.Structure):
    _fields_ = [("z", ctypes.c_void_p), ("h", ctypes.c_void_p), ("gh", ctypes.c_void_p), ("s", ctypes.c_void_p)]


class DominoDraftError(RuntimeError):
    """A libdomino_draft call returned a negative status."""


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "or `python -m domino_b200.build` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        pp = ctypes.POINTER(ctypes.c_void_p)
        lib.dd_create.argtypes = [ctypes.POINTER(DDConfig), ctypes.c_int, pp]
        lib.dd_set_weights.argtypes = [vp, ctypes.POINTER(DDWeights)]
        lib.dd_build_table.argtypes = [vp, vp, i64, vp, i64, vp, vp, vp]
        lib.dd_rollout.argtypes = [vp, vp, vp, vp, vp, vp]
        lib.dd_rollout_noalloc.argtypes = [ctypes.POINTER(DDConfig), ctypes.POINTER(DDWeights), ctypes.c_int,
                                           vp, vp, vp, vp, vp]
        lib.dd_noalloc_status.argtypes = [ctypes.c_int]
        lib.dd_draft_block.argtypes = [vp, vp, vp, vp, vp, vp]
        lib.dd_accept.argtypes = [vp, vp, i32, i32, vp, vp, vp]
        lib.dd_get_status.argtypes = [vp]
        lib.dd_last_error.argtypes = [vp]
        lib.dd_last_error.restype = ctypes.c_char_p
        lib.dd_version.argtypes = []
        lib.dd_version.restype = ctypes.c_char_p
        lib.dd_destroy.argtypes = [vp]
        lib.dd_set_timing.argtypes = [vp, ctypes.c_int]
        lib.dd_get_exchange_buffer.argtypes = [vp, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_uint64)]
        lib.dd_ipc_export.argtypes = [vp, vp]
        lib.dd_ipc_open.argtypes = [ctypes.c_int, vp, ctypes.POINTER(ctypes.c_void_p)]
        lib.dd_ipc_close.argtypes = [ctypes.c_int, vp]
        lib.dd_set_vocab_shard.argtypes = [vp, i32, i32, i64, i64, ctypes.POINTER(ctypes.c_void_p)]
        lib.dd_set_exchange_timeout.argtypes = [vp, ctypes.c_uint64]
        lib.dd_verify_accept.argtypes = [vp, vp, i32, i32, vp, vp, vp, vp, vp]
        lib.dd_set_weight_layout.argtypes = [vp, ctypes.c_int]
        lib.dd_set_rollout_mode.argtypes = [vp, ctypes.c_int]
        lib.dd_set_trace.argtypes = [vp, ctypes.POINTER(DDTrace)]
        lib.dd_set_middle.argtypes = [vp, ctypes.c_int]
        lib.dd_read_timing.argtypes = [vp, vp, vp, i32]
        for name in EXPORTS:
            if name not in ("dd_last_error", "dd_version"):
                getattr(lib, name).restype = ctypes.c_int
        _lib = lib
        return lib


def check(rc: int, handle=None, what: str = "") -> int:
    """Raise DominoDraftError for a negative return code."""
    if rc < 0:
        lib = load()
        msg = lib.dd_last_error(handle).decode(errors="replace")
        raise DominoDraftError(f"{what or 'libdomino_draft'} failed ({rc}): {msg}")
    return rc
