"""Loading helpers for the committed golden fixtures (tests/golden/*.npz)."""
from __future__ import annotations

import os

import numpy as np

from oracle.draft_oracle import DraftWeights, bf16_bits_to_f32

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def as_f32(a: np.ndarray) -> np.ndarray:
    """uint16 arrays hold bf16 bit patterns; everything else is already numeric."""
    if a.dtype == np.uint16:
        return bf16_bits_to_f32(a)
    return a.astype(np.float32)


def load(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def weights(fx: dict, dtype: str | None = None) -> DraftWeights:
    if dtype is None:
        dtype = str(fx["dtype"]) if "dtype" in fx else "bf16"
    opt = lambda k: as_f32(fx[k]) if k in fx else None  # noqa: E731
    return DraftWeights(
        fc1=as_f32(fx["fc1"]), fc2=as_f32(fx["fc2"]), w_ih=as_f32(fx["w_ih"]),
        w_hh=as_f32(fx["w_hh"]), embed=as_f32(fx["embed"]), dtype=dtype,
        fc1_bias=opt("fc1_bias"), fc2_bias=opt("fc2_bias"), b_ih=opt("b_ih"), b_hh=opt("b_hh"),
    )


ROLLOUT_CASES = ["rollout_bf16_b1", "rollout_bf16_b3_bias", "rollout_fp32_b1"]
TRACE_CASES = ["spec_trace_random", "spec_trace_full_accept", "spec_trace_partial"]
