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


LOOP_CASES = ["spec_loop_random", "spec_loop_varied", "spec_loop_full"]


def load_loop(name: str, device="cpu"):
    """A spec_generate fixture (tests/golden/make_golden.py spec_loop_case):
    the tiny target and drafter with the reference's weights, the prompts, and
    the reference's output ids and acceptance lengths per prompt."""
    import json

    import torch

    from domino_b200.stack import DFlashBackbone, StackConfig, TargetLM

    fx = load(name)
    tcfg = StackConfig(**json.loads(str(fx["target_config"])))
    dcfg = StackConfig(**json.loads(str(fx["draft_config"])))
    target, draft = TargetLM(tcfg), DFlashBackbone(dcfg)
    target.load_state_dict({k[2:]: torch.from_numpy(v) for k, v in fx.items() if k.startswith("t.")}, strict=True)
    draft.load_state_dict({k[2:]: torch.from_numpy(v) for k, v in fx.items() if k.startswith("d.")}, strict=True)
    n = int(fx["n_prompts"])
    return dict(
        target=target.to(device).eval(), draft=draft.to(device).eval(), fx=fx,
        prompts=[torch.from_numpy(fx[f"prompt_{i}"]) for i in range(n)],
        outputs=[fx[f"output_{i}"] for i in range(n)],
        accepts=[fx[f"accept_{i}"].tolist() for i in range(n)],
        max_new_tokens=int(fx["max_new_tokens"]),
    )
