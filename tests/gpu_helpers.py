"""Helpers shared by the GPU parity tests: module construction in the
reference's layout, oracle weights, and the teacher-forced token check."""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn as nn

from oracle import draft_oracle as O
from tests.fixtures import as_f32

TOL = 2e-2  # atol = rtol: bf16 logits/states, and the top-2 gap below which an argmax may differ

# One line per parity check, printed at the end of the run (tests/conftest.py).
PARITY_LOG: list = []


def _test_name() -> str:
    name = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    return name.split("::", 1)[-1]


def log_parity(text: str) -> None:
    PARITY_LOG.append(f"{_test_name()}: {text}")


def compare_states(label, got, ref, tol=TOL):
    """Assert ``|got - ref| <= tol + tol * |ref|`` elementwise (bf16 states and
    logits) and return (max abs difference, fraction of bit-identical values)."""
    g = got.float() if torch.is_tensor(got) else torch.from_numpy(np.asarray(got, np.float32))
    r = ref.float() if torch.is_tensor(ref) else torch.from_numpy(np.asarray(ref, np.float32))
    g = g.to(r.device)
    assert g.shape == r.shape, (label, tuple(g.shape), tuple(r.shape))
    if g.numel() == 0:
        return 0.0, 1.0
    diff = (g - r).abs()
    bad = diff > tol + tol * r.abs()
    assert not bool(bad.any()), (
        f"{label}: {int(bad.sum())} of {bad.numel()} values beyond atol=rtol={tol}; "
        f"max |diff| {float(diff.max()):.4g} at {np.unravel_index(int(diff.argmax()), tuple(diff.shape))}")
    return float(diff.max()), float((g == r).float().mean())


class DraftHead(nn.Module):
    """The two head modules the runner reads (code/dflash.py:261-274)."""

    def __init__(self, H, G, E, V, fc1_bias=False, fc2_bias=False, gru_bias=False):
        super().__init__()
        self.prefix_gru = nn.GRU(H, G, num_layers=1, batch_first=True, bias=gru_bias)
        self.embed_proj = nn.Sequential(nn.Linear(H + G, E, bias=fc1_bias), nn.SiLU(),
                                        nn.Linear(E, V, bias=fc2_bias))


class Target(nn.Module):
    def __init__(self, H, V):
        super().__init__()
        self.model = nn.Module()
        self.model.embed_tokens = nn.Embedding(V, H)
        self.lm_head = nn.Linear(H, V, bias=False)


def random_modules(H, G, E, V, *, seed=0, dtype=torch.bfloat16, device="cuda", fc2_std=0.05,
                   fc1_bias=False, fc2_bias=False, gru_bias=False):
    g = torch.Generator(device="cpu").manual_seed(seed)
    draft = DraftHead(H, G, E, V, fc1_bias, fc2_bias, gru_bias)
    target = Target(H, V)
    with torch.no_grad():
        for name, p in list(draft.named_parameters()) + list(target.named_parameters()):
            std = 0.02 if p.dim() == 2 else 0.05
            if name.startswith("embed_proj.2"):
                std = fc2_std
            p.copy_(torch.randn(p.shape, generator=g) * std)
        target.model.embed_tokens.weight.copy_(torch.randn(V, H, generator=g))
    return draft.to(device=device, dtype=dtype).eval(), target.to(device=device, dtype=dtype).eval()


MIDDLES = {"gelu": nn.GELU, "relu": nn.ReLU, "tanh": nn.Tanh}


def modules_from_fixture(fx, device="cuda"):
    B, H, G, E, V, S, P, fb1, fb2, gb = (int(x) for x in fx["meta"])
    draft = DraftHead(H, G, E, V, bool(fb1), bool(fb2), bool(gb))
    middle = str(fx["middle"]) if "middle" in fx else "silu"
    if middle == "identity":
        draft.embed_proj = nn.Sequential(draft.embed_proj[0], draft.embed_proj[2])
    elif middle != "silu":
        draft.embed_proj[1] = MIDDLES[middle]()
    target = Target(H, V)
    with torch.no_grad():
        draft.embed_proj[0].weight.copy_(torch.from_numpy(as_f32(fx["fc1"])))
        draft.embed_proj[-1].weight.copy_(torch.from_numpy(as_f32(fx["fc2"])))
        draft.prefix_gru.weight_ih_l0.copy_(torch.from_numpy(as_f32(fx["w_ih"])))
        draft.prefix_gru.weight_hh_l0.copy_(torch.from_numpy(as_f32(fx["w_hh"])))
        target.model.embed_tokens.weight.copy_(torch.from_numpy(as_f32(fx["embed"])))
        target.lm_head.weight.copy_(torch.from_numpy(as_f32(fx["lm_head"])))
        if fb1:
            draft.embed_proj[0].bias.copy_(torch.from_numpy(as_f32(fx["fc1_bias"])))
        if fb2:
            draft.embed_proj[-1].bias.copy_(torch.from_numpy(as_f32(fx["fc2_bias"])))
        if gb:
            draft.prefix_gru.bias_ih_l0.copy_(torch.from_numpy(as_f32(fx["b_ih"])))
            draft.prefix_gru.bias_hh_l0.copy_(torch.from_numpy(as_f32(fx["b_hh"])))
    dt = torch.bfloat16
    return draft.to(device=device, dtype=dt).eval(), target.to(device=device, dtype=dt).eval()


def _f32(t):
    return None if t is None else t.detach().float().cpu().numpy()


def oracle_weights(draft, target, dtype="bf16") -> O.DraftWeights:
    fc1, fc2 = draft.embed_proj[0], draft.embed_proj[2]
    gru = draft.prefix_gru
    return O.DraftWeights(
        fc1=_f32(fc1.weight), fc2=_f32(fc2.weight), w_ih=_f32(gru.weight_ih_l0), w_hh=_f32(gru.weight_hh_l0),
        embed=_f32(target.model.embed_tokens.weight), dtype=dtype,
        fc1_bias=_f32(fc1.bias), fc2_bias=_f32(fc2.bias),
        b_ih=_f32(getattr(gru, "bias_ih_l0", None)) if gru.bias else None,
        b_hh=_f32(getattr(gru, "bias_hh_l0", None)) if gru.bias else None,
    )


def random_inputs(B, S, H, V, P, target, *, seed=0, device="cuda", dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed + 1000)
    prefix = torch.randint(0, V, (B, P), generator=g).to(device)
    ph = torch.randn(B, S, H, generator=g).to(device=device, dtype=dtype)
    with torch.no_grad():
        base = target.lm_head(ph)
    return prefix, ph, base


def teacher_forced_check(w: O.DraftWeights, prefix, ph, base, gpu_tokens, min_exact=1.0):
    """Every GPU token equals the oracle's argmax given the same history, or is
    within TOL of the oracle's top logit (a near-tie).  Returns the exact-match
    fraction; asserts it is at least ``min_exact``."""
    tok = gpu_tokens.cpu().numpy() if torch.is_tensor(gpu_tokens) else np.asarray(gpu_tokens)
    tr = O.rollout(w, _np(prefix), _np(ph), _np(base), teacher_tokens=tok)
    exact = tr.tokens == tok
    slack = tr.max_logit - tr.chosen_logit
    bad = (~exact) & (slack > TOL + TOL * np.abs(tr.max_logit))
    assert not bad.any(), (
        f"tokens differ beyond the near-tie tolerance at {np.argwhere(bad).tolist()}: "
        f"gpu {tok[bad]}, oracle {tr.tokens[bad]}, slack {slack[bad]}"
    )
    frac = float(exact.mean())
    worst = float(slack[~exact].max()) if (~exact).any() else 0.0
    log_parity(f"tokens {int(exact.sum())}/{exact.size} exact ({frac:.3f}), worst near-tie slack {worst:.3g}")
    assert frac >= min_exact, f"only {frac:.3f} of the tokens are exact"
    return frac, tr


def _np(x):
    if torch.is_tensor(x):
        if x.dtype in (torch.bfloat16, torch.float16):
            return x.float().cpu().numpy()
        return x.cpu().numpy()
    return np.asarray(x)
