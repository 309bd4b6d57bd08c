"""Per-step state parity of the sm_100a rollout (through the C ABI's state
trace, ``dd_set_trace`` / ``runner.rollout_trace``).

The states are the ones code/kernel/domino.py:381-431 computes: the z
projection, the GRU state after every prefix token and every draft step, the
``h W_hh^T + b_hh`` fed to each GRU step and the s projection of every draft
step.  Each is compared, at atol = rtol = 2e-2, with

* the reference's own recorded values (tests/golden/rollout_*.npz, written by
  running the reference runner with its Triton kernels), for every step up
  to the first step at which a row's token differs from the reference's; and
* the oracle fed the GPU's tokens (teacher forcing), for every step.

Tokens: every token equals the oracle's argmax given the same history, or
is a near-tie within 2e-2.
"""
import numpy as np
import pytest
import torch

from oracle import draft_oracle as O
from tests.fixtures import ROLLOUT_CASES, as_f32, load
from tests.gpu_helpers import (
    compare_states, log_parity, modules_from_fixture, oracle_weights, random_inputs, random_modules,
    teacher_forced_check,
)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


def make_runner(draft, target, B, S, H, G, V, P, **kw):
    from domino_b200 import DraftCorrectionGraphRunner
    return DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), **kw)


def oracle_state_arrays(tr, P, S):
    """The oracle's teacher-forced states in the runner's trace layout."""
    h = list(tr.prefix_h) + [tr.h[t + 1] for t in range(S - 1)]
    gh = list(tr.prefix_gh) + list(tr.gh)
    return {
        "z": tr.z_part,
        "h": np.stack(h),
        "gh": np.stack(gh) if gh else np.zeros((0,) + tr.h[0].shape[:1] + (3 * tr.h[0].shape[1],), np.float32),
        "s": np.stack(tr.s_proj),
    }


def check_against_oracle(w, prefix, ph, base, tokens, states, P, S, min_exact):
    frac, tr = teacher_forced_check(w, prefix, ph, base, tokens, min_exact=min_exact)
    ref = oracle_state_arrays(tr, P, S)
    parts = []
    for k in ("z", "h", "gh", "s"):
        mx, same = compare_states(k, states[k], ref[k])
        parts.append(f"{k} max|d| {mx:.3g} bit-equal {same:.3f}")
    log_parity("states vs oracle: " + "; ".join(parts))
    return frac


@pytest.mark.parametrize("case", [c for c in ROLLOUT_CASES if "bf16" in c])
def test_golden_states_match_reference(case):
    """GPU states against the reference runner's own recorded states."""
    fx = load(case)
    B, H, G, E, V, S, P = (int(x) for x in fx["meta"][:7])
    draft, target = modules_from_fixture(fx)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    prefix = torch.from_numpy(fx["prefix_ids"]).cuda()
    ph = torch.from_numpy(as_f32(fx["parallel_hiddens"])).cuda().bfloat16()
    base = torch.from_numpy(as_f32(fx["base_logits"])).cuda().bfloat16()
    tokens, st = r.rollout_trace(prefix, ph, base)
    assert r.status() == 0
    # the traced call is the same computation as the graph-replayed one
    assert torch.equal(tokens, make_runner(draft, target, B, S, H, G, V, P)(prefix, ph, base))
    got = tokens.cpu().numpy()
    ref_tok = fx["tokens_triton"]
    # steps t < agree[b] saw the reference's history
    agree = np.where((got != ref_tok).any(1), np.argmax(got != ref_tok, axis=1), S)
    log_parity(f"tokens equal to the reference's: {int((got == ref_tok).sum())}/{got.size}")
    z_mx, _ = compare_states("z", st["z"], as_f32(fx["z_part"]))
    h0_mx, _ = compare_states("h0", st["h"][P - 1], as_f32(fx["h0"]))
    mx = {"s": 0.0, "gh": 0.0, "h": 0.0}
    s_ref, gh_ref, h_ref = as_f32(fx["s_proj"]), as_f32(fx["gh"]), as_f32(fx["h_out"])
    for b in range(B):
        for t in range(int(agree[b]) + 1 if agree[b] < S else S):
            # s of step t depends only on tokens before t
            mx["s"] = max(mx["s"], compare_states(f"s[b={b}, t={t}]", st["s"][t, b], s_ref[b, t])[0])
        for t in range(min(int(agree[b]) + 1, S - 1) if agree[b] < S else S - 1):
            mx["gh"] = max(mx["gh"], compare_states(f"gh[b={b}, t={t}]", st["gh"][P - 1 + t, b], gh_ref[b, t])[0])
        for t in range(min(int(agree[b]), S - 1)):
            mx["h"] = max(mx["h"], compare_states(f"h[b={b}, t={t}]", st["h"][P + t, b], h_ref[b, t])[0])
    log_parity(f"states vs reference: z {z_mx:.3g}, h0 {h0_mx:.3g}, s {mx['s']:.3g}, gh {mx['gh']:.3g}, "
               f"h {mx['h']:.3g} (max |diff|)")
    check_against_oracle(oracle_weights(draft, target), prefix, ph, base, tokens, st, P, S, min_exact=1.0)


STATE_SHAPES = [
    # B, H, G, E, V, S, P, biases, fc2_std, dtype
    (1, 256, 256, 320, 3000, 15, 1, False, 0.05, torch.bfloat16),
    (3, 128, 128, 200, 2000, 13, 3, True, 0.05, torch.bfloat16),
    (8, 128, 64, 136, 1500, 15, 2, True, 0.08, torch.bfloat16),
    (32, 128, 128, 256, 2500, 15, 1, False, 0.05, torch.bfloat16),
    (5, 256, 192, 320, 3001, 15, 1, True, 0.05, torch.float16),
]


@pytest.mark.parametrize("B,H,G,E,V,S,P,bias,fc2_std,dtype", STATE_SHAPES)
def test_states_match_oracle(B, H, G, E, V, S, P, bias, fc2_std, dtype):
    draft, target = random_modules(H, G, E, V, seed=B * 5 + G, fc2_std=fc2_std, dtype=dtype,
                                   fc1_bias=bias, fc2_bias=bias, gru_bias=bias)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=B + 50, dtype=dtype)
    tokens, st = r.rollout_trace(prefix, ph, base)
    assert r.status() == 0
    w = oracle_weights(draft, target, "fp16" if dtype == torch.float16 else "bf16")
    check_against_oracle(w, prefix, ph, base, tokens, st, P, S, min_exact=1.0)


def test_trace_leaves_the_rollout_unchanged():
    """Tracing copies states out between launches; the tokens are those of
    the untraced (persistent or phased) rollout."""
    from domino_b200 import _lib

    B, H, G, E, V, S, P = 4, 128, 128, 192, 1500, 15, 2
    draft, target = random_modules(H, G, E, V, seed=3, fc2_std=0.08, fc1_bias=True, gru_bias=True)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=9)
    plain = r(prefix, ph, base)
    traced, _ = r.rollout_trace(prefix, ph, base)
    assert torch.equal(plain, traced)
    assert r._lib.dd_set_rollout_mode(r._h, 0) == _lib.DD_OK
    assert torch.equal(r(prefix, ph, base), traced)
    assert r.status() == 0
