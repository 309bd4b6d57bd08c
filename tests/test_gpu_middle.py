"""Heads whose embed_proj middle is not a single SiLU (identity, ReLU, GELU,
Tanh, Sigmoid, a SiLU followed by Dropout).  For these the reference always
takes its PyTorch branch (code/kernel/domino.py:406-431): every op rounded to
the weight dtype, the fc2 logits rounded before and after the base logits are
added, a GRU cell with tanh.  The kernels reproduce it (dd_set_middle); the
checker is that branch's op sequence run with CUDA torch ops
(oracle/torch_branch.py), which is the reference's own GPU arithmetic for
these heads, teacher forced: every token equals its argmax or is a near-tie
within 2e-2.  The reference's own tokens (tests/golden/middle_*.npz) too.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

from tests.fixtures import as_f32, load
from tests.gpu_helpers import TOL, log_parity, modules_from_fixture, random_inputs, random_modules

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


def make_runner(draft, target, B, S, H, G, V, P, **kw):
    from domino_b200 import DraftCorrectionGraphRunner
    return DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), **kw)


def check_torch_branch(draft, target, prefix, ph, base, out, min_exact=1.0):
    from oracle import torch_branch as TB

    w = TB.head_from_modules(draft, target, device="cuda")
    rec = {}
    own = TB.rollout(w, prefix, ph, base, teacher_tokens=out, record=rec)
    exact = own == out
    slack = rec["top"] - rec["chosen"]
    assert torch.all(exact | (slack <= TOL + TOL * rec["top"].abs())), (out, own, slack)
    frac = exact.float().mean().item()
    log_parity(f"tokens {int(exact.sum())}/{exact.numel()} equal to the PyTorch branch's (teacher forced), "
               f"worst near-tie slack {float(slack[~exact].max()) if (~exact).any() else 0.0:.3g}")
    assert frac >= min_exact
    return frac


@pytest.mark.parametrize("case", ["middle_gelu_b2", "middle_identity_b2"])
def test_reference_middle_fixtures(case):
    fx = load(case)
    B, H, G, E, V, S, P = (int(x) for x in fx["meta"][:7])
    draft, target = modules_from_fixture(fx)
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix = torch.from_numpy(fx["prefix_ids"]).cuda()
    ph = torch.from_numpy(as_f32(fx["parallel_hiddens"])).cuda().bfloat16()
    base = torch.from_numpy(as_f32(fx["base_logits"])).cuda().bfloat16()
    out = r(prefix, ph, base)
    assert r.status() == 0
    same = (out.cpu().numpy() == fx["tokens_torch"]).mean()
    log_parity(f"{case}: {same:.3f} of the tokens equal the reference's (its PyTorch branch, on the CPU)")
    check_torch_branch(draft, target, prefix, ph, base, out)


MIDDLE_CASES = [
    # middle module, dtype, B, P
    (nn.GELU(), torch.bfloat16, 3, 1),
    (nn.GELU(approximate="tanh"), torch.bfloat16, 5, 2),
    (nn.ReLU(), torch.bfloat16, 8, 1),
    (nn.Tanh(), torch.float16, 2, 1),
    (nn.Sigmoid(), torch.bfloat16, 1, 1),
    (nn.Sequential(nn.SiLU(), nn.Dropout(0.1)), torch.bfloat16, 4, 1),
    (None, torch.bfloat16, 6, 3),            # embed_proj of two Linears: an identity middle
    (nn.GELU(), torch.float32, 3, 1),        # fp32 heads: the PyTorch branch in fp32
]


@pytest.mark.parametrize("middle,dtype,B,P", MIDDLE_CASES)
def test_other_middles_match_the_pytorch_branch(middle, dtype, B, P):
    H, G, E, V, S = 128, 128, 192, 2000, 15
    draft, target = random_modules(H, G, E, V, seed=B * 13 + P, fc2_std=0.1, dtype=torch.float32, gru_bias=True)
    if middle is None:
        draft.embed_proj = nn.Sequential(draft.embed_proj[0], draft.embed_proj[2])
    else:
        draft.embed_proj[1] = middle
    draft, target = draft.to(dtype).eval(), target.to(dtype).eval()
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=B, dtype=dtype)
    out = r(prefix, ph, base)
    assert r.status() == 0
    check_torch_branch(draft, target, prefix, ph, base, out)
    # the fused lm_head block takes the same branch
    K = P - 1 + S
    g = torch.Generator().manual_seed(2)
    ph2 = torch.randn(B, K, H, generator=g).cuda().to(dtype)
    last = torch.randint(0, V, (B,), generator=g).cuda()
    verify, base2 = r.draft_block(last, ph2)
    assert r.status() == 0
    check_torch_branch(draft, target, verify[:, :P], ph2[:, P - 1:], base2[:, P - 1:], verify[:, P:])
