"""Parity at the benchmark's full size (Qwen3-8B-shaped draft head: H = G = 4096,
E = 12288, V = 151936, bf16), where the CPU oracle would take minutes.

Checked against an fp32 PyTorch restatement of the same arithmetic on the GPU
(tests/torch_reference.py), teacher forced with our tokens, plus
size-independent properties: determinism, graph replay, the fused-lm_head
block agreeing with the runner call, and acceptance of a target that agrees
with the draft.
"""
import pytest
import torch

from tests.torch_reference import teacher_forced_rollout

pytestmark = pytest.mark.gpu

TOL = 2e-2
H = G = 4096
E = 12288
V = 151936
S = 15


@pytest.fixture(scope="module")
def model():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")
    import bench
    from domino_b200 import DraftCorrectionGraphRunner

    dev = torch.device("cuda", 0)
    draft, target = bench.build_modules(H, G, E, V, dev, seed=123)
    runner = DraftCorrectionGraphRunner(draft, target, 2, S, H, G, V, 1, dev)
    yield draft, target, runner
    runner.close()


def _inputs(target, B, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ph = torch.randn(B, S, H, generator=g, device="cuda").to(torch.bfloat16)
    prefix = torch.randint(0, V, (B, 1), generator=g, device="cuda")
    with torch.no_grad():
        base = target.lm_head(ph)
    return prefix, ph, base


def test_fullsize_tokens_teacher_forced(model):
    draft, target, runner = model
    for seed in (1, 2):
        prefix, ph, base = _inputs(target, 2, seed)
        out = runner(prefix, ph, base)
        assert runner.status() == 0
        own, chosen, top = teacher_forced_rollout(
            draft.embed_proj[0].weight, draft.embed_proj[2].weight, draft.prefix_gru.weight_hh_l0,
            runner.table, prefix, ph, base, out)
        exact = own == out
        slack = top - chosen
        assert torch.all(exact | (slack <= TOL + TOL * top.abs())), (out, own, slack)
        assert exact.float().mean().item() >= 0.9


def test_fullsize_determinism_and_graph_replay(model):
    draft, target, runner = model
    from domino_b200 import DraftCorrectionGraphRunner

    eager = DraftCorrectionGraphRunner(draft, target, 2, S, H, G, V, 1, torch.device("cuda", 0), use_graph=False)
    prefix, ph, base = _inputs(target, 2, 7)
    a = runner(prefix, ph, base)
    b = eager(prefix, ph, base)
    c = runner(prefix, ph, base)
    assert torch.equal(a, b) and torch.equal(a, c)
    eager.close()


def test_fullsize_draft_block_and_accept(model):
    draft, target, runner = model
    prefix, ph, base = _inputs(target, 2, 11)
    verify, base_out = runner.draft_block(prefix[:, 0], ph)
    assert runner.status() == 0
    ref = base.float()
    assert torch.all((base_out.float() - ref).abs() <= TOL + TOL * ref.abs())
    # identical base logits -> identical tokens to the runner call
    out = runner(prefix, ph, base_out)
    assert torch.equal(verify[:, 1:], out)
    # a target that agrees with the draft accepts the whole block
    posterior = torch.cat([verify[:, 1:], verify[:, -1:]], 1)
    acc, bonus = runner.accept(verify, posterior)
    assert acc.tolist() == [S, S]
    assert torch.equal(bonus, verify[:, -1])
