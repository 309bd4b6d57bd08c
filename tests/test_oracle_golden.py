"""Pin the CPU oracle to outputs of the reference itself (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py, which runs the
reference's ``DraftCorrectionGraphRunner`` (Triton kernels under the Triton
interpreter, and its PyTorch branch) and its ``spec_generate`` block loop.
"""
import numpy as np
import pytest

from oracle import draft_oracle as O
from tests.fixtures import ROLLOUT_CASES, TRACE_CASES, as_f32, load, weights

TOL = 2e-2  # atol = rtol for dtype-rounded states and logits


def close(a, b, tol=TOL):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return np.all(np.abs(a - b) <= tol + tol * np.abs(b)), float(np.max(np.abs(a - b)))


def test_bf16_rounding_matches_torch():
    import torch
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 37
    x[:4] = [0.0, -0.0, 1e-40, 3.0e38]
    ours = O.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)


def test_packed_key_order():
    rng = np.random.default_rng(1)
    v = rng.standard_normal(5000).astype(np.float32)
    v[100] = v[50]  # a tie: lower index must win
    v[10] = -np.inf
    keys = O.packed_argmax_key(v, np.arange(v.size))
    assert int(np.argmax(keys)) == int(O.argmax_lowest(v))
    w = np.full(8, 3.5, np.float32)
    assert int(np.argmax(O.packed_argmax_key(w, np.arange(8)))) == 0


def test_packed_key_nan_is_the_maximum_like_torch_argmax():
    """NaN ranks above +inf and the first NaN wins, as in torch.argmax."""
    import torch

    for v in ([1.0, np.nan, np.inf, -np.nan, 5.0], [-np.nan, 2.0, np.nan], [np.inf, 3.0, -np.nan]):
        v = np.asarray(v, np.float32)
        keys = O.packed_argmax_key(v, np.arange(v.size))
        expect = int(torch.argmax(torch.from_numpy(v)))
        assert int(np.argmax(keys)) == expect == int(O.argmax_lowest(v))


@pytest.mark.parametrize("case", ROLLOUT_CASES)
def test_table_and_z_part(case):
    fx = load(case)
    w = weights(fx)
    ok, err = close(w.get_table(), as_f32(fx["table"]))
    assert ok, err
    z = O.linear(as_f32(fx["parallel_hiddens"]), w.w_z, w.fc1_bias, w.dtype)
    ok, err = close(z, as_f32(fx["z_part"]))
    assert ok, err


@pytest.mark.parametrize("case", ROLLOUT_CASES)
def test_prefix_gru_h0(case):
    fx = load(case)
    w = weights(fx)
    h0 = O.prefix_gru(w, fx["prefix_ids"])
    ok, err = close(h0, as_f32(fx["h0"]))
    assert ok, err


@pytest.mark.parametrize("case", ROLLOUT_CASES)
def test_rollout_teacher_forced_states(case):
    """Fed the reference's own tokens, every per-step state agrees."""
    fx = load(case)
    w = weights(fx)
    ref_tok = fx["tokens_triton"]
    tr = O.rollout(w, fx["prefix_ids"], as_f32(fx["parallel_hiddens"]), as_f32(fx["base_logits"]),
                   teacher_tokens=ref_tok)
    S = ref_tok.shape[1]
    s_ref = as_f32(fx["s_proj"])
    for t in range(S):
        ok, err = close(tr.s_proj[t], s_ref[:, t])
        assert ok, (t, err)
    h_ref = as_f32(fx["h_out"])
    gh_ref = as_f32(fx["gh"])
    for t in range(S - 1):
        ok, err = close(tr.h[t + 1], h_ref[:, t])
        assert ok, (t, err)
        ok, err = close(tr.gh[t], gh_ref[:, t])
        assert ok, (t, err)
    ok, err = close(tr.prefix_h[-1], as_f32(fx["h0"]))
    assert ok, err
    # Own argmax vs the reference's token at every step: equal, or a near-tie.
    diff = tr.tokens != ref_tok
    assert np.all(tr.gaps[diff] < TOL), (np.argwhere(diff), tr.gaps[diff])


@pytest.mark.parametrize("case", ROLLOUT_CASES)
def test_rollout_free_running_tokens(case):
    """Free-running oracle tokens equal the reference Triton-path tokens."""
    fx = load(case)
    w = weights(fx)
    tr = O.rollout(w, fx["prefix_ids"], as_f32(fx["parallel_hiddens"]), as_f32(fx["base_logits"]))
    assert np.array_equal(tr.tokens, fx["tokens_triton"])
    if str(fx["dtype"]) == "fp32":
        # In fp32 the reference's PyTorch branch agrees with its Triton branch too.
        assert np.array_equal(tr.tokens, fx["tokens_torch"])


def test_lm_head_matches_reference_base_logits():
    fx = load("rollout_bf16_b3_bias")
    base = O.lm_head(as_f32(fx["parallel_hiddens"]), as_f32(fx["lm_head"]), "bf16")
    ok, err = close(base, as_f32(fx["base_logits"]))
    assert ok, err


def test_accept_cases():
    fx = load("accept_cases")
    a, bonus = O.accept(fx["verify_ids"], fx["posterior"])
    assert np.array_equal(a, fx["accept"])
    assert np.array_equal(bonus, fx["bonus"])


@pytest.mark.parametrize("case", TRACE_CASES)
def test_spec_generate_trace(case):
    """Replays every runner call and verify step of the reference block loop."""
    fx = load(case)
    w = weights(fx, "fp32" if fx["fc1"].dtype == np.float32 else "bf16")
    nblk = fx["runner_out"].shape[0]
    for i in range(nblk):
        tr = O.rollout(w, fx["prefix_ids"][i], as_f32(fx["parallel_hiddens"][i]), as_f32(fx["base_logits"][i]))
        assert np.array_equal(tr.tokens, fx["runner_out"][i]), i
        verify = fx["verify_ids"][i]
        assert np.array_equal(verify[:, 1:], fx["runner_out"][i])
        assert np.array_equal(verify[:, :1], fx["prefix_ids"][i])
        a, bonus = O.accept(verify, fx["posterior"][i])
        assert int(a[0]) + 1 == int(fx["acceptance_lengths"][i])
        assert int(bonus[0]) == int(fx["posterior"][i][0, a[0]])


@pytest.mark.parametrize("case", ROLLOUT_CASES)
def test_torch_branch_matches_reference_pytorch_branch(case):
    """The CPU benchmark leg (oracle/torch_branch.py) reproduces the tokens of
    the reference's PyTorch branch, recorded by running it (tokens_torch)."""
    import torch

    from oracle import torch_branch as TB
    from tests.gpu_helpers import modules_from_fixture

    fx = load(case)
    draft, target = modules_from_fixture(fx, device="cpu")
    if str(fx["dtype"]) == "fp32":
        draft, target = draft.float(), target.float()
        for mod, key in ((draft.embed_proj[0], "fc1"), (draft.embed_proj[2], "fc2")):
            mod.weight.data.copy_(torch.from_numpy(as_f32(fx[key])))
        draft.prefix_gru.weight_ih_l0.data.copy_(torch.from_numpy(as_f32(fx["w_ih"])))
        draft.prefix_gru.weight_hh_l0.data.copy_(torch.from_numpy(as_f32(fx["w_hh"])))
        target.model.embed_tokens.weight.data.copy_(torch.from_numpy(as_f32(fx["embed"])))
    dt = draft.embed_proj[0].weight.dtype
    w = TB.head_from_modules(draft, target)
    assert torch.equal(w.table.float(), torch.from_numpy(as_f32(fx["table"])))
    out = TB.rollout(w, torch.from_numpy(fx["prefix_ids"]), torch.from_numpy(as_f32(fx["parallel_hiddens"])).to(dt),
                     torch.from_numpy(as_f32(fx["base_logits"])).to(dt))
    assert np.array_equal(out.numpy(), fx["tokens_torch"])


@pytest.mark.parametrize("case", ["middle_gelu_b2", "middle_identity_b2"])
def test_torch_branch_matches_reference_for_other_middles(case):
    """Heads whose middle is not a single SiLU: the reference's runner takes its
    PyTorch branch, and the torch restatement (the checker of the kernels for
    these heads) gives its tokens."""
    import torch

    from oracle import torch_branch as TB
    from tests.gpu_helpers import modules_from_fixture

    fx = load(case)
    draft, target = modules_from_fixture(fx, device="cpu")
    w = TB.head_from_modules(draft, target)
    out = TB.rollout(w, torch.from_numpy(fx["prefix_ids"]), torch.from_numpy(as_f32(fx["parallel_hiddens"])).bfloat16(),
                     torch.from_numpy(as_f32(fx["base_logits"])).bfloat16())
    assert np.array_equal(out.numpy(), fx["tokens_torch"])
