"""fp32 draft heads (the reference's CPU-runnable configuration: fp32 weights,
fp32 arithmetic throughout, code/kernel/domino.py:58-136, 374-431), through
the C ABI: the CUDA-core fp32 weight stream (gemv_f32_kernel) and the fp32
GRU cell.

Checked against the reference's own recorded fp32 run (tests/golden/
rollout_fp32_b1.npz: in fp32 its Triton and PyTorch branches agree) and
against the oracle in fp32 (nothing rounded), teacher forced: tokens equal,
or a near-tie within 2e-2; states within atol = rtol = 2e-2 (in practice
~1e-6, the difference between two fp32 summation orders).
"""
import gc

import numpy as np
import pytest
import torch

from tests.fixtures import as_f32, load
from tests.gpu_helpers import (
    compare_states, log_parity, modules_from_fixture, oracle_weights, random_inputs, random_modules,
    teacher_forced_check,
)
from tests.test_gpu_states import check_against_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


def make_runner(draft, target, B, S, H, G, V, P, **kw):
    from domino_b200 import DraftCorrectionGraphRunner
    return DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), **kw)


def fp32_modules_from_fixture(fx):
    draft, target = modules_from_fixture(fx, device="cpu")
    draft, target = draft.float(), target.float()
    with torch.no_grad():
        for mod, key in ((draft.embed_proj[0], "fc1"), (draft.embed_proj[2], "fc2"), (target.lm_head, "lm_head")):
            mod.weight.copy_(torch.from_numpy(as_f32(fx[key])))
        draft.prefix_gru.weight_ih_l0.copy_(torch.from_numpy(as_f32(fx["w_ih"])))
        draft.prefix_gru.weight_hh_l0.copy_(torch.from_numpy(as_f32(fx["w_hh"])))
        target.model.embed_tokens.weight.copy_(torch.from_numpy(as_f32(fx["embed"])))
    return draft.cuda(), target.cuda()


def test_fp32_golden_matches_reference():
    fx = load("rollout_fp32_b1")
    B, H, G, E, V, S, P = (int(x) for x in fx["meta"][:7])
    draft, target = fp32_modules_from_fixture(fx)
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix = torch.from_numpy(fx["prefix_ids"]).cuda()
    ph = torch.from_numpy(as_f32(fx["parallel_hiddens"])).cuda()
    base = torch.from_numpy(as_f32(fx["base_logits"])).cuda()
    out = r(prefix, ph, base)
    assert r.status() == 0
    assert np.array_equal(out.cpu().numpy(), fx["tokens_triton"])
    assert np.array_equal(out.cpu().numpy(), fx["tokens_torch"])
    tokens, st = r.rollout_trace(prefix, ph, base)
    assert torch.equal(tokens, out)
    tab_mx, _ = compare_states("table", r.table, as_f32(fx["table"]))
    parts = [f"table {tab_mx:.3g}"]
    for name, got, ref in (("z", st["z"], as_f32(fx["z_part"])), ("h0", st["h"][P - 1], as_f32(fx["h0"])),
                           ("s", st["s"].transpose(0, 1), as_f32(fx["s_proj"])),
                           ("gh", st["gh"][P - 1:].transpose(0, 1), as_f32(fx["gh"])),
                           ("h", st["h"][P:].transpose(0, 1), as_f32(fx["h_out"]))):
        mx, _ = compare_states(name, got, ref)
        parts.append(f"{name} {mx:.3g}")
    log_parity("fp32 tokens equal the reference's; states vs reference (max |diff|): " + ", ".join(parts))
    check_against_oracle(oracle_weights(draft, target, "fp32"), prefix, ph, base, tokens, st, P, S, min_exact=1.0)


FP32_SHAPES = [
    # B, H, G, E, V, S, P, biases
    (1, 128, 128, 192, 3000, 15, 1, False),
    (3, 128, 96, 136, 2000, 13, 3, True),
    (20, 64, 64, 96, 1500, 15, 2, True),   # 20 X rows: two launches of <= 16 per phase
]


@pytest.mark.parametrize("B,H,G,E,V,S,P,bias", FP32_SHAPES)
def test_fp32_states_match_oracle(B, H, G, E, V, S, P, bias):
    draft, target = random_modules(H, G, E, V, seed=B * 3 + E, fc2_std=0.08, dtype=torch.float32,
                                   fc1_bias=bias, fc2_bias=bias, gru_bias=bias)
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=B + 7, dtype=torch.float32)
    out = r(prefix, ph, base)
    tokens, st = r.rollout_trace(prefix, ph, base)
    assert r.status() == 0
    assert torch.equal(out, tokens)
    w = oracle_weights(draft, target, "fp32")
    tab_mx, _ = compare_states("table", r.table, w.get_table())
    log_parity(f"fp32 table max|d| {tab_mx:.3g}")
    check_against_oracle(w, prefix, ph, base, tokens, st, P, S, min_exact=1.0)


def test_fp32_draft_block_fused_lm_head():
    from oracle import draft_oracle as O

    B, H, G, E, V, S, P = 3, 128, 128, 192, 1501, 13, 3
    draft, target = random_modules(H, G, E, V, seed=5, fc2_std=0.08, dtype=torch.float32)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    K = P - 1 + S
    g = torch.Generator().manual_seed(9)
    ph = torch.randn(B, K, H, generator=g).cuda()
    last = torch.randint(0, V, (B,), generator=g).cuda()
    verify, base = r.draft_block(last, ph)
    assert r.status() == 0 and base.dtype == torch.float32
    base_ref = O.lm_head(ph.cpu().numpy(), target.lm_head.weight.detach().cpu().numpy(), "fp32")
    mx, _ = compare_states("base logits", base, base_ref)
    v = verify.cpu().numpy()
    assert np.array_equal(v[:, 1:P], O.pure_draft_prefix(base.cpu().numpy(), P - 1))
    out = r(torch.from_numpy(v[:, :P]).cuda(), ph[:, P - 1:], base[:, P - 1:])
    assert torch.equal(out.cpu(), torch.from_numpy(v[:, P:]))
    log_parity(f"fp32 fused lm_head max|d| {mx:.3g}")


def test_fp32_qwen3_4b_shape_teacher_forced():
    """The reference's CPU-runnable configuration: Qwen3-4B-shaped fp32 head,
    H = G = 2560, E = 6912, V = 151936, batch 1 (checked against the fp32
    torch restatement, nothing rounded; the table built by cuBLAS)."""
    import bench
    from tests.torch_reference import build_table, teacher_forced_rollout

    H = G = 2560
    E, V, S = 6912, 151936, 15
    dev = torch.device("cuda", 0)
    draft, target = bench.build_modules(H, G, E, V, dev, seed=4)
    draft, target = draft.float(), target.float()
    r = make_runner(draft, target, 1, S, H, G, V, 1)
    try:
        g = torch.Generator(device="cuda").manual_seed(3)
        ph = torch.randn(1, S, H, generator=g, device="cuda")
        prefix = torch.randint(0, V, (1, 1), generator=g, device="cuda")
        with torch.no_grad():
            base = target.lm_head(ph)
        out = r(prefix, ph, base)
        tokens, st = r.rollout_trace(prefix, ph, base)
        assert r.status() == 0 and torch.equal(out, tokens)
        gru = draft.prefix_gru
        table = build_table(target.model.embed_tokens.weight, gru.weight_ih_l0)
        tab_mx, _ = compare_states("table", r.table, table)
        ref_states = {}
        own, chosen, top = teacher_forced_rollout(draft.embed_proj[0].weight, draft.embed_proj[2].weight,
                                                  gru.weight_hh_l0, table, prefix, ph, base, out,
                                                  states=ref_states, round_bf16=False)
        exact = own == out
        slack = top - chosen
        assert torch.all(exact | (slack <= 2e-2 + 2e-2 * top.abs()))
        line = f"fp32 Qwen3-4B shape: tokens {int(exact.sum())}/{exact.numel()} exact; table {tab_mx:.3g}"
        for k in ("z", "h", "gh", "s"):
            mx, _ = compare_states(k, st[k], ref_states[k])
            line += f", {k} {mx:.3g}"
        log_parity(line)
        assert bool(exact.all())
    finally:
        r.close()
        del r, draft, target
        gc.collect()
        torch.cuda.empty_cache()
