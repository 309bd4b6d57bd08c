"""Parity of the sm_100a path (through libdomino_draft's C ABI) with the
oracle and with the reference's own outputs (golden fixtures).

Token rule: every draft token equals the oracle's argmax given the same
history (teacher forcing), or the oracle's logit of that token is within
2e-2 (abs + rel) of its top logit (a near-tie).  Integer outputs
(acceptance, bonus tokens, prefix tokens over identical logits) are exact.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import draft_oracle as O
from tests.fixtures import ROLLOUT_CASES, as_f32, load
from tests.gpu_helpers import (
    TOL, modules_from_fixture, oracle_weights, random_inputs, random_modules, teacher_forced_check,
)

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail("GPU tests need an sm_100 device")


def make_runner(draft, target, B, S, H, G, V, P, **kw):
    from domino_b200 import DraftCorrectionGraphRunner
    return DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), **kw)


@pytest.mark.parametrize("case", [c for c in ROLLOUT_CASES if "bf16" in c])
def test_golden_fixture_tokens(case):
    """The reference's own tokens (Triton branch) for the fixture inputs."""
    fx = load(case)
    B, H, G, E, V, S, P = (int(x) for x in fx["meta"][:7])
    draft, target = modules_from_fixture(fx)
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix = torch.from_numpy(fx["prefix_ids"]).cuda()
    ph = torch.from_numpy(as_f32(fx["parallel_hiddens"])).cuda().bfloat16()
    base = torch.from_numpy(as_f32(fx["base_logits"])).cuda().bfloat16()
    out = r(prefix, ph, base)
    assert r.status() == 0
    ref = fx["tokens_triton"]
    got = out.cpu().numpy()
    w = oracle_weights(draft, target)
    frac, tr = teacher_forced_check(w, prefix, ph, base, out, min_exact=1.0)
    # Against the reference directly: where the reference's own step had a
    # clear winner (gap >= TOL under the reference's history), we agree.
    tr_ref = O.rollout(w, fx["prefix_ids"], as_f32(fx["parallel_hiddens"]), as_f32(fx["base_logits"]),
                       teacher_tokens=ref)
    first_diff = np.argmax(got != ref, axis=1)
    for b in range(B):
        if (got[b] == ref[b]).all():
            continue
        t = first_diff[b]
        assert tr_ref.gaps[b, t] < TOL, (b, t, tr_ref.gaps[b, t])


def test_table_matches_oracle():
    H, G, E, V = 128, 96, 160, 1000
    draft, target = random_modules(H, G, E, V, seed=3, gru_bias=True)
    r = make_runner(draft, target, 2, 15, H, G, V, 1, use_graph=False)
    w = oracle_weights(draft, target)
    ref = w.get_table()
    got = r.table.float().cpu().numpy()
    assert np.all(np.abs(got - ref) <= TOL + TOL * np.abs(ref))
    # bf16 rounding of an fp32 sum: all but a few elements are bit-identical
    assert np.mean(got == ref) > 0.99


SHAPES = [
    # B, H, G, E, V, S, P, biases, fc2_std
    (1, 256, 256, 320, 3000, 15, 1, False, 0.05),
    (5, 256, 192, 320, 3001, 15, 1, False, 0.05),
    (3, 128, 128, 200, 2000, 13, 3, True, 0.05),
    (8, 128, 64, 136, 1500, 15, 1, True, 0.08),
    (17, 64, 64, 96, 1000, 15, 2, False, 0.1),
    (32, 128, 128, 256, 2500, 15, 1, False, 0.05),
]


@pytest.mark.parametrize("B,H,G,E,V,S,P,bias,fc2_std", SHAPES)
def test_rollout_random_shapes(B, H, G, E, V, S, P, bias, fc2_std):
    draft, target = random_modules(H, G, E, V, seed=B * 7 + H, fc2_std=fc2_std,
                                   fc1_bias=bias, fc2_bias=bias, gru_bias=bias)
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=B)
    out = r(prefix, ph, base)
    assert r.status() == 0
    assert out.shape == (B, S) and out.dtype == torch.long
    teacher_forced_check(oracle_weights(draft, target), prefix, ph, base, out)


def test_rollout_fp16():
    B, H, G, E, V, S, P = 2, 128, 128, 192, 1200, 15, 1
    draft, target = random_modules(H, G, E, V, seed=11, dtype=torch.float16, fc2_std=0.08)
    r = make_runner(draft, target, B, S, H, G, V, P)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=5, dtype=torch.float16)
    out = r(prefix, ph, base)
    assert r.status() == 0
    teacher_forced_check(oracle_weights(draft, target, "fp16"), prefix, ph, base, out)


def test_graph_replay_matches_eager_and_is_deterministic():
    B, H, G, E, V, S, P = 4, 128, 128, 256, 2048, 15, 1
    draft, target = random_modules(H, G, E, V, seed=21, fc2_std=0.08)
    rg = make_runner(draft, target, B, S, H, G, V, P, use_graph=True)
    re = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    for seed in range(3):
        prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=seed)
        a = rg(prefix, ph, base)
        b = re(prefix, ph, base)
        c = rg(prefix, ph, base)
        assert torch.equal(a, b) and torch.equal(a, c)


@pytest.mark.parametrize("B,P", [(1, 1), (5, 3)])
def test_packed_and_row_major_weights_agree_exactly(B, P):
    """The packed tile layout feeds the tensor cores the same bytes as TMA."""
    H, G, E, V, S = 192, 128, 328, 3001, 13
    draft, target = random_modules(H, G, E, V, seed=61 + B, fc2_std=0.08, fc1_bias=True)
    rp = make_runner(draft, target, B, S, H, G, V, P, use_graph=False, pack_weights=True)
    rr = make_runner(draft, target, B, S, H, G, V, P, use_graph=False, pack_weights=False)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=2)
    assert torch.equal(rp(prefix, ph, base), rr(prefix, ph, base))
    K = P - 1 + S
    g = torch.Generator().manual_seed(4)
    ph2 = torch.randn(B, K, H, generator=g).cuda().bfloat16()
    last = torch.randint(0, V, (B,), generator=g).cuda()
    vp, bp = rp.draft_block(last, ph2)
    vr, br = rr.draft_block(last, ph2)
    assert torch.equal(vp, vr) and torch.equal(bp, br)
    assert rp.status() == 0 and rr.status() == 0


@pytest.mark.parametrize("B,H,G,E,V,S,P", [
    (1, 128, 128, 192, 1500, 15, 1),
    (3, 256, 192, 320, 3001, 13, 3),
    (8, 128, 64, 136, 2000, 15, 1),
    (17, 64, 64, 96, 1000, 15, 2),
])
def test_persistent_rollout_matches_phased_exactly(B, H, G, E, V, S, P):
    """The one-kernel rollout and the kernel-per-phase rollout split the work
    the same way, so their tokens are identical."""
    from domino_b200 import _lib

    draft, target = random_modules(H, G, E, V, seed=90 + B, fc2_std=0.08, fc1_bias=True, gru_bias=True)
    rp = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    rk = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    lib = _lib.load()
    assert lib.dd_set_rollout_mode(rp._h, 0) == _lib.DD_OK
    assert lib.dd_set_rollout_mode(rk._h, 1) == _lib.DD_OK
    for seed in range(2):
        prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=seed)
        a = rp(prefix, ph, base)
        b = rk(prefix, ph, base)
        assert torch.equal(a, b), (a, b)
    K = P - 1 + S
    g = torch.Generator().manual_seed(5)
    ph2 = torch.randn(B, K, H, generator=g).cuda().bfloat16()
    last = torch.randint(0, V, (B,), generator=g).cuda()
    va, ba = rp.draft_block(last, ph2)
    vb, bb = rk.draft_block(last, ph2)
    assert torch.equal(va, vb) and torch.equal(ba, bb)
    assert rp.status() == 0 and rk.status() == 0
    # and the persistent path is the one that ran
    lib.dd_set_timing(rp._h, 1)
    rp(prefix, ph, base)
    kinds = (ctypes.c_int32 * 64)()
    ms = (ctypes.c_float * 64)()
    n = lib.dd_read_timing(rp._h, kinds, ms, 64)
    lib.dd_set_timing(rp._h, 0)
    assert 9 in list(kinds[:n]), list(kinds[:n])


@pytest.mark.parametrize("B,V", [
    (3, 1500),   # one z / lm_head pass, N = 48
    (20, 2048),  # B*K = 300 rows: two passes (256 + 44), staged row-contiguous stores
    (20, 1501),  # same, base logits row stride not a multiple of 4: element-wise stores
])
def test_draft_block_fused_lm_head(B, V):
    H, G, E, S, P = 128, 128, 192, 13, 3
    draft, target = random_modules(H, G, E, V, seed=31 + B, fc2_std=0.08)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    K = P - 1 + S
    g = torch.Generator().manual_seed(9)
    ph = torch.randn(B, K, H, generator=g).cuda().bfloat16()
    last = torch.randint(0, V, (B,), generator=g).cuda()
    verify, base = r.draft_block(last, ph)
    assert r.status() == 0
    lm = target.lm_head.weight.detach().float().cpu().numpy()
    base_ref = O.lm_head(ph.float().cpu().numpy(), lm, "bf16")
    base_np = base.float().cpu().numpy()
    assert np.all(np.abs(base_np - base_ref) <= TOL + TOL * np.abs(base_ref))
    v = verify.cpu().numpy()
    assert np.array_equal(v[:, 0], last.cpu().numpy())
    # pure-draft prefix tokens are the argmax of the (bf16) base logits we wrote
    assert np.array_equal(v[:, 1:P], O.pure_draft_prefix(base_np, P - 1))
    # the rollout part equals the runner call fed the same inputs
    prefix_ids = torch.from_numpy(v[:, :P]).cuda()
    out = r(prefix_ids, ph[:, P - 1:], base[:, P - 1:])
    assert torch.equal(out.cpu(), torch.from_numpy(v[:, P:]))
    teacher_forced_check(oracle_weights(draft, target), prefix_ids, ph[:, P - 1:], base[:, P - 1:], out)


def test_accept_matches_oracle_and_reference_cases():
    from domino_b200 import DraftCorrectionGraphRunner  # noqa: F401  (loads the library)
    from domino_b200 import _lib
    lib = _lib.load()
    fx = load("accept_cases")
    rng = np.random.default_rng(0)
    B, K1 = 64, 16
    v = rng.integers(0, 50, (B, K1))
    p = rng.integers(0, 50, (B, K1))
    for b in range(B):
        a = b % K1
        p[b, :a] = v[b, 1:a + 1]
    cases = [(fx["verify_ids"], fx["posterior"]), (v, p)]
    for vv, pp in cases:
        vt = torch.from_numpy(np.ascontiguousarray(vv)).cuda()
        pt = torch.from_numpy(np.ascontiguousarray(pp)).cuda()
        acc = torch.empty(vt.shape[0], dtype=torch.int32, device="cuda")
        bonus = torch.empty(vt.shape[0], dtype=torch.long, device="cuda")
        _lib.check(lib.dd_accept(vt.data_ptr(), pt.data_ptr(), vt.shape[0], vt.shape[1], acc.data_ptr(),
                                 bonus.data_ptr(), torch.cuda.current_stream().cuda_stream))
        ea, eb = O.accept(vv, pp)
        assert np.array_equal(acc.cpu().numpy(), ea)
        assert np.array_equal(bonus.cpu().numpy(), eb)
    np.testing.assert_array_equal(O.accept(fx["verify_ids"], fx["posterior"])[0], fx["accept"])


def test_bad_prefix_token_sets_status_and_is_clamped():
    B, H, G, E, V, S, P = 2, 64, 64, 96, 700, 15, 1
    draft, target = random_modules(H, G, E, V, seed=41)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=1)
    prefix[0, 0] = V + 5
    r(prefix, ph, base)
    from domino_b200._lib import DD_STATUS_BAD_TOKEN
    assert r.status() & DD_STATUS_BAD_TOKEN
    assert r.status() == 0  # reading the status clears it


def test_spec_generate_trace_replay():
    """Replays the runner calls recorded inside the reference's block loop."""
    fx = load("spec_trace_partial")
    H, V, E, G = 64, 600, 96, 64
    draft, target = random_modules(H, G, E, V, seed=0)
    with torch.no_grad():
        draft.embed_proj[0].weight.copy_(torch.from_numpy(as_f32(fx["fc1"])))
        draft.embed_proj[2].weight.copy_(torch.from_numpy(as_f32(fx["fc2"])))
        draft.prefix_gru.weight_ih_l0.copy_(torch.from_numpy(as_f32(fx["w_ih"])))
        draft.prefix_gru.weight_hh_l0.copy_(torch.from_numpy(as_f32(fx["w_hh"])))
        target.model.embed_tokens.weight.copy_(torch.from_numpy(as_f32(fx["embed"])))
    r = make_runner(draft, target, 1, 15, H, G, V, 1)
    w = oracle_weights(draft, target)
    for i in range(fx["runner_out"].shape[0]):
        prefix = torch.from_numpy(fx["prefix_ids"][i]).cuda()
        ph = torch.from_numpy(as_f32(fx["parallel_hiddens"][i])).cuda().bfloat16()
        base = torch.from_numpy(as_f32(fx["base_logits"][i])).cuda().bfloat16()
        out = r(prefix, ph, base)
        # The trace ran in fp32; rounding the weights to bf16 keeps the
        # all-zero-logit ties (lowest index wins) and the winning row.
        teacher_forced_check(w, prefix, ph, base, out, min_exact=1.0)
        acc, bonus = r.accept(torch.from_numpy(fx["verify_ids"][i]).cuda(), torch.from_numpy(fx["posterior"][i]).cuda())
        assert int(acc[0]) + 1 == int(fx["acceptance_lengths"][i])


@pytest.mark.parametrize("B", [2, 6])  # the per-row (B <= 4) and the butterfly (B > 4) fc2 argmax
def test_nan_logits_win_like_torch_argmax(B):
    """NaN base logits: the draft token is the first NaN's index, as
    torch.argmax returns it (the reference's PyTorch branch, domino.py:409);
    an all-NaN hidden state makes an all-NaN base row, so the pure-draft
    prefix token is 0."""
    H, G, E, V, S, P = 128, 128, 192, 1500, 13, 2
    draft, target = random_modules(H, G, E, V, seed=71 + B, fc2_std=0.08)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=B)
    b = B - 1
    base[b, 4, 900] = float("nan")
    base[b, 4, 333] = float("nan")
    base[0, 6, V - 1] = float("nan")
    out = r(prefix, ph, base)
    assert r.status() == 0
    assert int(out[b, 4]) == 333 and int(out[0, 6]) == V - 1
    K = P - 1 + S
    g = torch.Generator().manual_seed(3)
    ph2 = torch.randn(B, K, H, generator=g).cuda().bfloat16()
    ph2[b, 0, :] = float("nan")
    last = torch.randint(0, V, (B,), generator=g).cuda()
    verify, base_out = r.draft_block(last, ph2)
    assert r.status() == 0
    assert bool(torch.isnan(base_out[b, 0]).all()) and int(verify[b, 1]) == 0


@pytest.mark.parametrize("B,P", [(1, 1), (5, 2), (32, 1)])
def test_fused_cell_matches_separate_cell_exactly(B, P, monkeypatch):
    """The GRU cell run in the fc2 launch's tail (after its grid barrier) and
    the cell in a launch of its own compute the same thing."""
    H, G, E, V, S = 128, 128, 192, 2500, 15
    draft, target = random_modules(H, G, E, V, seed=81 + B, fc2_std=0.08, gru_bias=True)
    monkeypatch.setenv("DD_FUSE_CELL", "0")
    rs = make_runner(draft, target, B, S, H, G, V, P)
    monkeypatch.setenv("DD_FUSE_CELL", "1")
    rf = make_runner(draft, target, B, S, H, G, V, P)
    for seed in range(2):
        prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=seed)
        assert torch.equal(rs(prefix, ph, base), rf(prefix, ph, base))
    K = P - 1 + S
    g = torch.Generator().manual_seed(6)
    ph2 = torch.randn(B, K, H, generator=g).cuda().bfloat16()
    last = torch.randint(0, V, (B,), generator=g).cuda()
    vs, _ = rs.draft_block(last, ph2)
    vf, _ = rf.draft_block(last, ph2)
    assert torch.equal(vs, vf)
    assert rs.status() == 0 and rf.status() == 0


@pytest.mark.parametrize("B,shape,dtype", [
    (B, shape, torch.bfloat16) for B in (6, 20, 32)
    for shape in ("DD_WIDE_PAIR=1", "DD_WIDE_EPI_WARPS=4", "DD_WIDE_TWO_PER_SM=0", "DD_WIDE_ONE_SLOT=1")
] + [(32, "DD_WIDE_PAIR=0", torch.float16), (32, "DD_WIDE_PAIR=1", torch.float16), (6, "DD_WIDE_PAIR=0", torch.float16)])
def test_wide_pass_launch_shapes(B, shape, dtype, monkeypatch):
    """The z / lm_head pass and the table build under each launch shape of
    the wide passes: CTA pairs (M = 256 tiles, cta_group::2), one epilogue
    warpgroup instead of two, one CTA per SM at N <= 128, two one-slot CTAs
    per SM above N = 128.  The lm_head and
    W_z rows make an odd number of 128-row tiles, so the last pair tile has
    an empty half.  Base logits against the oracle's lm_head, tokens by
    teacher forcing, the table against the default launch shape."""
    H, G, E, S, P, V = 128, 128, 320, 15, 2, 4741
    draft, target = random_modules(H, G, E, V, seed=57 + B, fc2_std=0.08, dtype=dtype)
    K = P - 1 + S
    g = torch.Generator().manual_seed(B)
    ph = torch.randn(B, K, H, generator=g).cuda().to(dtype)
    last = torch.randint(0, V, (B,), generator=g).cuda()
    ref_runner = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    name, val = shape.split("=")
    monkeypatch.setenv(name, val)
    r = make_runner(draft, target, B, S, H, G, V, P, use_graph=False)
    tab, tab_ref = r.table.float(), ref_runner.table.float()
    assert torch.all((tab - tab_ref).abs() <= TOL + TOL * tab_ref.abs())
    print(f"{shape} B={B}: table bit-equal to the default launch shape: {torch.equal(r.table, ref_runner.table)}")
    verify, base = r.draft_block(last, ph)
    assert r.status() == 0
    lm = target.lm_head.weight.detach().float().cpu().numpy()
    dt = "fp16" if dtype == torch.float16 else "bf16"
    base_ref = O.lm_head(ph.float().cpu().numpy(), lm, dt)
    base_np = base.float().cpu().numpy()
    assert np.all(np.abs(base_np - base_ref) <= TOL + TOL * np.abs(base_ref))
    v = verify.cpu().numpy()
    assert np.array_equal(v[:, 1:P], O.pure_draft_prefix(base_np, P - 1))
    prefix_ids = torch.from_numpy(v[:, :P]).cuda()
    out = r(prefix_ids, ph[:, P - 1:], base[:, P - 1:])
    assert torch.equal(out.cpu(), torch.from_numpy(v[:, P:]))
    teacher_forced_check(oracle_weights(draft, target, dt), prefix_ids, ph[:, P - 1:], base[:, P - 1:], out)
    r.close()
    ref_runner.close()
