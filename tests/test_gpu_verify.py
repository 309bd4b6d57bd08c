"""Fused target verify + acceptance (dd_verify_accept) against torch.argmax
and the oracle's acceptance (code/dflash.py:472-485): integers, so exact."""
import numpy as np
import pytest
import torch

from oracle import draft_oracle as O
from tests.gpu_helpers import random_modules

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


def _runner(B, V):
    from domino_b200 import DraftCorrectionGraphRunner

    draft, target = random_modules(64, 64, 96, V, seed=V % 97)
    return DraftCorrectionGraphRunner(draft, target, B, 15, 64, 64, V, 1, torch.device("cuda", 0), use_graph=False)


def _case(B, K1, V, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = torch.randn(B, K1, V, generator=g, device="cuda").to(dtype)
    if B > 1:
        logits[1, 3] = 0.5                      # a constant row: every index ties, 0 wins
        logits[1, 4, 17] = logits[1, 4, V - 5] = 50.0  # a duplicated maximum: the lower index wins
    post = torch.argmax(logits.float(), dim=-1)
    verify = torch.randint(0, V, (B, K1), generator=g, device="cuda")
    for b in range(B):
        a = (b * 5) % K1
        verify[b, 1:a + 1] = post[b, :a]
    return logits, verify, post


@pytest.mark.parametrize("V", [5003, 20011, 20016])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_verify_accept_matches_argmax_and_acceptance(V, dtype):
    B, K1 = 4, 16
    r = _runner(B, V)
    for seed in range(2):  # two calls in a row: the scratch clears itself
        logits, verify, post_ref = _case(B, K1, V, dtype, seed)
        post, acc, bonus = r.verify_accept(logits, verify)
        assert r.status() == 0
        assert torch.equal(post, post_ref)
        ea, eb = O.accept(verify.cpu().numpy(), post_ref.cpu().numpy())
        assert np.array_equal(acc.cpu().numpy(), ea)
        assert np.array_equal(bonus.cpu().numpy(), eb)
    r.close()


def test_verify_accept_full_vocab_and_full_acceptance():
    V, B, K1 = 151936, 2, 16
    r = _runner(B, V)
    logits, verify, post_ref = _case(B, K1, V, torch.bfloat16, 5)
    verify[:, 1:] = post_ref[:, :-1]               # the target agrees everywhere
    post, acc, bonus = r.verify_accept(logits, verify)
    assert torch.equal(post, post_ref)
    assert acc.tolist() == [K1 - 1] * B
    assert torch.equal(bonus, post_ref[:, -1])
    r.close()


@pytest.mark.parametrize("V", [20011, 20016])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_verify_accept_nan_ranks_first_like_torch_argmax(dtype, V):
    """A NaN logit wins over every number and the first NaN wins, as in
    torch.argmax (code/dflash.py:472).  The odd V leaves rows unaligned, so
    the scalar head and tail of the vector loop see NaNs too; the even V
    gives 16-byte aligned rows (no scalar head)."""
    B, K1 = 3, 16
    r = _runner(B, V)
    logits, verify, _ = _case(B, K1, V, dtype, 7)
    logits[0, 2, 9000] = float("nan")
    logits[0, 2, 7] = float("nan")          # the first NaN of the row
    logits[1, 5, V - 1] = float("nan")      # last element
    logits[2, 0, 0] = float("inf")
    logits[2, 0, 3] = float("nan")          # NaN above +inf
    logits[2, 7, :] = float("nan")          # all NaN: index 0
    post_ref = torch.argmax(logits.float(), dim=-1)
    post, acc, bonus = r.verify_accept(logits, verify)
    assert r.status() == 0
    assert torch.equal(post, post_ref)
    assert post[0, 2] == 7 and post[1, 5] == V - 1 and post[2, 0] == 3 and post[2, 7] == 0
    assert np.array_equal(post.cpu().numpy(), np.argmax(logits.float().cpu().numpy(), axis=-1))
    r.close()


@pytest.mark.parametrize("V", [20011, 20016])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_verify_accept_signed_zeros_and_infinities(dtype, V):
    """-0 and +0 are equal for torch.argmax, so the first zero wins whatever
    its sign; rows of -inf (all, or all but one) and tied +inf maxima keep
    the first index (code/dflash.py:472)."""
    B, K1 = 2, 16
    r = _runner(B, V)
    _, verify, _ = _case(B, K1, V, dtype, 11)
    logits = torch.full((B, K1, V), -1.0, device="cuda", dtype=dtype)
    logits[0, 0, 100] = -0.0
    logits[0, 0, 50] = 0.0                  # +0 first: 50
    logits[0, 1, 30] = 0.0
    logits[0, 1, 10] = -0.0                 # -0 first: 10, although +0 orders above -0 bitwise
    logits[0, 1, 15000] = -0.0
    logits[0, 2, :] = float("-inf")         # all -inf: 0
    logits[0, 3, :] = float("-inf")
    logits[0, 3, V - 3] = -1.0              # one finite value among -inf
    logits[1, 4, 12000] = float("inf")
    logits[1, 4, 11999] = float("inf")      # tied +inf: 11999
    post_ref = torch.argmax(logits.float(), dim=-1)
    post, _, _ = r.verify_accept(logits, verify)
    assert r.status() == 0
    assert torch.equal(post, post_ref)
    assert post[0, 0] == 50 and post[0, 1] == 10 and post[0, 2] == 0 and post[0, 3] == V - 3
    assert post[1, 4] == 11999
    assert np.array_equal(post.cpu().numpy(), np.argmax(logits.float().cpu().numpy(), axis=-1))
    r.close()


@pytest.mark.parametrize("B,K1", [(1, 1), (1, 16), (3, 5), (32, 64)])
def test_verify_accept_grid_shapes_full_vocab(B, K1):
    """The vocab of a row is cut into as many chunks as one wave of CTAs
    allows: from 1 row (many chunks) to 32 x 64 rows (one chunk per row)."""
    V = 151936
    r = _runner(B, V)
    logits, verify, post_ref = _case(B, K1, V, torch.bfloat16, 13 + B + K1)
    logits[0, K1 - 1, V - 1] = 40.0         # maximum at the last entry of a row
    post_ref = torch.argmax(logits.float(), dim=-1)
    post, acc, bonus = r.verify_accept(logits, verify)
    assert r.status() == 0
    assert torch.equal(post, post_ref)
    ea, eb = O.accept(verify.cpu().numpy(), post_ref.cpu().numpy())
    assert np.array_equal(acc.cpu().numpy(), ea)
    assert np.array_equal(bonus.cpu().numpy(), eb)
    r.close()

