"""The batched block loop (domino_b200.spec_decode) with the CUDA draft step
(DraftCorrectionGraphRunner.draft_block, fused verify_accept) against the
reference's own spec_generate outputs (tests/golden/spec_loop_*.npz): output
ids and acceptance lengths per request, one request at a time and three
requests of different lengths in one batch (rows then accept different
numbers of tokens and sit at different positions)."""
import numpy as np
import pytest
import torch

from tests.fixtures import LOOP_CASES, load_loop
from tests.gpu_helpers import log_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


@pytest.mark.parametrize("case", LOOP_CASES)
def test_gpu_loop_matches_reference(case):
    from domino_b200 import DraftCorrectionGraphRunner
    from domino_b200.spec_decode import spec_generate

    c = load_loop(case, device="cuda")
    draft, target = c["draft"], c["target"]
    cfg = draft.cfg
    P = cfg.pure_draft_prefix_len
    dev = torch.device("cuda", 0)

    def runner(B):
        return DraftCorrectionGraphRunner(draft, target, B, 15 - P, cfg.hidden_size, cfg.gru_hidden_dim,
                                          cfg.vocab_size, 1 + P, dev)

    for i, prompt in enumerate(c["prompts"]):
        r = runner(1)
        res = spec_generate(draft, target, r, [prompt], c["max_new_tokens"])
        assert r.status() == 0
        assert np.array_equal(res.output_ids[0].cpu().numpy(), c["outputs"][i]), i
        assert res.acceptance_lengths[0] == c["accepts"][i], i
    r = runner(3)
    res = spec_generate(draft, target, r, c["prompts"], c["max_new_tokens"], time_blocks=True)
    assert r.status() == 0
    for i in range(3):
        assert np.array_equal(res.output_ids[i].cpu().numpy(), c["outputs"][i]), i
        assert res.acceptance_lengths[i] == c["accepts"][i], i
    log_parity(f"{case}: 3 requests in one batch equal the reference's, {res.blocks} blocks, acceptance "
               f"{[sum(a) / len(a) for a in res.acceptance_lengths]}")
