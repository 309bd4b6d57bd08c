"""The batched block loop (domino_b200.spec_decode) and the models around the
draft step (domino_b200.stack), on the CPU, against outputs of the reference
itself (tests/golden/spec_loop_*.npz, written by running its spec_generate,
code/dflash.py:304-526, one prompt at a time).

The CUDA draft step is replaced here by a stand-in with the same two calls,
built on the oracle's torch restatement of the reference's draft step (test
infrastructure); tests/test_gpu_spec_loop.py runs the same loop with the real
runner on the GPU.
"""
import numpy as np
import pytest
import torch

from tests.fixtures import LOOP_CASES, load_loop


class OracleRunner:
    """``draft_block`` / ``verify_accept`` of DraftCorrectionGraphRunner, in torch CPU ops."""

    def __init__(self, draft, target, batch, prefix_len):
        from oracle import torch_branch as TB

        self.tb = TB
        self.head = TB.head_from_modules(draft, target)
        self.batch_size = batch
        self.prefix_len = prefix_len
        self.prefix_token_count = 1 + prefix_len
        self.steps = 15 - prefix_len

    def draft_block(self, last, ph):
        return self.tb.draft_block(self.head, last, ph, self.prefix_len), None

    def verify_accept(self, logits, verify):
        post = torch.argmax(logits, dim=-1)
        acc = (verify[:, 1:] == post[:, :-1]).long().cumprod(1).sum(1)
        return post, acc.int(), post.gather(1, acc[:, None])[:, 0]


def test_target_matches_transformers_qwen3():
    """TargetLM (ragged KV cache) against transformers' Qwen3ForCausalLM with the
    same weights: logits and hidden-state features, prefill then a block."""
    import json

    from transformers import Qwen3Config, Qwen3ForCausalLM

    case = load_loop("spec_loop_random")
    t = case["target"]
    c = json.loads(str(case["fx"]["target_config"]))
    hf_cfg = Qwen3Config(vocab_size=c["vocab_size"], hidden_size=c["hidden_size"],
                         intermediate_size=c["intermediate_size"], num_hidden_layers=c["num_hidden_layers"],
                         num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
                         head_dim=c["head_dim"], rms_norm_eps=c["rms_norm_eps"], max_position_embeddings=512)
    hf_cfg._attn_implementation = "eager"
    hf = Qwen3ForCausalLM(hf_cfg).eval()
    hf.load_state_dict(t.state_dict(), strict=True)
    ids = case["prompts"][0][None]
    with torch.no_grad():
        ref = hf(ids, output_hidden_states=True)
    cache = t.new_cache(1, 64)
    layers = [1, 3]
    logits, feats = t(ids, cache, torch.ones_like(ids, dtype=torch.bool), feature_layers=layers)
    assert torch.allclose(logits, ref.logits, atol=1e-5, rtol=1e-5)
    want = torch.cat([ref.hidden_states[i + 1] for i in layers], -1)  # the last layer's entry is normed
    assert torch.allclose(feats, want, atol=1e-5, rtol=1e-5)
    assert int(cache.length[0]) == ids.shape[1]


@pytest.mark.parametrize("case", LOOP_CASES)
def test_loop_matches_reference_one_and_three_rows(case):
    from domino_b200.spec_decode import spec_generate

    c = load_loop(case)
    draft, target = c["draft"], c["target"]
    P = draft.cfg.pure_draft_prefix_len
    for i, prompt in enumerate(c["prompts"]):
        res = spec_generate(draft, target, OracleRunner(draft, target, 1, P), [prompt], c["max_new_tokens"])
        assert np.array_equal(res.output_ids[0].numpy(), c["outputs"][i]), i
        assert res.acceptance_lengths[0] == c["accepts"][i], i
    res = spec_generate(draft, target, OracleRunner(draft, target, 3, P), c["prompts"], c["max_new_tokens"])
    for i in range(3):
        assert np.array_equal(res.output_ids[i].numpy(), c["outputs"][i]), i
        assert res.acceptance_lengths[i] == c["accepts"][i], i
