"""Generate the golden fixtures under tests/golden/ by running the reference.

Run where a checkout of the reference (jianuo-huang/Domino) is available,
naming its root in ``DOMINO_REFERENCE`` (required); the fixtures it writes are
committed, so nothing else needs the reference at run time.

    DOMINO_REFERENCE=/path/to/Domino python tests/golden/make_golden.py

What it runs, all on CPU:

* ``DraftCorrectionGraphRunner`` (code/kernel/domino.py:229-508) unchanged,
  with ``torch.cuda.Stream/stream/CUDAGraph/graph`` replaced by no-op shims so
  that its warm-up/capture code runs without a GPU and ``graph.replay()``
  calls ``_forward_impl``.
  - Triton branch: its three ``@triton.jit`` kernels under
    ``TRITON_INTERPRET=1`` (the reference's own fp32 numerics);
  - PyTorch branch: the same runner with ``HAS_TRITON = False``.
  The runner's ``_fused_step_triton`` / ``_fused_gru_cell`` methods and the
  prefix ``nn.GRU`` are wrapped to record their inputs and outputs
  (h0, s_proj, gi, gh, h per step).
* ``DFlashDraftModel.spec_generate`` (code/dflash.py:304-526) with a tiny
  random ``Qwen3ForCausalLM`` target, with the runner plugged in as
  ``graph_runner``; every runner call and every verify step is recorded.
* The acceptance expression of code/dflash.py:473-478 on synthetic
  (verify_ids, posterior) pairs.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")
if not os.environ.get("DOMINO_REFERENCE"):
    sys.exit("set DOMINO_REFERENCE to the root of a Domino checkout (the directory holding code/)")
REF = Path(os.environ["DOMINO_REFERENCE"]) / "code"
OUT = Path(__file__).resolve().parent

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn as nn  # noqa: E402

sys.path.insert(0, str(REF))
import transformers  # noqa: E402,F401  (import before the shims below)
import kernel.domino as kd  # noqa: E402


# --------------------------------------------------------------------------
# CUDA stream / graph shims so the reference runner constructs on CPU
# --------------------------------------------------------------------------
class _Stream:
    def __init__(self, *a, **k):
        pass

    def wait_stream(self, *a, **k):
        pass


class _Graph:
    def __init__(self):
        self.fn = None

    def replay(self):
        self.fn()


class _Ctx:
    def __init__(self, *a, **k):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


torch.cuda.Stream = _Stream
torch.cuda.current_stream = lambda *a, **k: _Stream()
torch.cuda.stream = _Ctx
torch.cuda.CUDAGraph = _Graph
torch.cuda.graph = _Ctx


class TinyDraftHead(nn.Module):
    """Just the two head modules the runner reads (dflash.py:261-274)."""

    def __init__(self, H, G, E, V, fc1_bias, fc2_bias, gru_bias):
        super().__init__()
        self.prefix_gru = nn.GRU(H, G, num_layers=1, batch_first=True, bias=gru_bias)
        self.embed_proj = nn.Sequential(
            nn.Linear(H + G, E, bias=fc1_bias), nn.SiLU(), nn.Linear(E, V, bias=fc2_bias)
        )


class TinyTarget(nn.Module):
    def __init__(self, H, V):
        super().__init__()
        self.model = nn.Module()
        self.model.embed_tokens = nn.Embedding(V, H)
        self.lm_head = nn.Linear(H, V, bias=False)


def _np(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy, bf16 as uint16 bit patterns, everything else as is."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _make_runner(draft, target, B, S, H, G, V, P, triton: bool):
    kd.HAS_TRITON = triton
    r = kd.DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cpu"))
    r.graph.fn = r._forward_impl
    return r


def _instrument(r):
    rec = {"s_proj": [], "tok": [], "gi": [], "gh": [], "h_in": [], "h_out": [], "h0": []}
    step = r._fused_step_triton
    cell = r._fused_gru_cell

    def step_w(z, s, base):
        out = step(z, s, base)
        rec["s_proj"].append(s.clone())
        rec["tok"].append(out.clone())
        return out

    def cell_w(gi, gh, h, h_out):
        cell(gi, gh, h, h_out)
        rec["gi"].append(gi.clone())
        rec["gh"].append(gh.clone())
        rec["h_in"].append(h.clone())
        rec["h_out"].append(h_out.clone())

    def gru_hook(mod, inp, out):
        rec["h0"].append(out[1].squeeze(0).clone())

    r._fused_step_triton = step_w
    r._fused_gru_cell = cell_w
    hook = r.draft_model.prefix_gru.register_forward_hook(gru_hook)
    return rec, hook


def rollout_case(name, *, seed, B, H, G, E, V, S, P, dtype, fc1_bias=False, fc2_bias=False, gru_bias=False):
    torch.manual_seed(seed)
    draft = TinyDraftHead(H, G, E, V, fc1_bias, fc2_bias, gru_bias)
    target = TinyTarget(H, V)
    with torch.no_grad():
        for p in list(draft.parameters()) + list(target.parameters()):
            p.normal_(0.0, 0.02 if p.dim() == 2 else 0.05)
        target.model.embed_tokens.weight.normal_(0.0, 1.0)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    draft = draft.to(tdt)
    target = target.to(tdt)
    prefix_ids = torch.randint(0, V, (B, P))
    ph = torch.randn(B, S, H).to(tdt)
    with torch.no_grad():
        base = target.lm_head(ph)                    # dflash.py:424
    data = {}
    r_tri = _make_runner(draft, target, B, S, H, G, V, P, triton=True)
    rec, hook = _instrument(r_tri)
    out_tri = r_tri(prefix_ids, ph, base)
    hook.remove()
    r_pt = _make_runner(draft, target, B, S, H, G, V, P, triton=False)
    out_pt = r_pt(prefix_ids, ph, base)
    data.update(
        meta=np.array([B, H, G, E, V, S, P, int(fc1_bias), int(fc2_bias), int(gru_bias)], np.int64),
        dtype=np.array(dtype),
        fc1=_np(draft.embed_proj[0].weight),
        fc2=_np(draft.embed_proj[2].weight),
        w_ih=_np(draft.prefix_gru.weight_ih_l0),
        w_hh=_np(draft.prefix_gru.weight_hh_l0),
        embed=_np(target.model.embed_tokens.weight),
        lm_head=_np(target.lm_head.weight),
        table=_np(r_tri._gru_input_proj_table),
        prefix_ids=prefix_ids.numpy(),
        parallel_hiddens=_np(ph),
        base_logits=_np(base),
        tokens_triton=out_tri.numpy(),
        tokens_torch=out_pt.numpy(),
        z_part=_np(torch.nn.functional.linear(ph, r_tri.w_z, r_tri.fc1_bias)),
        h0=_np(rec["h0"][0]),
        s_proj=np.stack([_np(x) for x in rec["s_proj"]], 1),
        gh=np.stack([_np(x) for x in rec["gh"]], 1),
        h_out=np.stack([_np(x) for x in rec["h_out"]], 1),
    )
    if fc1_bias:
        data["fc1_bias"] = _np(draft.embed_proj[0].bias)
    if fc2_bias:
        data["fc2_bias"] = _np(draft.embed_proj[2].bias)
    if gru_bias:
        data["b_ih"] = _np(draft.prefix_gru.bias_ih_l0)
        data["b_hh"] = _np(draft.prefix_gru.bias_hh_l0)
    np.savez_compressed(OUT / f"{name}.npz", **data)
    agree = (out_tri == out_pt).float().mean().item()
    print(f"{name}: triton vs torch-branch token agreement {agree:.3f}")


def middle_case(name, *, seed, B, H, G, E, V, S, P, middle: str):
    """A head whose embed_proj middle is not a single SiLU: the reference's
    runner then takes its PyTorch branch (code/kernel/domino.py:406-431) on
    any device.  Records the weights, the inputs and its tokens."""
    torch.manual_seed(seed)
    draft = TinyDraftHead(H, G, E, V, False, False, False)
    if middle == "identity":
        draft.embed_proj = nn.Sequential(draft.embed_proj[0], draft.embed_proj[2])
    else:
        draft.embed_proj[1] = {"gelu": nn.GELU(), "relu": nn.ReLU(), "tanh": nn.Tanh()}[middle]
    target = TinyTarget(H, V)
    with torch.no_grad():
        for p in list(draft.parameters()) + list(target.parameters()):
            p.normal_(0.0, 0.02 if p.dim() == 2 else 0.05)
        target.model.embed_tokens.weight.normal_(0.0, 1.0)
        draft.embed_proj[-1].weight.normal_(0.0, 0.1)  # a correction large enough to move the argmax
    draft, target = draft.to(torch.bfloat16), target.to(torch.bfloat16)
    prefix_ids = torch.randint(0, V, (B, P))
    ph = torch.randn(B, S, H).to(torch.bfloat16)
    with torch.no_grad():
        base = target.lm_head(ph)
    r = _make_runner(draft, target, B, S, H, G, V, P, triton=True)
    assert not r._can_triton_fuse, "a non-SiLU middle must take the PyTorch branch"
    out = r(prefix_ids, ph, base)
    np.savez_compressed(
        OUT / f"{name}.npz",
        meta=np.array([B, H, G, E, V, S, P, 0, 0, 0], np.int64), dtype=np.array("bf16"), middle=np.array(middle),
        fc1=_np(draft.embed_proj[0].weight), fc2=_np(draft.embed_proj[-1].weight),
        w_ih=_np(draft.prefix_gru.weight_ih_l0), w_hh=_np(draft.prefix_gru.weight_hh_l0),
        embed=_np(target.model.embed_tokens.weight), lm_head=_np(target.lm_head.weight),
        prefix_ids=prefix_ids.numpy(), parallel_hiddens=_np(ph), base_logits=_np(base),
        tokens_torch=out.numpy(),
    )
    print(f"{name}: PyTorch-branch tokens {out.tolist()}")


def accept_case():
    """Synthetic (verify_ids, posterior) pairs through dflash.py:473-484."""
    g = torch.Generator().manual_seed(7)
    rows = []
    K = 15
    for a in list(range(K + 1)) + [0, 3, 15, 7, 1]:
        verify = torch.randint(0, 1000, (1, K + 1), generator=g)
        posterior = torch.randint(0, 1000, (1, K + 1), generator=g)
        posterior[0, :a] = verify[0, 1:a + 1]
        if a < K:
            posterior[0, a] = (verify[0, a + 1] + 1) % 1000
        rows.append((verify, posterior))
    verify = torch.cat([v for v, _ in rows])
    posterior = torch.cat([p for _, p in rows])
    acc, bonus = [], []
    for i in range(verify.shape[0]):
        v, p = verify[i:i + 1], posterior[i:i + 1]
        acceptance_length = (v[:, 1:] == p[:, :-1]).cumprod(dim=1).sum(dim=1)[0].item()
        acc.append(acceptance_length)
        bonus.append(p[:, acceptance_length].item())
    np.savez_compressed(
        OUT / "accept_cases.npz",
        verify_ids=verify.numpy(),
        posterior=posterior.numpy(),
        accept=np.array(acc, np.int32),
        bonus=np.array(bonus, np.int64),
    )
    print("accept_cases:", acc)


def spec_generate_trace(name, *, seed, mode: str, max_new_tokens: int):
    """Record the runner's calls inside the reference's own block loop.

    mode "random": random heads, acceptance is almost always 0.
    mode "full":   target logits are all zero (posterior = token 0 everywhere)
                   and the draft's base logits and fc2 are zero, so every
                   draft logit ties at 0 and the lowest index (0) wins: the
                   whole block is accepted.
    mode "partial": as "full" but one fc2 row is non-zero, so that row wins
                   at the steps where its correction bias is positive and the
                   block is accepted up to the first such step.
    """
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from dflash import DFlashDraftModel

    torch.manual_seed(seed)
    H, V, E, G = 64, 600, 96, 64
    tcfg = Qwen3Config(
        vocab_size=V, hidden_size=H, intermediate_size=128, num_hidden_layers=4,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=512,
    )
    tcfg._attn_implementation = "eager"
    target = Qwen3ForCausalLM(tcfg).eval()
    dcfg = Qwen3Config(
        vocab_size=V, hidden_size=H, intermediate_size=128, num_hidden_layers=1,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=512,
    )
    dcfg._attn_implementation = "eager"
    dcfg.block_size = 16
    dcfg.num_target_layers = 4
    dcfg.dflash_config = {
        "projector_type": "domino", "emb_dim": E, "gru_hidden_dim": G,
        "mask_token_id": V - 1, "pure_draft_prefix_len": 0, "target_layer_ids": [1],
    }
    draft = DFlashDraftModel(dcfg).eval()
    with torch.no_grad():
        for p in draft.embed_proj.parameters():
            p.normal_(0.0, 0.02)
        for p in draft.prefix_gru.parameters():
            p.normal_(0.0, 0.05)
        if mode in ("full", "partial"):
            target.model.norm.weight.zero_()
            draft.norm.weight.zero_()
            draft.embed_proj[2].weight.zero_()
        if mode == "partial":
            draft.embed_proj[2].weight[5].normal_(0.0, 0.5)
    kd.HAS_TRITON = True
    runner = kd.DraftCorrectionGraphRunner(draft, target, 1, 15, H, G, V, 1, torch.device("cpu"))
    runner.graph.fn = runner._forward_impl
    calls = []
    orig_call = runner.__call__

    class Rec:
        def __call__(self, prefix_ids, ph, base):
            out = orig_call(prefix_ids, ph, base)
            calls.append((prefix_ids.clone(), ph.clone(), base.clone(), out.clone()))
            return out

    verifies = []
    orig_fwd = target.forward

    def fwd(input_ids=None, **kw):
        out = orig_fwd(input_ids=input_ids, **kw)
        if input_ids is not None and input_ids.shape[1] == 16:
            verifies.append((input_ids.clone(), torch.argmax(out.logits, dim=-1).clone()))
        return out

    target.forward = fwd
    prompt = torch.randint(0, V - 1, (1, 24))
    res = draft.spec_generate(
        prompt, target, max_new_tokens=max_new_tokens, temperature=0.0, block_size=16,
        graph_runner=Rec(), return_dict=True,
    )
    n = len(calls)
    assert n == len(verifies), (n, len(verifies))
    np.savez_compressed(
        OUT / f"{name}.npz",
        fc1=_np(draft.embed_proj[0].weight), fc2=_np(draft.embed_proj[2].weight),
        w_ih=_np(draft.prefix_gru.weight_ih_l0), w_hh=_np(draft.prefix_gru.weight_hh_l0),
        embed=_np(target.model.embed_tokens.weight),
        prefix_ids=np.stack([c[0].numpy() for c in calls]),
        parallel_hiddens=np.stack([_np(c[1]) for c in calls]),
        base_logits=np.stack([_np(c[2]) for c in calls]),
        runner_out=np.stack([c[3].numpy() for c in calls]),
        verify_ids=np.stack([v[0].numpy() for v in verifies]),
        posterior=np.stack([v[1].numpy() for v in verifies]),
        acceptance_lengths=np.array(res.acceptance_lengths, np.int64),
        output_ids=res.output_ids.numpy(),
    )
    print(f"{name}: {n} blocks, acceptance lengths {res.acceptance_lengths}")


def _config_json(cfg) -> str:
    """The Qwen3 config fields a Qwen3-style stack needs, as JSON."""
    import json

    rope = getattr(cfg, "rope_parameters", None) or {}
    d = dict(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
             num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
             num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps,
             rope_theta=float(rope.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))))
    dc = getattr(cfg, "dflash_config", None)
    if dc:
        d.update(block_size=cfg.block_size, target_layer_ids=list(dc["target_layer_ids"]),
                 mask_token_id=dc["mask_token_id"], emb_dim=dc["emb_dim"], gru_hidden_dim=dc["gru_hidden_dim"],
                 pure_draft_prefix_len=dc.get("pure_draft_prefix_len", 0))
    return json.dumps(d)


def spec_loop_case(name, *, seed, mode: str, prompt_lens, max_new_tokens: int, draft_layers: int = 1,
                   target_layer_ids=(1,), prefix_len: int = 0):
    """The reference's whole spec_generate (code/dflash.py:304-526) for several
    prompts, one call each (it is batch-1 only), with every parameter of the
    tiny target and drafter saved so that another implementation of the loop
    can be checked against its outputs and acceptance lengths.

    Modes as in spec_generate_trace: "random" heads (acceptance mostly 1);
    "partial" (zero target logits, one live fc2 row); "full" (every draft
    token accepted); "varied" (see below: acceptance varies per block and per
    prompt).
    """
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from dflash import DFlashDraftModel

    torch.manual_seed(seed)
    H, V, E, G = 64, 600, 96, 64
    tcfg = Qwen3Config(
        vocab_size=V, hidden_size=H, intermediate_size=128, num_hidden_layers=4,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=512,
    )
    tcfg._attn_implementation = "eager"
    target = Qwen3ForCausalLM(tcfg).eval()
    dcfg = Qwen3Config(
        vocab_size=V, hidden_size=H, intermediate_size=128, num_hidden_layers=draft_layers,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=512,
    )
    dcfg._attn_implementation = "eager"
    dcfg.block_size = 16
    dcfg.num_target_layers = 4
    dcfg.dflash_config = {
        "projector_type": "domino", "emb_dim": E, "gru_hidden_dim": G, "mask_token_id": V - 1,
        "pure_draft_prefix_len": prefix_len, "target_layer_ids": list(target_layer_ids),
    }
    draft = DFlashDraftModel(dcfg).eval()
    with torch.no_grad():
        for p in draft.embed_proj.parameters():
            p.normal_(0.0, 0.02)
        for p in draft.prefix_gru.parameters():
            p.normal_(0.0, 0.05)
        if mode in ("full", "partial"):
            target.model.norm.weight.zero_()
            draft.norm.weight.zero_()
            draft.embed_proj[2].weight.zero_()
        if mode == "partial":
            draft.embed_proj[2].weight[5].normal_(0.0, 0.5)
        if mode == "varied":
            # zero target lm_head: posterior 0 everywhere and base logits 0;
            # the drafter's hidden states stay live, so the sign of token 5's
            # correction (the one live fc2 row) changes from position to
            # position and row to row, and so does the acceptance
            target.lm_head.weight.zero_()
            draft.embed_proj[2].weight.zero_()
            row = torch.randn(E) * 0.5
            draft.embed_proj[2].weight[5] = row - row.mean()  # zero-mean: the sign follows mid's fluctuations
            draft.embed_proj[0].weight[:, :H] *= 20.0  # a large z part: mid moves with the block's hidden states
    kd.HAS_TRITON = True
    S = 15 - prefix_len
    runner = kd.DraftCorrectionGraphRunner(draft, target, 1, S, H, G, V, 1 + prefix_len, torch.device("cpu"))
    runner.graph.fn = runner._forward_impl
    data = {"target_config": np.array(_config_json(tcfg)), "draft_config": np.array(_config_json(dcfg)),
            "max_new_tokens": np.array(max_new_tokens)}
    for k, v in target.state_dict().items():
        data["t." + k] = v.detach().numpy()
    for k, v in draft.state_dict().items():
        data["d." + k] = v.detach().numpy()
    accs = []
    for i, n in enumerate(prompt_lens):
        prompt = torch.randint(0, V - 1, (1, n))
        res = draft.spec_generate(prompt, target, max_new_tokens=max_new_tokens, temperature=0.0, block_size=16,
                                  graph_runner=runner, return_dict=True)
        data[f"prompt_{i}"] = prompt[0].numpy()
        data[f"output_{i}"] = res.output_ids[0].numpy()
        data[f"accept_{i}"] = np.array(res.acceptance_lengths, np.int64)
        accs.append(res.acceptance_lengths)
    data["n_prompts"] = np.array(len(prompt_lens))
    np.savez_compressed(OUT / f"{name}.npz", **data)
    print(f"{name}: acceptance lengths per prompt {accs}")


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    with torch.inference_mode():
        rollout_case("rollout_bf16_b1", seed=1, B=1, H=64, G=64, E=96, V=600, S=15, P=1, dtype="bf16")
        rollout_case("rollout_bf16_b3_bias", seed=2, B=3, H=64, G=48, E=80, V=600, S=13, P=3,
                     dtype="bf16", fc1_bias=True, fc2_bias=True, gru_bias=True)
        rollout_case("rollout_fp32_b1", seed=3, B=1, H=64, G=64, E=96, V=600, S=15, P=1, dtype="fp32")
        accept_case()
        middle_case("middle_gelu_b2", seed=11, B=2, H=64, G=64, E=96, V=600, S=15, P=1, middle="gelu")
        middle_case("middle_identity_b2", seed=12, B=2, H=64, G=48, E=80, V=600, S=13, P=2, middle="identity")
    spec_generate_trace("spec_trace_random", seed=4, mode="random", max_new_tokens=10)
    spec_generate_trace("spec_trace_full_accept", seed=5, mode="full", max_new_tokens=40)
    spec_generate_trace("spec_trace_partial", seed=38, mode="partial", max_new_tokens=20)
    loops = dict(prompt_lens=(24, 13, 31))
    spec_loop_case("spec_loop_random", seed=6, mode="random", max_new_tokens=24, draft_layers=2,
                   target_layer_ids=(1, 2), prefix_len=1, **loops)
    spec_loop_case("spec_loop_varied", seed=38, mode="varied", max_new_tokens=48, **loops)
    spec_loop_case("spec_loop_full", seed=5, mode="full", max_new_tokens=40, **loops)


if __name__ == "__main__":
    main()
