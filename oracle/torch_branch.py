"""The reference's PyTorch branch of the draft step, restated in torch ops.

TEST INFRASTRUCTURE ONLY, never part of the product, in two roles:

* the CPU leg of the benchmark (``bench.py --impl reference`` and the
  ``cpu_baseline`` record): it runs the reference's CPU op sequence (torch's
  bf16 kernels on the host, AMX where the CPU has it), so that the timed CPU
  baseline is as fast as the reference's own code on the same host, which the
  numpy restatement in fp32 (oracle/draft_oracle.py) is not;
* the parity checker of heads whose ``embed_proj`` middle is not a single SiLU:
  for those the reference always takes this branch, so on a GPU these ops (CUDA
  torch kernels) are the reference's own arithmetic.  For SiLU heads the numpy
  oracle, which restates the Triton branch, is the checker.

What it restates, op for op:

* ``_forward_impl``'s PyTorch branch (code/kernel/domino.py:374-431), which
  the reference takes without Triton and, on any device, for a middle that is
  not a single SiLU: ``z = F.linear(hiddens, W_z, b1)`` (381-385);
  ``h = GRU(embed(prefix_ids))`` (387-391); per step ``s = F.linear(h, W_s)``
  (397), ``mid = middle(z_t + s)`` (406-408), ``logits = base_t + F.linear(mid, fc2, b2)`` (409-410),
  ``argmax`` (411), then ``gi = table[token]``, ``gh = F.linear(h, W_hh, b_hh)``
  and the GRU cell with ``tanh`` (418-431);
* the table ``F.linear(embed, W_ih, b_ih)`` (domino.py:322-327), built once;
* ``base_logits = lm_head(parallel_hiddens)`` and the pure-draft prefix
  argmax (code/dflash.py:424-427).

Pinned: its tokens equal the reference's PyTorch-branch tokens recorded in
tests/golden/rollout_*.npz (``tokens_torch``), bit for bit
(tests/test_oracle_golden.py).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn.functional as F


@dataclass
class TorchHead:
    """Host copies of the head, in the model dtype, in the reference's layouts."""

    w_z: torch.Tensor                 # [E, H] = fc1[:, :H]
    w_s: torch.Tensor                 # [E, G] = fc1[:, H:]
    fc2: torch.Tensor                 # [V, E]
    gru: torch.nn.GRU                 # prefix_gru (weights W_ih [3G, H], W_hh [3G, G])
    embed: torch.Tensor               # [V, H] target embed_tokens
    table: torch.Tensor               # [V, 3G] = F.linear(embed, W_ih, b_ih)
    lm_head: Optional[torch.Tensor] = None  # [V, H]
    fc1_bias: Optional[torch.Tensor] = None
    fc2_bias: Optional[torch.Tensor] = None
    middle: Callable = F.silu         # embed_proj's middle module (domino.py:406-408)

    @property
    def w_hh(self):
        return self.gru.weight_hh_l0

    @property
    def b_hh(self):
        return self.gru.bias_hh_l0 if self.gru.bias else None


@torch.inference_mode()
def head_from_modules(draft, target, table: Optional[torch.Tensor] = None, device="cpu") -> TorchHead:
    """A ``TorchHead`` from the reference's modules (code/kernel/domino.py:260-327),
    on the CPU by default.  On a GPU the same ops run the reference's PyTorch
    branch with CUDA torch kernels, which is the reference's own arithmetic for
    a head whose middle is not a single SiLU.

    ``table`` may be given (for example built on a GPU and copied here) to skip
    the one-time ``embed @ W_ih^T`` on the host.
    """
    cpu = torch.device(device)
    fc1, fc2 = draft.embed_proj[0], draft.embed_proj[-1]
    H = target.model.embed_tokens.weight.shape[1]
    gru_src = draft.prefix_gru
    gru = torch.nn.GRU(gru_src.input_size, gru_src.hidden_size, num_layers=1, batch_first=True,
                       bias=gru_src.bias, dtype=gru_src.weight_ih_l0.dtype)
    gru.load_state_dict({k: v.detach().to(cpu) for k, v in gru_src.state_dict().items()})
    gru = gru.to(cpu).eval()
    mods = list(draft.embed_proj.children())
    middle = torch.nn.Sequential(*mods[1:-1]).to(cpu).eval() if len(mods) > 2 else torch.nn.Identity()
    w1 = fc1.weight.detach().to(cpu)
    embed = target.model.embed_tokens.weight.detach().to(cpu)
    if table is None:
        table = F.linear(embed, gru.weight_ih_l0, gru.bias_ih_l0 if gru.bias else None)
    lm = getattr(target, "lm_head", None)
    return TorchHead(
        w_z=w1[:, :H].contiguous(), w_s=w1[:, H:].contiguous(), fc2=fc2.weight.detach().to(cpu), gru=gru,
        embed=embed, table=table.to(cpu).contiguous(),
        lm_head=lm.weight.detach().to(cpu) if lm is not None else None,
        fc1_bias=fc1.bias.detach().to(cpu) if fc1.bias is not None else None,
        fc2_bias=fc2.bias.detach().to(cpu) if fc2.bias is not None else None,
        middle=middle,
    )


@torch.inference_mode()
def rollout(w: TorchHead, prefix_ids: torch.Tensor, parallel_hiddens: torch.Tensor,
            base_logits: torch.Tensor, teacher_tokens: Optional[torch.Tensor] = None, record=None) -> torch.Tensor:
    """[B, 1+p] ids, [B, S, H] hiddens, [B, S, V] base logits -> [B, S] tokens
    (code/kernel/domino.py:374-431, PyTorch branch).

    With ``teacher_tokens`` [B, S] the GRU is fed those tokens instead of the
    argmax (teacher forcing); with ``record`` (a dict) it also records, per
    step, the logit of the fed token and the top logit (``chosen``, ``top``,
    [B, S] fp32) for the near-tie rule of the parity tests."""
    B, S, _ = parallel_hiddens.shape
    dev = parallel_hiddens.device
    z_all = F.linear(parallel_hiddens, w.w_z, w.fc1_bias)                # 381-385
    _, hidden = w.gru(F.embedding(prefix_ids, w.embed))                  # 387-391
    out = torch.zeros(B, S, dtype=torch.long, device=dev)
    chosen = torch.zeros(B, S, device=dev)
    top = torch.zeros(B, S, device=dev)
    for t in range(S):
        h = hidden.squeeze(0)
        s = F.linear(h, w.w_s, None)                                     # 397
        mid = w.middle(z_all[:, t:t + 1, :] + s.unsqueeze(1))            # 406-408
        logits = base_logits[:, t:t + 1, :] + F.linear(mid, w.fc2, w.fc2_bias)  # 409-410
        tok = torch.argmax(logits, dim=-1)                               # 411
        out[:, t:t + 1] = tok
        if teacher_tokens is not None:
            tok = teacher_tokens[:, t:t + 1].to(dev)
        if record is not None:
            top[:, t] = logits.float().amax(-1)[:, 0]
            chosen[:, t] = logits.float()[:, 0].gather(1, tok)[:, 0]
        if t + 1 < S:                                                    # 416-431
            gi = w.table[tok.squeeze(-1)]
            gh = F.linear(h, w.w_hh, w.b_hh)
            g = gi.shape[-1] // 3
            r = torch.sigmoid(gi[:, :g] + gh[:, :g])
            zg = torch.sigmoid(gi[:, g:2 * g] + gh[:, g:2 * g])
            n = torch.tanh(gi[:, 2 * g:] + r * gh[:, 2 * g:])
            hidden = ((1.0 - zg) * n + zg * h).unsqueeze(0)
    if record is not None:
        record["chosen"], record["top"] = chosen, top
    return out


@torch.inference_mode()
def draft_block(w: TorchHead, last_token: torch.Tensor, parallel_hiddens: torch.Tensor, prefix_len: int):
    """The draft side of one block (code/dflash.py:424-439): base logits, the
    pure-draft prefix tokens, the rollout.  Returns verify ids [B, K + 1]."""
    base = F.linear(parallel_hiddens, w.lm_head)                         # dflash.py:424
    ids = [last_token.reshape(-1, 1)]
    if prefix_len > 0:
        ids.append(torch.argmax(base[:, :prefix_len], dim=-1))           # dflash.py:425-427
    prefix = torch.cat(ids, 1)
    toks = rollout(w, prefix, parallel_hiddens[:, prefix_len:], base[:, prefix_len:])
    return torch.cat([prefix, toks], 1)
