"""fp32 PyTorch restatement of the draft step, for full-size parity checks on
the GPU (the numpy oracle restates the same arithmetic; at V = 151936 and
E = 12288 it is too slow to run per test).  Test infrastructure only.

Same rounding points as oracle/draft_oracle.py (the reference's Triton
branch, code/kernel/domino.py:374-431): linear outputs and GRU states rounded
to bf16, the correction step and the GRU cell in fp32.
"""
from __future__ import annotations

import torch


_ROUND = [True]  # False: fp32 heads, nothing is rounded (set by teacher_forced_rollout)


def _rb(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float() if _ROUND[0] else x.float()


def _linear(x, w, b=None):
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return _rb(y)


def _cell(gi, gh, h):
    G = h.shape[-1]
    r = torch.sigmoid(gi[:, :G] + gh[:, :G])
    z = torch.sigmoid(gi[:, G:2 * G] + gh[:, G:2 * G])
    n = 2.0 * torch.sigmoid(2.0 * (gi[:, 2 * G:] + r * gh[:, 2 * G:])) - 1.0
    return _rb((1.0 - z) * n + z * h)


@torch.no_grad()
def build_table(embed, w_ih, b_ih=None):
    """The GRU input table ``F.linear(embed, W_ih, b_ih)`` (code/kernel/domino.py:322-327),
    computed here by cuBLAS in the weight dtype, independently of the kernel under test."""
    return torch.nn.functional.linear(embed, w_ih, b_ih).contiguous()


@torch.no_grad()
def teacher_forced_rollout(fc1, fc2, w_hh, table, prefix_ids, parallel_hiddens, base_logits, tokens,
                           fc1_bias=None, fc2_bias=None, b_hh=None, states=None, round_bf16=True):
    """Own argmax, logit of the fed token and top logit per step, fed ``tokens``.

    fc1 [E, H+G], fc2 [V, E], w_hh [3G, G], table [V, 3G] (bf16 tensors on the
    GPU); prefix_ids [B, P]; parallel_hiddens [B, S, H]; base_logits [B, S, V];
    tokens [B, S] (the tokens under test).  With ``states`` (a dict) it also
    records the per-step states in the layout of the runner's ``rollout_trace``:
    ``z`` [B, S, E], ``h`` [P + S - 1, B, G], ``gh`` [P + S - 2, B, 3G],
    ``s`` [S, B, E] (fp32 tensors holding bf16-rounded values).  With
    ``round_bf16=False`` nothing is rounded (fp32 heads).
    """
    _ROUND[0] = round_bf16
    B, S, H = parallel_hiddens.shape
    G = w_hh.shape[1]
    P = prefix_ids.shape[1]
    fc2_f = fc2.float()
    z = _linear(parallel_hiddens.reshape(B * S, H), fc1[:, :H], fc1_bias).reshape(B, S, -1)
    w_s = fc1[:, H:]
    hs, ghs, ss = [], [], []
    h = torch.zeros(B, G, device=fc1.device)
    for j in range(P):
        gi = table[prefix_ids[:, j]].float()
        gh = _linear(h, w_hh, b_hh)
        if j > 0:
            ghs.append(gh)
        h = _cell(gi, gh, h)
        hs.append(h)
    own = torch.zeros(B, S, dtype=torch.long, device=fc1.device)
    chosen = torch.zeros(B, S, device=fc1.device)
    top = torch.zeros(B, S, device=fc1.device)
    for t in range(S):
        s = _linear(h, w_s)
        ss.append(s)
        pre = z[:, t] + s
        mid = pre * torch.sigmoid(pre)
        logits = mid @ fc2_f.t()
        if fc2_bias is not None:
            logits = logits + fc2_bias.float()
        logits = logits + base_logits[:, t].float()
        own[:, t] = torch.argmax(logits, dim=-1)
        top[:, t] = logits.gather(1, own[:, t:t + 1]).squeeze(1)
        chosen[:, t] = logits.gather(1, tokens[:, t:t + 1]).squeeze(1)
        if t + 1 < S:
            gi = table[tokens[:, t]].float()
            gh = _linear(h, w_hh, b_hh)
            ghs.append(gh)
            h = _cell(gi, gh, h)
            hs.append(h)
    if states is not None:
        states["z"] = z
        states["h"] = torch.stack(hs)
        states["gh"] = torch.stack(ghs) if ghs else torch.zeros(0, B, 3 * G, device=fc1.device)
        states["s"] = torch.stack(ss)
    return own, chosen, top
