"""CPU oracle for the Domino per-block draft step.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product (``domino_b200``) never imports, links or calls anything here.

It restates, in numpy, the arithmetic of the reference's draft-correction
runner (``code/kernel/domino.py``) along the Triton branch, which is the path
the reference's CUDA-graph runner takes on a GPU:

* ``F.linear`` outputs (``z_part``, ``s_proj``, ``gh``, the ``W_ih`` table,
  ``lm_head``) are rounded to the model dtype (bf16 for Domino checkpoints),
  code/kernel/domino.py:381-385, 397, 420, 325-327; code/dflash.py:424.
* The correction step accumulates ``sum_m fc2[v,m] * SiLU(z[m] + s[m])`` in
  fp32 from the dtype-rounded ``z``/``s``, adds ``fc2_bias`` and the base
  logits in fp32 and takes the argmax with the lowest index winning ties,
  code/kernel/domino.py:58-170.
* The GRU cell runs in fp32 from dtype-rounded ``gi``/``gh``/``h`` and stores
  the new state in the model dtype; ``tanh(x)`` is written ``2*sigmoid(2x)-1``
  exactly as code/kernel/domino.py:217-226 does.
* The prefix GRU over ``prefix_ids`` (code/kernel/domino.py:387-391, which
  calls ``nn.GRU`` on ``embed_tokens(prefix_ids)``) is restated with the same
  cell and the precomputed ``embed @ W_ih^T`` table, so it agrees with the
  reference's ``nn.GRU`` to within bf16 rounding (checked against the golden
  fixtures with atol/rtol 2e-2).
* Greedy acceptance follows code/dflash.py:472-487.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by running the reference itself
(``tests/golden/make_golden.py``).

Weights are passed as float32 numpy arrays whose values are already
representable in the model dtype; ``dtype`` selects where results are rounded
("bf16", "fp16" or "fp32" = no rounding).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

__all__ = [
    "round_to",
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "linear",
    "silu",
    "sigmoid",
    "gru_cell",
    "build_table",
    "prefix_gru",
    "correction_logits",
    "argmax_lowest",
    "top2_gap",
    "DraftWeights",
    "RolloutTrace",
    "rollout",
    "lm_head",
    "pure_draft_prefix",
    "accept",
    "orderable_key",
    "packed_argmax_key",
]


# ----------------------------------------------------------------------------
# dtype rounding
# ----------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round-to-nearest-even, NaN kept quiet."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), out)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> fp32 values (exact)."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` and return them as fp32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


# ----------------------------------------------------------------------------
# elementwise pieces
# ----------------------------------------------------------------------------

def sigmoid(x: np.ndarray) -> np.ndarray:
    """fp32 logistic, 1 / (1 + exp(-x)) (Triton's ``tl.sigmoid``)."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    """``preact * sigmoid(preact)`` in fp32, code/kernel/domino.py:95-96."""
    x = np.asarray(x, dtype=np.float32)
    return (x * sigmoid(x)).astype(np.float32)


def linear(x: np.ndarray, w: np.ndarray, b: Optional[np.ndarray], dtype: str) -> np.ndarray:
    """``F.linear(x, w, b)`` with an fp32 accumulator and a ``dtype`` result.

    The products of two bf16 values are exact in fp32; the sum order differs
    from cuBLAS only in the last fp32 bits, which the tolerances absorb.
    """
    y = np.asarray(x, dtype=np.float32) @ np.asarray(w, dtype=np.float32).T
    if b is not None:
        y = y + np.asarray(b, dtype=np.float32)
    return round_to(y, dtype)


def gru_cell(gi: np.ndarray, gh: np.ndarray, h: np.ndarray, dtype: str) -> np.ndarray:
    """Fused GRU cell, code/kernel/domino.py:172-226.

    ``gi``/``gh`` are ``[..., 3G]`` with PyTorch's (r, z, n) gate order and
    already include their biases; math in fp32, the new state is rounded to
    the state dtype (``h_new.to(h_ptr.dtype.element_ty)``, domino.py:226).
    """
    gi = np.asarray(gi, dtype=np.float32)
    gh = np.asarray(gh, dtype=np.float32)
    h = np.asarray(h, dtype=np.float32)
    G = h.shape[-1]
    i_r, i_z, i_n = gi[..., :G], gi[..., G:2 * G], gi[..., 2 * G:]
    h_r, h_z, h_n = gh[..., :G], gh[..., G:2 * G], gh[..., 2 * G:]
    r = sigmoid(i_r + h_r)
    z = sigmoid(i_z + h_z)
    n = np.float32(2.0) * sigmoid(np.float32(2.0) * (i_n + r * h_n)) - np.float32(1.0)
    h_new = (np.float32(1.0) - z) * n + z * h
    return round_to(h_new, dtype)


# ----------------------------------------------------------------------------
# argmax helpers
# ----------------------------------------------------------------------------

def argmax_lowest(x: np.ndarray) -> np.ndarray:
    """Argmax over the last axis; ties go to the lowest index.

    ``torch.argmax`` and the reference's two-level Triton reduction (strict
    ``>`` across 512-wide partials, domino.py:166) both return the first
    maximum, as does ``np.argmax``.
    """
    return np.argmax(np.asarray(x, dtype=np.float32), axis=-1)


def top2_gap(x: np.ndarray) -> np.ndarray:
    """``max - second max`` over the last axis (0 when the top value repeats)."""
    x = np.asarray(x, dtype=np.float32)
    part = np.partition(x, -2, axis=-1)
    return (part[..., -1] - part[..., -2]).astype(np.float32)


def orderable_key(v: np.ndarray) -> np.ndarray:
    """Map fp32 to uint32 so that unsigned order equals float order."""
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)


def packed_argmax_key(v: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """64-bit key whose unsigned max is the (value, lowest index) argmax.

    High word: order-preserving image of the fp32 logit, and the top value
    for a NaN of either sign (``torch.argmax`` and ``np.argmax`` rank NaN
    above every number and return the first one, code/dflash.py:472); low
    word: ``0xFFFFFFFF - idx`` so that, among equal values, the lowest index
    wins.  This is the word the GPU kernels combine with ``atomicMax``.
    """
    v = np.asarray(v, dtype=np.float32)
    hi32 = np.where(np.isnan(v), np.uint32(0xFFFFFFFF), orderable_key(v)).astype(np.uint32)
    hi = hi32.astype(np.uint64) << np.uint64(32)
    lo = (np.uint64(0xFFFFFFFF) - np.asarray(idx, dtype=np.uint64)) & np.uint64(0xFFFFFFFF)
    return hi | lo


# ----------------------------------------------------------------------------
# weights
# ----------------------------------------------------------------------------

@dataclass
class DraftWeights:
    """Correction-head parameters, in the reference's layouts.

    fc1   [E, H+G]   ``embed_proj[0].weight``; split into W_z = fc1[:, :H],
                     W_s = fc1[:, H:] (domino.py:272-273)
    fc2   [V, E]     ``embed_proj[-1].weight`` (domino.py:276)
    w_ih  [3G, H]    ``prefix_gru.weight_ih_l0`` (domino.py:317)
    w_hh  [3G, G]    ``prefix_gru.weight_hh_l0`` (domino.py:318)
    embed [V, H]     ``target.model.embed_tokens.weight`` (domino.py:324)
    """

    fc1: np.ndarray
    fc2: np.ndarray
    w_ih: np.ndarray
    w_hh: np.ndarray
    embed: np.ndarray
    dtype: str = "bf16"
    fc1_bias: Optional[np.ndarray] = None
    fc2_bias: Optional[np.ndarray] = None
    b_ih: Optional[np.ndarray] = None
    b_hh: Optional[np.ndarray] = None
    table: Optional[np.ndarray] = None

    @property
    def H(self) -> int:
        return self.embed.shape[1]

    @property
    def G(self) -> int:
        return self.w_hh.shape[1]

    @property
    def E(self) -> int:
        return self.fc1.shape[0]

    @property
    def V(self) -> int:
        return self.fc2.shape[0]

    @property
    def w_z(self) -> np.ndarray:
        return self.fc1[:, : self.H]

    @property
    def w_s(self) -> np.ndarray:
        return self.fc1[:, self.H:]

    def get_table(self) -> np.ndarray:
        if self.table is None:
            self.table = build_table(self.embed, self.w_ih, self.b_ih, self.dtype)
        return self.table


def build_table(embed: np.ndarray, w_ih: np.ndarray, b_ih: Optional[np.ndarray], dtype: str) -> np.ndarray:
    """GRU input table ``F.linear(embed, W_ih, b_ih)`` -> [V, 3G], domino.py:322-327."""
    return linear(embed, w_ih, b_ih, dtype)


def prefix_gru(w: DraftWeights, prefix_ids: np.ndarray, states: Optional[dict] = None) -> np.ndarray:
    """h0 = GRU over ``embed(prefix_ids)`` from a zero state, domino.py:387-391.

    Restated as ``gi = table[token]``, ``gh = W_hh h + b_hh``, fused cell, one
    prefix token at a time.  Returns ``[B, G]`` in the state dtype.  With
    ``states`` (a dict) it also records ``states["h"]``, the state after each
    prefix token, and ``states["gh"]``, the ``gh`` of every token after the
    first (the first token's is ``b_hh``, from the zero state).
    """
    prefix_ids = np.asarray(prefix_ids, dtype=np.int64)
    B, P = prefix_ids.shape
    table = w.get_table()
    h = np.zeros((B, w.G), dtype=np.float32)
    for j in range(P):
        gi = table[prefix_ids[:, j]]
        gh = linear(h, w.w_hh, w.b_hh, w.dtype)
        h = gru_cell(gi, gh, h, w.dtype)
        if states is not None:
            states.setdefault("h", []).append(h.copy())
            if j > 0:
                states.setdefault("gh", []).append(gh)
    return h


def correction_logits(w: DraftWeights, z_t: np.ndarray, s_t: np.ndarray, base_t: np.ndarray) -> np.ndarray:
    """fp32 logits of one correction step, domino.py:58-136.

    ``acc[b, v] = sum_m fc2[v, m] * SiLU(z[b, m] + s[b, m]) (+ fc2_bias[v]) + base[b, v]``
    """
    mid = silu(np.asarray(z_t, np.float32) + np.asarray(s_t, np.float32))
    acc = mid @ np.asarray(w.fc2, np.float32).T
    if w.fc2_bias is not None:
        acc = acc + np.asarray(w.fc2_bias, np.float32)
    acc = acc + np.asarray(base_t, np.float32)
    return acc.astype(np.float32)


@dataclass
class RolloutTrace:
    tokens: np.ndarray                    # [B, S] int64, the oracle's own argmax per step
    gaps: np.ndarray                      # [B, S] fp32 top-2 gap of the step's logits
    chosen_logit: np.ndarray              # [B, S] fp32 logit of the token fed back
    max_logit: np.ndarray                 # [B, S] fp32 largest logit of the step
    fed_tokens: np.ndarray                # [B, S] tokens fed to the GRU (teacher or own)
    h0: np.ndarray                        # [B, G]
    h: list = field(default_factory=list)  # per step, the GRU state entering the step
    s_proj: list = field(default_factory=list)
    z_part: Optional[np.ndarray] = None   # [B, S, E]
    logits: list = field(default_factory=list)
    gh: list = field(default_factory=list)        # per step t < S-1, h_t W_hh^T + b_hh (domino.py:420)
    prefix_h: list = field(default_factory=list)  # state after each prefix token
    prefix_gh: list = field(default_factory=list)  # gh of each prefix token after the first


def rollout(
    w: DraftWeights,
    prefix_ids: np.ndarray,
    parallel_hiddens: np.ndarray,
    base_logits: np.ndarray,
    teacher_tokens: Optional[np.ndarray] = None,
    keep_logits: bool = False,
) -> RolloutTrace:
    """The runner's rollout, code/kernel/domino.py:374-431 (Triton branch).

    prefix_ids [B, 1+p], parallel_hiddens [B, S, H], base_logits [B, S, V].
    With ``teacher_tokens`` the GRU is fed those tokens instead of the
    oracle's own argmax (teacher forcing), so that a near-tie at one step
    does not change the inputs of the later steps; the oracle's own argmax
    and its top-2 gap are still recorded for every step.
    """
    dtype = w.dtype
    prefix_ids = np.asarray(prefix_ids, dtype=np.int64)
    ph = np.asarray(parallel_hiddens, dtype=np.float32)
    base = np.asarray(base_logits, dtype=np.float32)
    B, S, _ = ph.shape
    z_part = linear(ph, w.w_z, w.fc1_bias, dtype)               # domino.py:381-385
    pre: dict = {}
    h = prefix_gru(w, prefix_ids, pre)                          # domino.py:387-391
    table = w.get_table()
    tokens = np.zeros((B, S), np.int64)
    fed = np.zeros((B, S), np.int64)
    gaps = np.zeros((B, S), np.float32)
    chosen = np.zeros((B, S), np.float32)
    top = np.zeros((B, S), np.float32)
    trace = RolloutTrace(tokens, gaps, chosen, top, fed, h0=h.copy(), z_part=z_part,
                         prefix_h=pre.get("h", []), prefix_gh=pre.get("gh", []))
    for t in range(S):
        trace.h.append(h.copy())
        s_proj = linear(h, w.w_s, None, dtype)                  # domino.py:397
        trace.s_proj.append(s_proj)
        logits = correction_logits(w, z_part[:, t], s_proj, base[:, t])
        if keep_logits:
            trace.logits.append(logits)
        own = argmax_lowest(logits)
        tokens[:, t] = own
        gaps[:, t] = top2_gap(logits)
        top[:, t] = logits[np.arange(B), own]
        cur = own if teacher_tokens is None else np.asarray(teacher_tokens, np.int64)[:, t]
        fed[:, t] = cur
        chosen[:, t] = logits[np.arange(B), cur]
        if t + 1 < S:                                           # domino.py:416-431
            gi = table[cur]
            gh = linear(h, w.w_hh, w.b_hh, dtype)                # domino.py:420
            trace.gh.append(gh)
            h = gru_cell(gi, gh, h, dtype)
    return trace


# ----------------------------------------------------------------------------
# lm_head, pure-draft prefix, acceptance
# ----------------------------------------------------------------------------

def lm_head(parallel_hiddens: np.ndarray, w_lm: np.ndarray, dtype: str) -> np.ndarray:
    """``base_logits = target.lm_head(parallel_hiddens)``, code/dflash.py:424."""
    return linear(parallel_hiddens, w_lm, None, dtype)


def pure_draft_prefix(base_logits: np.ndarray, prefix_len: int) -> np.ndarray:
    """Greedy tokens of the first ``prefix_len`` positions, code/dflash.py:425-427."""
    return argmax_lowest(np.asarray(base_logits, np.float32)[:, :prefix_len])


def accept(verify_ids: np.ndarray, posterior: np.ndarray):
    """Greedy prefix acceptance, code/dflash.py:472-485, for every row.

    verify_ids [B, K+1] = (last accepted token, K draft tokens);
    posterior  [B, K+1] = the target's greedy tokens at those positions.
    Returns ``(a, bonus)``: ``a[b]`` = number of leading draft tokens that
    equal the target's (``(verify[:,1:] == posterior[:,:-1]).cumprod(1).sum(1)``)
    and ``bonus[b] = posterior[b, a[b]]``.  The reference keeps row 0 only and
    records ``a + 1`` as the block's acceptance length (dflash.py:486).
    """
    v = np.asarray(verify_ids, np.int64)
    p = np.asarray(posterior, np.int64)
    match = (v[:, 1:] == p[:, :-1]).astype(np.int64)
    a = np.cumprod(match, axis=1).sum(axis=1).astype(np.int32)
    bonus = p[np.arange(p.shape[0]), a].astype(np.int64)
    return a, bonus
