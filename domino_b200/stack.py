"""The models on either side of the draft step, for the batched block loop.

* ``TargetLM`` -- a Qwen3 causal LM (the target that verifies each block and
  whose hidden states feed the drafter), parameter names as in
  ``transformers``' ``Qwen3ForCausalLM`` so its state dict loads unchanged.
* ``DFlashBackbone`` -- the Domino draft model: the DFlash block-parallel
  backbone (code/dflash.py:54-205, 234-302) plus the correction head modules
  the runner reads (``embed_proj``, ``prefix_gru``, code/dflash.py:261-274),
  parameter names as in the reference's ``DFlashDraftModel`` so a Domino
  checkpoint's state dict loads unchanged.

Both run batched with a per-row ("ragged") KV cache: row b of a batch holds
``length[b]`` valid entries and new keys / values are written at each row's
own positions, so rows that accepted different numbers of tokens continue
from different positions without padding holes (the reference's loop is
batch-1 only and crops one ``DynamicCache``, code/dflash.py:322-325, 488).

Numerics follow ``transformers`` 5.x Qwen3 (RMSNorm in fp32, rotary tables in
fp32, eager attention with an fp32 softmax and a min-float mask), so that
with the same weights the logits agree with the reference's to rounding.
This is host-side glue (PyTorch ops); the draft step itself runs in
libdomino_draft.so.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class StackConfig:
    """The fields of a Qwen3 config the stack needs (``transformers.Qwen3Config``)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    # DFlash drafter only (code/dflash.py:234-258)
    block_size: int = 16
    target_layer_ids: List[int] = field(default_factory=list)
    mask_token_id: int = 0
    emb_dim: int = 0
    gru_hidden_dim: int = 0
    pure_draft_prefix_len: int = 0
    shift_label: bool = False  # draft all block_size positions instead of block_size - 1 (dflash.py:347-349)

    @classmethod
    def from_hf(cls, cfg) -> "StackConfig":
        rope = getattr(cfg, "rope_parameters", None) or {}
        theta = rope.get("rope_theta", getattr(cfg, "rope_theta", 1e6))
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        out = cls(cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                  cfg.num_attention_heads, cfg.num_key_value_heads, head_dim, cfg.rms_norm_eps, float(theta))
        dc = getattr(cfg, "dflash_config", None)
        if dc:
            out.block_size = int(getattr(cfg, "block_size", 16))
            out.target_layer_ids = list(dc.get("target_layer_ids") or build_target_layer_ids(
                cfg.num_target_layers, cfg.num_hidden_layers))
            out.mask_token_id = int(dc["mask_token_id"])
            out.emb_dim = int(dc["emb_dim"])
            out.gru_hidden_dim = int(dc["gru_hidden_dim"])
            out.pure_draft_prefix_len = int(dc.get("pure_draft_prefix_len", 0))
            out.shift_label = bool(dc.get("shift_label", False))
        return out


def build_target_layer_ids(num_target_layers: int, num_draft_layers: int) -> List[int]:
    """Target layers whose outputs feed the drafter (code/dflash.py:207-219)."""
    if num_draft_layers == 1:
        return [num_target_layers // 2]
    start, end = 1, num_target_layers - 3
    return [int(round(start + i * (end - start) / (num_draft_layers - 1))) for i in range(num_draft_layers)]


class RMSNorm(nn.Module):
    def __init__(self, n: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n))
        self.eps = eps

    def forward(self, x):
        dt = x.dtype
        x = x.float()
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * x.to(dt)


_INV_FREQ: dict = {}


def rope_tables(cfg: StackConfig, positions: torch.Tensor, dtype):
    """cos, sin [B, T, head_dim] for integer positions [B, T] (fp32 math, then ``dtype``).

    The inverse frequencies are computed on the host, as ``transformers`` does,
    and moved to the device once."""
    d = cfg.head_dim
    key = (d, cfg.rope_theta, positions.device)
    inv = _INV_FREQ.get(key)
    if inv is None:
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
        inv = _INV_FREQ.setdefault(key, inv.to(positions.device))
    freqs = positions.float()[..., None] * inv[None, None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    """x [B, heads, T, D] with cos / sin [B, T, D]."""
    cos, sin = cos[:, None], sin[:, None]
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


class RaggedKVCache:
    """Keys / values [B, kv_heads, capacity + 1, head_dim] per layer and a
    valid length per row.  ``write`` puts new entries at per-row positions;
    the extra last slot takes the entries that are not valid, so no call
    needs the host to count them (the forward passes are free of host
    synchronisation and can be captured in a CUDA graph)."""

    def __init__(self, layers: int, batch: int, kv_heads: int, capacity: int, head_dim: int, dtype, device):
        self.k = [torch.zeros(batch, kv_heads, capacity + 1, head_dim, dtype=dtype, device=device)
                  for _ in range(layers)]
        self.v = [torch.zeros_like(t) for t in self.k]
        self.length = torch.zeros(batch, dtype=torch.long, device=device)
        self.capacity = capacity

    def write(self, layer: int, k, v, slots, valid):
        """k, v [B, kv_heads, T, D] to cache slots [B, T] where ``valid`` [B, T]."""
        B, _, T, _ = k.shape
        b_idx = torch.arange(B, device=k.device).repeat_interleave(T)
        s = torch.where(valid, slots, self.capacity).reshape(-1)
        self.k[layer][b_idx, :, s] = k.transpose(1, 2).reshape(B * T, k.shape[1], k.shape[3])
        self.v[layer][b_idx, :, s] = v.transpose(1, 2).reshape(B * T, v.shape[1], v.shape[3])


def _attend(q, k, v, allowed, groups: int, scaling: float):
    """Eager attention (``transformers``' eager_attention_forward): q [B, H, T, D],
    k / v [B, KV, L, D], allowed [B, T, L] -> [B, T, H * D]."""
    if groups > 1:
        k = k.repeat_interleave(groups, dim=1)
        v = v.repeat_interleave(groups, dim=1)
    w = torch.matmul(q, k.transpose(2, 3)) * scaling
    w = w.masked_fill(~allowed[:, None], torch.finfo(w.dtype).min)
    w = F.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    out = torch.matmul(w, v)
    return out.transpose(1, 2).reshape(q.shape[0], q.shape[2], -1)


class Attention(nn.Module):
    def __init__(self, cfg: StackConfig):
        super().__init__()
        h, d = cfg.hidden_size, cfg.head_dim
        self.cfg = cfg
        self.q_proj = nn.Linear(h, cfg.num_attention_heads * d, bias=False)
        self.k_proj = nn.Linear(h, cfg.num_key_value_heads * d, bias=False)
        self.v_proj = nn.Linear(h, cfg.num_key_value_heads * d, bias=False)
        self.o_proj = nn.Linear(cfg.num_attention_heads * d, h, bias=False)
        self.q_norm = RMSNorm(d, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(d, cfg.rms_norm_eps)

    def heads(self, x, proj, norm):
        B, T, _ = x.shape
        y = proj(x).view(B, T, -1, self.cfg.head_dim)
        return (norm(y) if norm is not None else y).transpose(1, 2)


class MLP(nn.Module):
    def __init__(self, cfg: StackConfig):
        super().__init__()
        self.gate_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, cfg: StackConfig):
        super().__init__()
        self.self_attn = Attention(cfg)
        self.mlp = MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class _Model(nn.Module):
    def __init__(self, cfg: StackConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class TargetLM(nn.Module):
    """Qwen3 causal LM with a ragged KV cache (parameter names of ``Qwen3ForCausalLM``)."""

    def __init__(self, cfg: StackConfig):
        super().__init__()
        self.cfg = cfg
        self.model = _Model(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)

    def new_cache(self, batch: int, capacity: int) -> RaggedKVCache:
        p = self.lm_head.weight
        return RaggedKVCache(self.cfg.num_hidden_layers, batch, self.cfg.num_key_value_heads, capacity,
                             self.cfg.head_dim, p.dtype, p.device)

    @torch.inference_mode()
    def forward(self, ids, cache: RaggedKVCache, valid, feature_layers: Sequence[int] = (), logits_at=None):
        """Append ``ids`` [B, T] (entries where ``valid`` [B, T]; valid entries
        of a row are a prefix of it) after each row's cached tokens, causally.

        Returns ``(logits, features)``: logits [B, T, V] (or [B, V] at the
        positions ``logits_at`` [B]) and the concatenated outputs of
        ``feature_layers`` [B, T, len * H] (``transformers``' hidden_states
        convention: the last layer's entry is the final-normed output), then
        advances ``cache.length`` by each row's valid count.
        """
        cfg = self.cfg
        B, T = ids.shape
        start = cache.length.clone()
        pos = start[:, None] + torch.arange(T, device=ids.device)[None]
        slots = pos.clamp(max=cache.capacity - 1)
        L = cache.capacity  # keys past a row's length are masked
        key_pos = torch.arange(L, device=ids.device)
        allowed = key_pos[None, None, :] <= pos[:, :, None]
        allowed = allowed | ~valid[:, :, None]  # padded queries attend to everything (ignored)
        x = self.model.embed_tokens(ids)
        cos, sin = rope_tables(cfg, pos, x.dtype)
        groups = cfg.num_attention_heads // cfg.num_key_value_heads
        feats = {}
        for li, layer in enumerate(self.model.layers):
            a = layer.self_attn
            hn = layer.input_layernorm(x)
            q = apply_rope(a.heads(hn, a.q_proj, a.q_norm), cos, sin)
            k = apply_rope(a.heads(hn, a.k_proj, a.k_norm), cos, sin)
            v = a.heads(hn, a.v_proj, None)
            cache.write(li, k, v, slots, valid)
            o = _attend(q, cache.k[li][:, :, :L], cache.v[li][:, :, :L], allowed, groups, a.cfg.head_dim ** -0.5)
            x = x + a.o_proj(o)
            x = x + layer.mlp(layer.post_attention_layernorm(x))
            if li in feature_layers and li != cfg.num_hidden_layers - 1:
                feats[li] = x
        x = self.model.norm(x)
        for li in feature_layers:
            if li == cfg.num_hidden_layers - 1:
                feats[li] = x
        cache.length.copy_(start + valid.sum(1))
        if logits_at is not None:
            x = x[torch.arange(B, device=ids.device), logits_at]
        logits = self.lm_head(x)
        features = torch.cat([feats[i] for i in feature_layers], dim=-1) if feature_layers else None
        return logits, features


class DFlashBackbone(nn.Module):
    """The Domino draft model (parameter names of the reference's ``DFlashDraftModel``,
    code/dflash.py:234-274): DFlash layers that attend from the block's
    positions to [context features ‖ block] without a causal mask, plus the
    correction head modules ``embed_proj`` and ``prefix_gru``."""

    def __init__(self, cfg: StackConfig):
        super().__init__()
        self.cfg = cfg
        H = cfg.hidden_size
        self.layers = nn.ModuleList([DecoderLayer(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(H, cfg.rms_norm_eps)
        self.fc = nn.Linear(len(cfg.target_layer_ids) * H, H, bias=False)
        self.hidden_norm = RMSNorm(H, cfg.rms_norm_eps)
        self.prefix_gru = nn.GRU(H, cfg.gru_hidden_dim, num_layers=1, batch_first=True, bias=False)
        self.embed_proj = nn.Sequential(nn.Linear(H + cfg.gru_hidden_dim, cfg.emb_dim, bias=False), nn.SiLU(),
                                        nn.Linear(cfg.emb_dim, cfg.vocab_size, bias=False))

    def new_cache(self, batch: int, capacity: int) -> RaggedKVCache:
        p = self.fc.weight
        return RaggedKVCache(self.cfg.num_hidden_layers, batch, self.cfg.num_key_value_heads, capacity,
                             self.cfg.head_dim, p.dtype, p.device)

    @torch.inference_mode()
    def forward(self, ctx_features, ctx_valid, noise, cache: RaggedKVCache):
        """The block's hidden states (code/dflash.py:278-302, attention 107-155).

        ctx_features [B, C, len(layers) * H]: target features of the tokens
        accepted since the last call (valid where ``ctx_valid`` [B, C], a
        prefix of each row); noise [B, T, H]: embeddings of the block (last
        accepted token, then mask tokens).  The context keys / values stay in
        ``cache`` (its length grows by the valid context); the block's are
        used for this call only, as the reference crops them (dflash.py:422).
        Returns the normed hidden states of the block [B, T, H].
        """
        cfg = self.cfg
        B, C, _ = ctx_features.shape
        T = noise.shape[1]
        dev = noise.device
        start = cache.length.clone()
        n_ctx = ctx_valid.sum(1)
        ctx_pos = start[:, None] + torch.arange(C, device=dev)[None]
        blk_pos = (start + n_ctx)[:, None] + torch.arange(T, device=dev)[None]
        ctx_h = self.hidden_norm(self.fc(ctx_features))
        x = noise
        cos_c, sin_c = rope_tables(cfg, ctx_pos, x.dtype)
        cos_b, sin_b = rope_tables(cfg, blk_pos, x.dtype)
        L = cache.capacity  # keys past a row's context + block are masked
        key_pos = torch.arange(L, device=dev)
        allowed = (key_pos[None, :] < (start + n_ctx + T)[:, None])[:, None, :].expand(B, T, L)
        slots_c = ctx_pos.clamp(max=cache.capacity - 1)
        slots_b = blk_pos.clamp(max=cache.capacity - 1)
        all_b = torch.ones(B, T, dtype=torch.bool, device=dev)
        groups = cfg.num_attention_heads // cfg.num_key_value_heads
        for li, layer in enumerate(self.layers):
            a = layer.self_attn
            hn = layer.input_layernorm(x)
            q = apply_rope(a.heads(hn, a.q_proj, a.q_norm), cos_b, sin_b)
            k_c = apply_rope(a.heads(ctx_h, a.k_proj, a.k_norm), cos_c, sin_c)
            k_b = apply_rope(a.heads(hn, a.k_proj, a.k_norm), cos_b, sin_b)
            cache.write(li, k_c, a.heads(ctx_h, a.v_proj, None), slots_c, ctx_valid)
            cache.write(li, k_b, a.heads(hn, a.v_proj, None), slots_b, all_b)
            o = _attend(q, cache.k[li][:, :, :L], cache.v[li][:, :, :L], allowed, groups, a.cfg.head_dim ** -0.5)
            x = x + a.o_proj(o)
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        cache.length.copy_(start + n_ctx)
        return self.norm(x)
