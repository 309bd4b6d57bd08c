"""Batched greedy speculative decoding with the Domino drafter.

``spec_generate`` is the block loop of the reference's
``DFlashDraftModel.spec_generate`` (code/dflash.py:304-526) for a batch of
requests.  Each row keeps its own position, its own KV-cache lengths and its
own acceptance, so rows that accept different numbers of tokens continue from
different positions in the same batch (the reference runs one sequence,
dflash.py:322-325).  Per block, for every row:

1. the drafter's backbone reads the target features of the tokens accepted
   since the last block and the block's embeddings (dflash.py:411-422);
2. the draft step -- base logits, pure-draft prefix, correction rollout --
   runs in libdomino_draft.so (``runner.draft_block``, dflash.py:424-439);
3. the target verifies the block (dflash.py:464-470);
4. the greedy verify and the acceptance run fused in one pass over the
   target's logits (``runner.verify_accept``, dflash.py:472-478);
5. the accepted tokens and the bonus token are written, the caches are cut
   back to the new position and the accepted tokens' features become the next
   block's context (dflash.py:479-493).

Greedy decoding only (temperature 0), as the draft step is.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch

from .stack import DFlashBackbone, TargetLM


@dataclass
class SpecResult:
    output_ids: List[torch.Tensor]        # per row: prompt + generated ids (mask ids removed, as the reference)
    acceptance_lengths: List[List[int]]   # per row: accepted draft tokens + 1, one entry per block
    num_input_tokens: List[int]
    num_output_tokens: List[int]
    blocks: int = 0
    decode_ms: float = 0.0                # device time of the block loop (after the prefill)
    draft_ms: float = 0.0                 # of which: drafter backbone + draft step (device time)
    verify_ms: float = 0.0                # of which: target verify + fused acceptance
    extra: dict = field(default_factory=dict)


class _NoEvent:
    def record(self):
        pass

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 0.0


def _events(on_gpu: bool = True):
    if not on_gpu:
        return _NoEvent(), _NoEvent()
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


@torch.inference_mode()
def spec_generate(draft: DFlashBackbone, target: TargetLM, runner, prompts: Sequence[torch.Tensor],
                  max_new_tokens: int = 2048, block_size: Optional[int] = None,
                  stop_token_ids: Optional[Sequence[int]] = None, time_blocks: bool = False,
                  use_graphs: Optional[bool] = None) -> SpecResult:
    """Greedy speculative decoding of ``len(prompts)`` requests at once.

    ``runner`` is a ``DraftCorrectionGraphRunner`` built for this drafter and
    target with ``batch_size = len(prompts)``, ``steps = k - pure_draft_prefix_len``
    and ``prefix_token_count = 1 + pure_draft_prefix_len``, where k =
    ``block_size - 1`` (``block_size`` with ``shift_label``) draft positions
    (code/benchmark.py:160-177).  ``prompts`` are 1-D token id tensors of any
    lengths.

    Every block's work is device-side and in place (no host synchronisation
    inside a block), so on a GPU (``use_graphs``, default on) the drafter half
    and the verify half of the steady-state block are each captured once in a
    CUDA graph and replayed; the host reads one flag per block to stop.  With
    ``time_blocks`` both halves are timed with CUDA events around the replays.
    """
    cfg = draft.cfg
    dev = target.lm_head.weight.device
    gpu = dev.type == "cuda"
    if use_graphs is None:
        use_graphs = gpu
    bs = int(block_size or cfg.block_size)
    k_draft = bs if cfg.shift_label else bs - 1  # draft positions per block (dflash.py:392)
    mask_id = cfg.mask_token_id
    B = len(prompts)
    if runner.batch_size != B or runner.steps + runner.prefix_token_count - 1 != k_draft:
        raise ValueError(f"runner must be built for batch {B} and {k_draft} draft positions")
    plen = torch.tensor([int(p.numel()) for p in prompts], device=dev)
    max_len = plen + int(max_new_tokens)
    cap = int(max_len.max()) + 2 * bs + 2
    out = torch.full((B, cap), mask_id, dtype=torch.long, device=dev)
    pmax = int(plen.max())
    ids = torch.full((B, pmax), mask_id, dtype=torch.long, device=dev)
    for b, p in enumerate(prompts):
        ids[b, : p.numel()] = p.to(dev)
        out[b, : p.numel()] = p.to(dev)
    rows = torch.arange(B, device=dev)
    tcache = target.new_cache(B, cap)
    dcache = draft.new_cache(B, cap)
    layers = cfg.target_layer_ids
    max_blocks = int(max_new_tokens) + 2

    # prefill (dflash.py:362-383)
    valid = torch.arange(pmax, device=dev)[None] < plen[:, None]
    logits, ctx0 = target(ids, tcache, valid, feature_layers=layers, logits_at=plen - 1)
    out[rows, plen] = torch.argmax(logits, dim=-1)

    # block state, updated in place
    start = plen.clone()
    done = torch.zeros(B, dtype=torch.bool, device=dev)
    ctx = torch.zeros(B, k_draft + 1, ctx0.shape[-1], dtype=ctx0.dtype, device=dev)
    ctx_valid = torch.zeros(B, k_draft + 1, dtype=torch.bool, device=dev)
    verify_buf = torch.zeros(B, k_draft + 1, dtype=torch.long, device=dev)
    acc_log = torch.zeros(max_blocks, B, dtype=torch.long, device=dev)
    blk = torch.zeros(1, dtype=torch.long, device=dev)
    stop = torch.tensor(list(stop_token_ids), device=dev) if stop_token_ids else None
    offs = torch.arange(bs, device=dev)
    j = torch.arange(k_draft + 2, device=dev)[None]
    all_true = torch.ones(B, k_draft + 1, dtype=torch.bool, device=dev)
    gen_cols = torch.arange(cap, device=dev)[None]

    def draft_half(c, cv):
        # 1-2: drafter backbone, then the draft step in the kernels
        block_ids = out.gather(1, start[:, None] + offs[None])
        noise = target.model.embed_tokens(block_ids)
        hidden = draft(c, cv, noise, dcache)[:, -k_draft:]  # dflash.py:420-421
        verify, _ = runner.draft_block(out.gather(1, start[:, None])[:, 0], hidden)
        verify_buf.copy_(verify)

    def verify_half():
        # 3-4: target verify, greedy acceptance fused with the argmax
        tlogits, feats = target(verify_buf, tcache, all_true, feature_layers=layers)
        posterior, acc, bonus = runner.verify_accept(tlogits, verify_buf)
        # 5: positions start .. start + a take verify[0 .. a], position
        # start + a + 1 the bonus token posterior[a]; caches cut back
        # (dflash.py:479-493).  Finished rows stay where they are.
        acc = acc.long()
        live = ~done
        n_acc = torch.where(live, acc + 1, torch.zeros_like(acc))
        cols = start[:, None] + j
        vals = torch.cat([verify_buf, verify_buf[:, -1:]], 1)
        vals = torch.where(j == acc[:, None] + 1, bonus[:, None], vals)
        write = live[:, None] & (j <= acc[:, None] + 1)
        out.scatter_(1, cols, torch.where(write, vals, out.gather(1, cols)))
        start.add_(n_acc)
        tcache.length.copy_(start)
        ctx.copy_(feats)
        ctx_valid.copy_(j[:, : k_draft + 1] < n_acc[:, None])
        acc_log.index_copy_(0, blk, n_acc[None])
        blk.add_(1)
        d = start >= max_len
        if stop is not None:
            in_gen = (gen_cols >= plen[:, None]) & (gen_cols < start[:, None])
            d = d | (torch.isin(out, stop) & in_gen).any(1)
        done.copy_(d)

    draft_ms = verify_ms = 0.0
    blocks = 0
    g_draft = g_verify = None
    t0, t1 = _events(gpu)
    t0.record()
    while True:
        if time_blocks:
            e0, e1 = _events(gpu)
            e2, e3 = _events(gpu)
            e0.record()
        if blocks == 0:
            draft_half(ctx0, valid)  # the prompt is the first block's context
        elif g_draft is not None:
            g_draft.replay()
        else:
            draft_half(ctx, ctx_valid)
        if time_blocks:
            e1.record()
            e2.record()
        if g_verify is not None:
            g_verify.replay()
        else:
            verify_half()
        if time_blocks:
            e3.record()
            e3.synchronize()
            draft_ms += e0.elapsed_time(e1)
            verify_ms += e2.elapsed_time(e3)
        blocks += 1
        if bool(done.all()) or blocks >= max_blocks:
            break
        if use_graphs and blocks == 2 and g_draft is None:
            # the steady-state block has run once eagerly: capture both halves
            g_draft, g_verify = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_draft):
                draft_half(ctx, ctx_valid)
            with torch.cuda.graph(g_verify):
                verify_half()
    t1.record()
    t1.synchronize()
    log = acc_log[:blocks].tolist()
    accs = [[row[b] for row in log if row[b] > 0] for b in range(B)]
    outs, n_out = [], []
    for b in range(B):
        row = out[b, : int(max_len[b])]
        row = row[row != mask_id]
        if stop is not None:
            hit = torch.isin(row[int(plen[b]):], stop).nonzero()
            if hit.numel():
                row = row[: int(plen[b]) + int(hit[0, 0]) + 1]
        outs.append(row)
        n_out.append(int(row.numel() - plen[b]))
    return SpecResult(outs, accs, plen.tolist(), n_out, blocks, t0.elapsed_time(t1), draft_ms, verify_ms)
