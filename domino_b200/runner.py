"""Drop-in replacement for the reference's ``DraftCorrectionGraphRunner``.

Same constructor and call signature as code/kernel/domino.py:245-256 and
495-508, so it can be passed as ``graph_runner=`` to the reference's
``DFlashDraftModel.spec_generate`` (code/dflash.py:313, 429-439).  The whole
rollout runs as the hand-written sm_100a kernels of libdomino_draft.so
(``dd_rollout``), captured once into a CUDA graph like the reference does;
PyTorch only provides device memory, the stream and the graph.

Additions on the same object:
  * ``accept(verify_ids, posterior)`` -- greedy acceptance of every row
    (code/dflash.py:472-485) -> (accept int32 [B], bonus int64 [B]);
  * ``draft_block(last_token, parallel_hiddens)`` -- the whole draft side of a
    block with the base-logit lm_head fused in (code/dflash.py:424-439);
    needs ``target_model.lm_head``.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import _lib

__all__ = ["DraftCorrectionGraphRunner", "unwrap_correction_mlp", "DominoDraftError"]

DominoDraftError = _lib.DominoDraftError


def unwrap_correction_mlp(embed_proj: nn.Module):
    """(fc1, middle, fc2) of ``embed_proj``; same checks as code/kernel/domino.py:15-50."""
    if not isinstance(embed_proj, nn.Sequential):
        raise TypeError("Graph runner requires draft_model.embed_proj to be nn.Sequential.")
    modules = list(embed_proj.children())
    if len(modules) < 2:
        raise ValueError("embed_proj must contain at least two layers.")
    if not isinstance(modules[0], nn.Linear):
        raise ValueError("embed_proj first layer must be nn.Linear.")
    if not isinstance(modules[-1], nn.Linear):
        raise ValueError("embed_proj last layer must be nn.Linear.")
    middle = nn.Sequential(*modules[1:-1]) if len(modules) > 2 else nn.Identity()
    return modules[0], middle, modules[-1]


def _middle_is_silu(middle: nn.Module) -> bool:
    """The SiLU guard of code/kernel/domino.py:280-287."""
    if isinstance(middle, nn.SiLU):
        return True
    return (
        isinstance(middle, nn.Sequential)
        and len(list(middle.children())) == 1
        and isinstance(list(middle.children())[0], nn.SiLU)
    )


def middle_kind(middle: nn.Module) -> int:
    """The kernels' code for ``embed_proj``'s middle.

    One ``nn.SiLU`` (alone or as the single child of a Sequential) is the
    reference's fused path (code/kernel/domino.py:280-289); every other middle
    runs its PyTorch branch (domino.py:406-431), which the kernels reproduce for
    an identity, ReLU, GELU (erf or tanh), Tanh, Sigmoid or SiLU, with Dropout
    and Identity modules around it (eval mode).  Anything else raises
    ``NotImplementedError``: there is no fallback that would compute it another way.
    """
    if _middle_is_silu(middle):
        return _lib.DD_MIDDLE_SILU

    def flat(m):
        return [x for c in m.children() for x in flat(c)] if isinstance(m, nn.Sequential) else [m]

    acts = [m for m in flat(middle) if not isinstance(m, (nn.Identity, nn.Dropout))]
    if not acts:
        return _lib.DD_MIDDLE_IDENTITY
    if len(acts) == 1:
        a = acts[0]
        if isinstance(a, nn.ReLU):
            return _lib.DD_MIDDLE_RELU
        if isinstance(a, nn.GELU):
            return _lib.DD_MIDDLE_GELU_TANH if a.approximate == "tanh" else _lib.DD_MIDDLE_GELU
        if isinstance(a, nn.Tanh):
            return _lib.DD_MIDDLE_TANH
        if isinstance(a, nn.Sigmoid):
            return _lib.DD_MIDDLE_SIGMOID
        if isinstance(a, nn.SiLU):
            return _lib.DD_MIDDLE_SILU_ROUNDED
    raise NotImplementedError(
        f"embed_proj middle {middle!r}: the B200 runner implements an identity, ReLU, GELU, Tanh, Sigmoid or SiLU "
        "middle (with Dropout / Identity around it)")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


_DTYPES = {torch.bfloat16: _lib.DD_BF16, torch.float16: _lib.DD_FP16, torch.float32: _lib.DD_F32}


class DraftCorrectionGraphRunner:
    """Greedy draft-correction rollout on B200 (drop-in for the reference runner).

    Args mirror code/kernel/domino.py:245-256.  Extra keywords:
      use_graph:   capture ``dd_rollout`` into a CUDA graph at construction
                   (default True, as the reference always does).
      vocab_shard: split fc2 and lm_head by vocab rows over the ranks of the
                   default torch.distributed process group (one process per
                   GPU); every rank must construct the runner with the same
                   weights and call it with the same inputs.  The per-step
                   argmax is combined across GPUs inside the kernels.
      pack_weights: keep a tile-packed copy of the streamed matrices (W_z,
                   W_s, W_hh, fc2, lm_head), streamed with 1-D bulk copies;
                   the default streams the module parameters in place.
    """

    def __init__(
        self,
        draft_model: nn.Module,
        target_model: nn.Module,
        batch_size: int,
        steps: int,
        hidden_dim: int,
        gru_hidden_dim: int,
        vocab_size: int,
        prefix_token_count: int,
        device: torch.device,
        use_graph: bool = True,
        vocab_shard: bool = False,
        pack_weights: bool = False,
    ):
        self.steps = int(steps)
        self.draft_model = draft_model
        self.target_model = target_model
        self.prefix_token_count = int(prefix_token_count)
        self.gru_hidden_dim = int(gru_hidden_dim)
        self.batch_size = int(batch_size)
        self.hidden_dim = int(hidden_dim)
        self.vocab_size = int(vocab_size)

        fc1, self.middle, fc2 = unwrap_correction_mlp(draft_model.embed_proj)
        expected_in = hidden_dim + gru_hidden_dim
        if fc1.in_features != expected_in:
            raise ValueError(
                f"Correction MLP input dim mismatch: got {fc1.in_features}, "
                f"expected {expected_in} = hidden_dim + gru_hidden_dim."
            )
        self._middle_kind = middle_kind(self.middle)
        gru = draft_model.prefix_gru
        if gru.num_layers != 1 or gru.bidirectional:
            raise ValueError("prefix_gru must be a single-layer unidirectional nn.GRU")

        dtype = next(draft_model.parameters()).dtype
        if dtype not in _DTYPES:
            raise NotImplementedError(f"the B200 runner computes with bf16, fp16 or fp32 weights, got {dtype}")
        self.dtype = dtype
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("DraftCorrectionGraphRunner runs on a CUDA device (sm_100a)")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device

        # Non-owning views of the module parameters (the reference's
        # `.detach().contiguous()` copies only when a view is non-contiguous).
        self._fc1 = fc1.weight.detach()
        self._fc1_bias = fc1.bias.detach().contiguous() if fc1.bias is not None else None
        self._fc2 = fc2.weight.detach()
        self._fc2_bias = fc2.bias.detach().contiguous() if fc2.bias is not None else None
        self._w_ih = gru.weight_ih_l0.detach()
        self._w_hh = gru.weight_hh_l0.detach()
        self._b_ih = gru.bias_ih_l0.detach().contiguous() if gru.bias else None
        self._b_hh = gru.bias_hh_l0.detach().contiguous() if gru.bias else None
        embed = target_model.model.embed_tokens.weight.detach()
        lm = getattr(target_model, "lm_head", None)
        self._lm_head = lm.weight.detach() if isinstance(lm, nn.Linear) and lm.bias is None else None
        for name in ("_fc1", "_fc2", "_w_ih", "_w_hh"):
            t = getattr(self, name)
            if t.stride(-1) != 1:
                setattr(self, name, t.contiguous())
        if embed.stride(-1) != 1:
            embed = embed.contiguous()

        self._lib = _lib.load()
        self.rank, self.world, self.vocab_begin, self.vocab_end = 0, 1, 0, self.vocab_size
        if vocab_shard:
            import torch.distributed as dist
            from .parallel import shard_rows

            if dist.is_available() and dist.is_initialized():
                self.rank, self.world = dist.get_rank(), dist.get_world_size()
            if self.world > 8:
                raise ValueError("vocab sharding supports up to 8 ranks")
            start, count = shard_rows(self.vocab_size, self.world, self.rank)
            self.vocab_begin, self.vocab_end = start, start + count
        cfg = _lib.DDConfig(
            batch=self.batch_size, steps=self.steps, hidden=self.hidden_dim, gru_hidden=self.gru_hidden_dim,
            emb_dim=fc1.out_features, vocab=self.vocab_size, prefix_tokens=self.prefix_token_count,
            dtype=_DTYPES[dtype],
        )
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(self._lib.dd_create(ctypes.byref(cfg), device.index, ctypes.byref(handle)), None, "dd_create")
        self._h = handle
        _lib.check(self._lib.dd_set_middle(self._h, self._middle_kind), self._h, "dd_set_middle")

        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device)
            # table[v] = embed[v] @ W_ih^T + b_ih (code/kernel/domino.py:322-327)
            self._table = torch.empty(self.vocab_size, 3 * self.gru_hidden_dim, dtype=dtype, device=device)
            _lib.check(
                self._lib.dd_build_table(
                    self._h, embed.data_ptr(), embed.stride(0), self._w_ih.data_ptr(), self._w_ih.stride(0),
                    _ptr(self._b_ih), self._table.data_ptr(), stream.cuda_stream,
                ),
                self._h, "dd_build_table",
            )
            self._peer_ptrs = []
            if self.world > 1:
                self._setup_vocab_shard()
            v0, v1 = self.vocab_begin, self.vocab_end
            fc2_rows = self._fc2[v0:v1]
            lm_rows = self._lm_head[v0:v1] if self._lm_head is not None else None
            fc2_bias = self._fc2_bias[v0:v1] if self._fc2_bias is not None else None
            self._weights = _lib.DDWeights(
                fc1=self._fc1.data_ptr(), fc1_ld=self._fc1.stride(0), fc1_bias=_ptr(self._fc1_bias),
                fc2=fc2_rows.data_ptr(), fc2_ld=fc2_rows.stride(0), fc2_bias=_ptr(fc2_bias),
                w_hh=self._w_hh.data_ptr(), w_hh_ld=self._w_hh.stride(0), b_hh=_ptr(self._b_hh),
                table=self._table.data_ptr(), table_ld=self._table.stride(0),
                lm_head=_ptr(lm_rows), lm_head_ld=lm_rows.stride(0) if lm_rows is not None else 0,
            )
            _lib.check(self._lib.dd_set_weight_layout(self._h, 1 if pack_weights else 0), self._h, "layout")
            _lib.check(self._lib.dd_set_weights(self._h, ctypes.byref(self._weights)), self._h, "dd_set_weights")

            B, S = self.batch_size, self.steps
            self.static_prefix_ids = torch.zeros(B, self.prefix_token_count, dtype=torch.long, device=device)
            self.static_parallel_hiddens = torch.zeros(B, S, self.hidden_dim, dtype=dtype, device=device)
            self.static_base_logits = torch.zeros(B, S, self.vocab_size, dtype=dtype, device=device)
            self.static_out = torch.zeros(B, S, dtype=torch.long, device=device)
            self._accept_out = torch.zeros(B, dtype=torch.int32, device=device)
            self._bonus_out = torch.zeros(B, dtype=torch.long, device=device)

            self.graph = None
            if use_graph:
                s = torch.cuda.Stream(device)
                s.wait_stream(torch.cuda.current_stream(device))
                with torch.cuda.stream(s):
                    for _ in range(3):
                        self._forward_impl()
                torch.cuda.current_stream(device).wait_stream(s)
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self._forward_impl()

    def _setup_vocab_shard(self):
        """Map every rank's exchange buffer here (CUDA IPC) and make this handle a vocab shard."""
        import torch.distributed as dist

        buf = ctypes.c_void_p()
        _lib.check(self._lib.dd_get_exchange_buffer(self._h, ctypes.byref(buf), None), self._h, "exchange buffer")
        blob = ctypes.create_string_buffer(64)
        _lib.check(self._lib.dd_ipc_export(buf, blob), None, "dd_ipc_export")
        from .parallel import all_gather_bytes

        blobs = all_gather_bytes(blob.raw)
        ptrs = (ctypes.c_void_p * self.world)()
        for j, b in enumerate(blobs):
            if j == self.rank:
                ptrs[j] = buf.value
                continue
            p = ctypes.c_void_p()
            _lib.check(self._lib.dd_ipc_open(self.device.index, ctypes.create_string_buffer(b, 64), ctypes.byref(p)),
                       None, f"dd_ipc_open(rank {j})")
            ptrs[j] = p.value
            self._peer_ptrs.append(p.value)
        _lib.check(self._lib.dd_set_vocab_shard(self._h, self.rank, self.world, self.vocab_begin, self.vocab_end,
                                                ptrs), self._h, "dd_set_vocab_shard")
        # every rank has mapped every buffer before anyone publishes into it
        dist.barrier()

    # ------------------------------------------------------------------ core
    def _forward_impl(self, stream=None):
        """Enqueue one rollout over the static buffers (code/kernel/domino.py:374-431)."""
        st = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(
            self._lib.dd_rollout(
                self._h, self.static_prefix_ids.data_ptr(), self.static_parallel_hiddens.data_ptr(),
                self.static_base_logits.data_ptr(), self.static_out.data_ptr(), st,
            ),
            self._h, "dd_rollout",
        )

    @torch.inference_mode()
    def __call__(self, prefix_ids: torch.Tensor, parallel_hiddens: torch.Tensor, base_logits: torch.Tensor) -> torch.Tensor:
        """[B, 1+p] ids, [B, S, H] hiddens, [B, S, V] base logits -> [B, S] int64 draft tokens."""
        self.static_prefix_ids.copy_(prefix_ids)
        self.static_parallel_hiddens.copy_(parallel_hiddens)
        self.static_base_logits.copy_(base_logits)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._forward_impl()
        return self.static_out.clone()

    # ------------------------------------------------------------ additions
    @torch.inference_mode()
    def accept(self, verify_ids: torch.Tensor, posterior: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Greedy acceptance of every row (code/dflash.py:472-485).

        Returns ``(a, bonus)`` with ``a[b]`` = accepted draft tokens (the
        reference records ``a + 1`` as the acceptance length) and
        ``bonus[b] = posterior[b, a[b]]``.
        """
        v = verify_ids.to(self.device, torch.long).contiguous()
        p = posterior.to(self.device, torch.long).contiguous()
        if v.shape != p.shape or v.dim() != 2:
            raise ValueError("verify_ids and posterior must both be [B, K+1]")
        B, K1 = v.shape
        acc = torch.empty(B, dtype=torch.int32, device=self.device)
        bonus = torch.empty(B, dtype=torch.long, device=self.device)
        _lib.check(
            self._lib.dd_accept(v.data_ptr(), p.data_ptr(), B, K1, acc.data_ptr(), bonus.data_ptr(),
                                torch.cuda.current_stream(self.device).cuda_stream),
            None, "dd_accept",
        )
        return acc, bonus

    @torch.inference_mode()
    def verify_accept(self, target_logits: torch.Tensor, verify_ids: torch.Tensor):
        """Greedy verify fused with acceptance (code/dflash.py:472-485).

        target_logits [B, K+1, V] (bf16, fp16 or fp32), verify_ids [B, K+1].
        Returns ``(posterior [B, K+1] int64, accept [B] int32, bonus [B] int64)``
        with ``posterior = argmax(target_logits, -1)`` computed in the same pass.
        """
        dt = {torch.bfloat16: _lib.DD_BF16, torch.float16: _lib.DD_FP16, torch.float32: _lib.DD_F32}
        if target_logits.dtype not in dt:
            raise TypeError(f"target_logits dtype {target_logits.dtype}")
        logits = target_logits.to(self.device).contiguous()
        v = verify_ids.to(self.device, torch.long).contiguous()
        B, K1, V = logits.shape
        if B != self.batch_size or V != self.vocab_size or tuple(v.shape) != (B, K1):
            raise ValueError(f"expected logits [{self.batch_size}, K+1, {self.vocab_size}] and verify_ids [B, K+1]")
        posterior = torch.empty(B, K1, dtype=torch.long, device=self.device)
        acc = torch.empty(B, dtype=torch.int32, device=self.device)
        bonus = torch.empty(B, dtype=torch.long, device=self.device)
        _lib.check(
            self._lib.dd_verify_accept(self._h, logits.data_ptr(), dt[logits.dtype], K1, v.data_ptr(),
                                       posterior.data_ptr(), acc.data_ptr(), bonus.data_ptr(),
                                       torch.cuda.current_stream(self.device).cuda_stream),
            self._h, "dd_verify_accept",
        )
        return posterior, acc, bonus

    @torch.inference_mode()
    def draft_block(self, last_token: torch.Tensor, parallel_hiddens: torch.Tensor,
                    base_logits_out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Draft side of one block with the lm_head fused (code/dflash.py:424-439).

        last_token [B] (verify_ids[:, 0]); parallel_hiddens [B, p+S, H].
        Returns ``(verify_ids [B, p+S+1] int64, base_logits [B, p+S, V])``; with
        ``vocab_shard`` the base logits hold this rank's vocab columns only.
        """
        if self._lm_head is None:
            raise ValueError("target_model.lm_head (bias-free nn.Linear) is required for draft_block")
        B = self.batch_size
        K = self.prefix_token_count - 1 + self.steps
        ph = parallel_hiddens.to(self.device, self.dtype).contiguous()
        if tuple(ph.shape) != (B, K, self.hidden_dim):
            raise ValueError(f"parallel_hiddens must be [{B}, {K}, {self.hidden_dim}]")
        last = last_token.to(self.device, torch.long).reshape(B).contiguous()
        if base_logits_out is None:
            base_logits_out = torch.empty(B, K, self.vocab_end - self.vocab_begin, dtype=self.dtype,
                                          device=self.device)
        verify = torch.empty(B, K + 1, dtype=torch.long, device=self.device)
        _lib.check(
            self._lib.dd_draft_block(self._h, last.data_ptr(), ph.data_ptr(), base_logits_out.data_ptr(),
                                     verify.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream),
            self._h, "dd_draft_block",
        )
        return verify, base_logits_out

    @torch.inference_mode()
    def rollout_trace(self, prefix_ids: torch.Tensor, parallel_hiddens: torch.Tensor, base_logits: torch.Tensor):
        """One eager rollout (like ``__call__``) that also returns its per-step states.

        Returns ``(tokens [B, S], states)`` with ``states`` holding, in the
        weight dtype (code/kernel/domino.py:381-431):
          ``z``  [B, S, E]        z projection (+ fc1 bias);
          ``h``  [P + S - 1, B, G] GRU state after each prefix token, then
                                   after the GRU step of each draft step;
          ``gh`` [P + S - 2, B, 3G] ``h W_hh^T + b_hh`` fed to those GRU steps
                                   (prefix tokens after the first, then draft steps);
          ``s``  [S, B, E]        s projections.
        P = ``prefix_token_count``.  Unsharded runners only.
        """
        if self.world > 1:
            raise ValueError("rollout_trace needs an unsharded runner")
        B, S, P, E = self.batch_size, self.steps, self.prefix_token_count, self._fc1.shape[0]
        G, dev, dt = self.gru_hidden_dim, self.device, self.dtype
        st = {
            "z": torch.zeros(B, S, E, dtype=dt, device=dev),
            "h": torch.zeros(P + S - 1, B, G, dtype=dt, device=dev),
            "gh": torch.zeros(max(P + S - 2, 1), B, 3 * G, dtype=dt, device=dev),
            "s": torch.zeros(S, B, E, dtype=dt, device=dev),
        }
        tr = _lib.DDTrace(z=st["z"].data_ptr(), h=st["h"].data_ptr(), gh=st["gh"].data_ptr(), s=st["s"].data_ptr())
        self.static_prefix_ids.copy_(prefix_ids)
        self.static_parallel_hiddens.copy_(parallel_hiddens)
        self.static_base_logits.copy_(base_logits)
        _lib.check(self._lib.dd_set_trace(self._h, ctypes.byref(tr)), self._h, "dd_set_trace")
        try:
            self._forward_impl()
        finally:
            self._lib.dd_set_trace(self._h, None)
        st["gh"] = st["gh"][: P + S - 2]
        return self.static_out.clone(), st

    def status(self) -> int:
        """Synchronise and return (and clear) the device status bits (DD_STATUS_*)."""
        return _lib.check(self._lib.dd_get_status(self._h), self._h, "dd_get_status")

    @property
    def table(self) -> torch.Tensor:
        """The GRU input table embed @ W_ih^T + b_ih, [V, 3G]."""
        return self._table

    def close(self):
        """Free the handle.  A vocab-sharded runner must be closed by every rank
        (the call contains a barrier over the default process group)."""
        if getattr(self, "_h", None):
            self.graph = None
            if self.world > 1:
                # Peers publish argmax words and s / gh flags into this rank's
                # exchange buffer with system-scope stores: every rank drains
                # its own work and waits for all the others before any buffer
                # is unmapped or freed (the mirror of the setup barrier).
                import torch.distributed as dist

                torch.cuda.synchronize(self.device)
                if dist.is_available() and dist.is_initialized():
                    dist.barrier()
            for p in getattr(self, "_peer_ptrs", []):
                self._lib.dd_ipc_close(self.device.index, p)
            self._peer_ptrs = []
            self._lib.dd_destroy(self._h)
            self._h = None

    def __del__(self):
        # A finaliser cannot join a barrier (ranks collect garbage at different
        # times), so a vocab-sharded runner that was never closed keeps its
        # exchange buffer until the process exits rather than freeing memory
        # that a peer may still write into.
        try:
            if getattr(self, "world", 1) == 1:
                self.close()
        except Exception:
            pass
