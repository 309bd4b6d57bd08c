"""Vocab-sharded draft step: each rank owns a slice of fc2 / lm_head rows and
the per-step argmax words are combined across GPUs inside the kernels.

* one GPU, no exchange: a handle restricted to a vocab slice picks the
  argmax over that slice (checks the global-index / base-column plumbing);
* one GPU, a peer that never publishes: the bounded wait for the other
  rank's word runs out, the kernel reports DD_STATUS_TIMEOUT and returns;
* two GPUs (skipped with fewer): two processes, each a vocab shard, give the
  tokens of the unsharded runner.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

from oracle import draft_oracle as O
from tests.gpu_helpers import TOL, oracle_weights, random_inputs, random_modules

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability(0)[0] != 10:
        pytest.fail("GPU tests need an sm_100 device")


def _sliced_rollout_check(w, prefix, ph, base, tokens, v0, v1):
    """Teacher-forced oracle over vocab rows [v0, v1) only."""
    prefix = prefix.cpu().numpy()
    ph = ph.float().cpu().numpy()
    base = base.float().cpu().numpy()
    tokens = tokens.cpu().numpy()
    B, S, _ = ph.shape
    z = O.linear(ph, w.w_z, w.fc1_bias, w.dtype)
    h = O.prefix_gru(w, prefix)
    table = w.get_table()
    fc2 = w.fc2[v0:v1]
    bias = None if w.fc2_bias is None else w.fc2_bias[v0:v1]
    exact = 0
    for t in range(S):
        s = O.linear(h, w.w_s, None, w.dtype)
        mid = O.silu(z[:, t] + s)
        logits = mid @ fc2.T + (0 if bias is None else bias) + base[:, t, v0:v1]
        own = np.argmax(logits, axis=1) + v0
        for b in range(B):
            assert v0 <= tokens[b, t] < v1
            if own[b] == tokens[b, t]:
                exact += 1
            else:
                top = logits[b].max()
                assert top - logits[b, tokens[b, t] - v0] <= TOL + TOL * abs(top)
        if t + 1 < S:
            h = O.gru_cell(table[tokens[:, t]], O.linear(h, w.w_hh, w.b_hh, w.dtype), h, w.dtype)
    return exact / (B * S)


def _handle(draft, target, B, S, H, G, V, P, table):
    from domino_b200 import _lib

    lib = _lib.load()
    cfg = _lib.DDConfig(batch=B, steps=S, hidden=H, gru_hidden=G, emb_dim=draft.embed_proj[0].out_features,
                        vocab=V, prefix_tokens=P, dtype=_lib.DD_BF16)
    h = ctypes.c_void_p()
    _lib.check(lib.dd_create(ctypes.byref(cfg), 0, ctypes.byref(h)), None, "dd_create")
    return lib, h


def _weights(runner, draft, v0, v1):
    from domino_b200 import _lib

    fc1, fc2 = runner._fc1, runner._fc2[v0:v1]
    return _lib.DDWeights(fc1=fc1.data_ptr(), fc1_ld=fc1.stride(0), fc2=fc2.data_ptr(), fc2_ld=fc2.stride(0),
                          w_hh=runner._w_hh.data_ptr(), w_hh_ld=runner._w_hh.stride(0),
                          table=runner.table.data_ptr(), table_ld=runner.table.stride(0))


def test_vocab_slice_single_gpu():
    from domino_b200 import DraftCorrectionGraphRunner, _lib

    B, H, G, E, V, S, P = 2, 128, 128, 192, 1500, 15, 1
    draft, target = random_modules(H, G, E, V, seed=5, fc2_std=0.08)
    runner = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), use_graph=False)
    lib, h = _handle(draft, target, B, S, H, G, V, P, runner.table)
    v0, v1 = 301, 1130
    _lib.check(lib.dd_set_vocab_shard(h, 0, 1, v0, v1, None), h, "shard")
    w = _weights(runner, draft, v0, v1)
    _lib.check(lib.dd_set_weights(h, ctypes.byref(w)), h, "weights")
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=3)
    out = torch.empty(B, S, dtype=torch.long, device="cuda")
    _lib.check(lib.dd_rollout(h, prefix.data_ptr(), ph.data_ptr(), base.data_ptr(), out.data_ptr(),
                              torch.cuda.current_stream().cuda_stream), h, "rollout")
    assert lib.dd_get_status(h) == 0
    frac = _sliced_rollout_check(oracle_weights(draft, target), prefix, ph, base, out, v0, v1)
    assert frac >= 0.9
    lib.dd_destroy(h)


def test_exchange_wait_is_bounded_and_reported():
    """Rank 0 of 2 whose peer never publishes: every step's wait runs out."""
    from domino_b200 import DraftCorrectionGraphRunner, _lib

    B, H, G, E, V, S, P = 1, 64, 64, 96, 800, 3, 1
    draft, target = random_modules(H, G, E, V, seed=9)
    runner = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0), use_graph=False)
    lib, h = _handle(draft, target, B, S, H, G, V, P, runner.table)
    sink = torch.zeros(4096, dtype=torch.int64, device="cuda")  # stands in for the peer's buffer
    peers = (ctypes.c_void_p * 2)(None, sink.data_ptr())
    _lib.check(lib.dd_set_vocab_shard(h, 0, 2, 0, V // 2, peers), h, "shard")
    _lib.check(lib.dd_set_exchange_timeout(h, 20_000_000), h, "timeout")  # 20 ms
    w = _weights(runner, draft, 0, V // 2)
    _lib.check(lib.dd_set_weights(h, ctypes.byref(w)), h, "weights")
    prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=1)
    out = torch.empty(B, S, dtype=torch.long, device="cuda")
    _lib.check(lib.dd_rollout(h, prefix.data_ptr(), ph.data_ptr(), base.data_ptr(), out.data_ptr(),
                              torch.cuda.current_stream().cuda_stream), h, "rollout")
    status = lib.dd_get_status(h)
    assert status >= 0 and status & _lib.DD_STATUS_TIMEOUT
    # the context is still usable: an unsharded call afterwards works
    assert (out >= 0).all() and (out < V).all()
    again = runner(prefix, ph, base)
    assert runner.status() == 0 and again.shape == (B, S)
    lib.dd_destroy(h)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from domino_b200 import DraftCorrectionGraphRunner

        B, H, G, E, V, S, P = 3, 256, 256, 384, 6007, 15, 1
        draft, target = random_modules(H, G, E, V, seed=21, fc2_std=0.08, device=f"cuda:{rank}")
        prefix, ph, base = random_inputs(B, S, H, V, P, target, seed=4, device=f"cuda:{rank}")
        r = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", rank),
                                       vocab_shard=True)
        outs = [r(prefix, ph, base).cpu().numpy() for _ in range(2)]
        status = r.status()
        verify, _ = r.draft_block(prefix[:, 0], ph)
        status |= r.status()
        dist.barrier()
        r.close()
        # numpy only: torch CPU tensors cross the queue as shared-memory fds,
        # which are gone once this process exits
        res = {"rank": rank, "outs": outs, "verify": verify.cpu().numpy(), "status": status,
               "range": (r.vocab_begin, r.vocab_end)}
        # A wide z / lm_head pass (20 rows x 17 positions: two passes of 176,
        # two epilogue warpgroups) whose last pass exchanges the pure-draft
        # prefix argmax words across the ranks.
        B2, P2 = 20, 3
        g2 = torch.Generator(device=f"cuda:{rank}").manual_seed(13)
        ph2 = torch.randn(B2, P2 - 1 + S, H, generator=g2, device=f"cuda:{rank}").to(torch.bfloat16)
        last2 = torch.randint(0, V, (B2,), generator=g2, device=f"cuda:{rank}")
        r2 = DraftCorrectionGraphRunner(draft, target, B2, S, H, G, V, P2, torch.device("cuda", rank),
                                        vocab_shard=True)
        verify2, _ = r2.draft_block(last2, ph2)
        res["status2"] = r2.status()
        res["verify2"] = verify2.cpu().numpy()
        dist.barrier()
        r2.close()
        if rank == 0:
            ref2 = DraftCorrectionGraphRunner(draft, target, B2, S, H, G, V, P2, torch.device("cuda", 0))
            res["ref2"] = ref2.draft_block(last2, ph2)[0].cpu().numpy()
        if rank == 0:
            ref = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P, torch.device("cuda", 0))
            res["ref"] = ref(prefix, ph, base).cpu().numpy()
            res["w"] = oracle_weights(draft, target)
            res["inputs"] = (prefix.cpu().numpy(), ph.float().cpu().numpy(), base.float().cpu().numpy())
        q.put(res)
    finally:
        dist.destroy_process_group()


def test_vocab_shard_two_gpus_matches_unsharded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda d: d["rank"])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0]["range"] == (0, 3004) and res[1]["range"] == (3004, 6007)
    for d in res:
        assert d["status"] == 0
        assert np.array_equal(d["outs"][0], d["outs"][1])
    # every rank produced the same tokens
    assert np.array_equal(res[0]["outs"][0], res[1]["outs"][0])
    assert np.array_equal(res[0]["verify"], res[1]["verify"])
    from tests.gpu_helpers import log_parity, teacher_forced_check

    prefix, ph, base = res[0]["inputs"]
    # the shards split the fp32 sums at other points than one GPU does, so a
    # near-tie may go either way
    teacher_forced_check(res[0]["w"], prefix, ph, base, res[0]["outs"][0], min_exact=0.95)
    # equal to the unsharded runner except at near-ties
    differ = float(np.mean(res[0]["outs"][0] != res[0]["ref"]))
    log_parity(f"2-GPU vocab shard: {1 - differ:.3f} of the tokens equal the unsharded runner's")
    assert differ <= 0.1
    assert np.array_equal(res[0]["verify"][:, 0], prefix[:, 0])
    # batch 20 with a pure-draft prefix: the wide z / lm_head pass, sharded
    for d in res:
        assert d["status2"] == 0
    assert np.array_equal(res[0]["verify2"], res[1]["verify2"])
    P2 = 3
    assert np.array_equal(res[0]["verify2"][:, :P2], res[0]["ref2"][:, :P2])  # last token + prefix argmax
    differ2 = float(np.mean(res[0]["verify2"][:, P2:] != res[0]["ref2"][:, P2:]))
    log_parity(f"2-GPU vocab shard, batch 20 with a 2-token prefix: prefix tokens exact, "
               f"{1 - differ2:.3f} of the drafted tokens equal the unsharded runner's")
    assert differ2 <= 0.1
