"""Time the reference's own CPU path of the draft step beside its stand-ins.

TEST INFRASTRUCTURE ONLY (a measurement of the benchmark's CPU leg, never of
the product).  The benchmark's reference arm cannot run the reference itself
where the benchmark runs (the reference is a source tree without packaging
metadata, so it cannot be installed there); it runs oracle/torch_branch.py,
the reference's PyTorch-branch op sequence restated in torch CPU ops.  This
script measures, on one host and on the same workload, whether that stand-in
is as fast as the reference's own code:

* reference: ``DraftCorrectionGraphRunner`` (code/kernel/domino.py:229-508),
  imported unchanged from a checkout named by ``DOMINO_REFERENCE``, with its
  PyTorch branch (``HAS_TRITON = False``, domino.py:406-431) and its CUDA
  stream/graph calls replaced by no-ops so that it runs on the CPU, plus the
  base logits ``target.lm_head(parallel_hiddens)`` (code/dflash.py:424);
* torch branch: ``bench.cpu_block`` (oracle/torch_branch.py: lm_head,
  pure-draft prefix, rollout), the benchmark's CPU leg;
* numpy oracle: oracle/draft_oracle.py (lm_head, rollout) in fp32 numpy, the
  parity checker, which earlier served as the CPU leg.

All on every host thread, batch 1, block 16, on seeded random weights.

    DOMINO_REFERENCE=/path/to/Domino python oracle/time_reference_cpu.py --model qwen3-8b
"""
from __future__ import annotations

import argparse
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


class _Stream:
    def __init__(self, *a, **k):
        pass

    def wait_stream(self, *a, **k):
        pass


class _Graph:
    fn = None

    def replay(self):
        self.fn()


class _Ctx:
    def __init__(self, *a, **k):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--blocks", type=int, default=3)
    args = ap.parse_args()
    ref = os.environ.get("DOMINO_REFERENCE")
    if not ref:
        sys.exit("set DOMINO_REFERENCE to the root of a Domino checkout (the directory holding code/)")
    import numpy as np
    import torch

    torch.cuda.Stream = _Stream
    torch.cuda.current_stream = lambda *a, **k: _Stream()
    torch.cuda.stream = _Ctx
    torch.cuda.CUDAGraph = _Graph
    torch.cuda.graph = _Ctx
    sys.path.insert(0, os.path.join(ref, "code"))
    import kernel.domino as kd

    import bench
    from oracle.draft_oracle import round_to

    threads = bench.host_threads()
    torch.set_num_threads(threads)
    m = bench.MODELS[args.model]
    H, G, E, V, S, P = m["H"], m["G"], m["E"], m["V"], 15, 0
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    t0 = time.perf_counter()
    draft, target = bench.build_modules(H, G, E, V, torch.device("cpu"), seed=0)
    draft, target = draft.to(dt), target.to(dt)
    rng = np.random.default_rng(0)
    ph_np = round_to(rng.standard_normal((1, S, H)).astype(np.float32), "bf16")
    last = rng.integers(0, V, (1,))
    ph = torch.from_numpy(ph_np).to(dt)
    prefix = torch.from_numpy(last.reshape(1, 1))

    kd.HAS_TRITON = False
    runner = kd.DraftCorrectionGraphRunner(draft, target, 1, S, H, G, V, 1, torch.device("cpu"))
    runner.graph.fn = runner._forward_impl
    print(f"setup {time.perf_counter() - t0:.1f} s ({threads} threads, {args.dtype})", flush=True)

    def ref_block():
        with torch.inference_mode():
            base = target.lm_head(ph)              # code/dflash.py:424
            return runner(prefix, ph, base)        # code/kernel/domino.py:495-508

    ref_block()  # warm-up
    t0 = time.perf_counter()
    for _ in range(args.blocks):
        ref_block()
    t_ref = (time.perf_counter() - t0) / args.blocks
    del runner

    head = bench.cpu_head(draft, target)
    last_t = torch.from_numpy(last)
    bench.cpu_block(head, ph, last_t, P)  # warm-up
    t0 = time.perf_counter()
    for _ in range(args.blocks):
        bench.cpu_block(head, ph, last_t, P)
    t_tb = (time.perf_counter() - t0) / args.blocks
    table = head.table
    del head

    from oracle import draft_oracle as O

    def f32(t):
        return t.detach().float().numpy()

    w = O.DraftWeights(fc1=f32(draft.embed_proj[0].weight), fc2=f32(draft.embed_proj[2].weight),
                       w_ih=f32(draft.prefix_gru.weight_ih_l0), w_hh=f32(draft.prefix_gru.weight_hh_l0),
                       embed=np.zeros((1, H), np.float32), dtype=args.dtype, table=f32(table))
    lm = f32(target.lm_head.weight)

    def port_block():
        base = O.lm_head(ph_np, lm, args.dtype)
        return O.rollout(w, last.reshape(-1, 1), ph_np, base).tokens

    port_block()  # warm-up
    t0 = time.perf_counter()
    for _ in range(args.blocks):
        port_block()
    t_port = (time.perf_counter() - t0) / args.blocks
    print(f"{args.model} H={H} G={G} E={E} V={V}, batch 1, {S} draft tokens, {threads} threads")
    print(f"  reference PyTorch branch ({args.dtype}):   {t_ref:.3f} s/block = {S / t_ref:.2f} draft tok/s")
    print(f"  torch branch restated ({args.dtype}):      {t_tb:.3f} s/block = {S / t_tb:.2f} draft tok/s")
    print(f"  numpy oracle (fp32):                  {t_port:.3f} s/block = {S / t_port:.2f} draft tok/s")
    print(f"  restated / reference speed = {t_ref / t_tb:.2f}; numpy oracle / reference speed = {t_ref / t_port:.2f}")


if __name__ == "__main__":
    main()
