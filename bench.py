#!/usr/bin/env python
"""Benchmark of the Domino per-block draft step on B200.

One step = the draft side of one speculative block (block 16) for every row
of the batch, through the public API (``DraftCorrectionGraphRunner.draft_block``
+ ``.accept``, i.e. ``dd_draft_block`` + ``dd_accept``):

  lm_head base logits for the 15 draft positions  ->  z = hiddens @ W_z^T
  ->  h0 = GRU(last token)  ->  15 x [ s = h W_s^T -> SiLU mid -> fc2 + base
  -> argmax -> GRU step ]  ->  greedy acceptance against the target's tokens.

Workload (default): the Qwen3-8B-shaped draft head, bf16, batch 1 per GPU,
H = G = 4096, E = 12288, V = 151936, seeded random-init weights N(0, 0.02),
hidden states N(0, 1), target tokens equal to the draft's own tokens for the
first k ~ U{0..15} positions and different after.  The weights streamed every
step (8.7 GB) are ~70x the 126 MB L2, so no L2 flush is needed between steps.

Multi-GPU: one process per GPU, each runs its own batch (requests are
independent; no collective on the data path): weak scaling.  Times are CUDA
events on each rank, max over ranks.

``--impl reference`` times the reference's CPU path of the draft step on this
host's cores, on the same workload, config, steps and warm-up: the op
sequence of its PyTorch branch (code/kernel/domino.py:374-431) restated in
oracle/torch_branch.py, whose tokens equal the reference's.  The reference
itself is a Python source tree without packaging metadata (no setup.py or
pyproject.toml), so it cannot be installed where this benchmark runs.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "draft tokens/sec per GPU & µs per draft block (block=16) at 1/2/4/8 B200; HBM/TC roofline %"
MODELS = {
    "qwen3-8b": dict(H=4096, G=4096, E=12288, V=151936),
    "qwen3-4b": dict(H=2560, G=2560, E=6912, V=151936),
    "qwen3.6-27b": dict(H=5120, G=5120, E=17408, V=151936),
}
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0            # burst; sustained under the power cap ~1400
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=sorted(MODELS), default="qwen3-8b")
    ap.add_argument("--batch", type=int, default=1, help="rows per GPU (weak scaling)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="split this many rows over the ranks instead (strong scaling)")
    ap.add_argument("--vocab-shard", action="store_true",
                    help="every rank runs the same rows on its slice of the vocab (strong scaling)")
    ap.add_argument("--emb-dim", type=int, default=None, help="override E (correction-MLP width)")
    ap.add_argument("--hidden", type=int, default=None, help="override H = G (small profiling cases)")
    ap.add_argument("--vocab", type=int, default=None,
                    help="override V (e.g. one rank's share of a vocab-sharded head, measured on one GPU)")
    ap.add_argument("--block", type=int, default=16)
    ap.add_argument("--prefix-len", type=int, default=0, help="pure_draft_prefix_len")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=150.0)
    ap.add_argument("--spec-loop", action="store_true",
                    help="the end-to-end synthetic spec-decode loop instead of the draft step: a random-init "
                         "Qwen3-8B-shaped target (36 layers) verifying the drafter's blocks")
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--new-tokens", type=int, default=2048)
    ap.add_argument("--draft-layers", type=int, default=5)
    ap.add_argument("--requests", type=int, default=2, help="--spec-loop: requests per GPU")
    return ap.parse_args()


def shapes(args):
    m = dict(MODELS[args.model])
    if args.emb_dim:
        m["E"] = args.emb_dim
    if args.hidden:
        m["H"] = m["G"] = args.hidden
    if args.vocab:
        m["V"] = args.vocab
    S = args.block - 1 - args.prefix_len
    return m["H"], m["G"], m["E"], m["V"], S, args.prefix_len


def algorithmic_bytes(B, H, G, E, V, S, P, w=2):
    """Bytes the draft step must move per block (weights once per use)."""
    K = S + P
    weights = V * H + E * H + S * (E * G + V * E) + max(0, S + P - 1) * 3 * G * G
    acts = 2 * B * K * V * 2          # base logits written + read
    acts += B * (S + P) * 3 * G * 2   # gathered table rows
    acts += B * K * H * 2 + B * K * E * 2 * 2  # hidden states read, z written + read
    return weights * w + acts


def fc2_bytes(B, E, V, w=2):
    """Algorithmic bytes of one fc2 phase launch: fc2 once + one base-logit row per batch row."""
    return V * E * w + B * V * 2


def workload_name(args, B, H, G, E, V, S, P):
    return (f"{args.model}-shaped Domino draft head, bf16, batch {B}/GPU, block {args.block} "
            f"({S} draft + {P} prefix tokens), H={H} G={G} E={E} V={V}")


def bench_config(args, B, rows_total, world, sharded, H, G, E, V, S, P):
    """The ``config`` dict of the JSON line; both arms print the same one."""
    return {
        "workload": workload_name(args, B, H, G, E, V, S, P),
        "batch_per_gpu": B, "global_batch": rows_total, "block": args.block, "seq_len": args.block,
        "parallelism": (f"vocab{world} (fc2 / lm_head rows sharded; argmax words exchanged over NVLink "
                        "inside the kernels)") if sharded else f"dp{world} (request batch sharded, no collective)",
        "l2": "no flush: inputs larger than L2 (the weights streamed every step are ~70x the 126 MB L2)",
    }


def measured_peak_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_peak_tflops():
    """(burst, sustained) dense bf16 TFLOP/s of this pool's B200s (cuBLAS), or the fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback"


def zlm_passes(rows):
    """X rows per z / lm_head pass and the pass count, as the library splits them
    (at most 256 per pass, as equal as the 16-row MMA granularity allows)."""
    passes = -(-rows // 256)
    per = -(-rows // passes)
    return -(-per // 16) * 16, passes


def measure_cublas_linear(device, n, k, r, iters=10):
    """cuBLAS (torch F.linear) on the same GEMM as one z / lm_head pass:
    [n x k] . [k x r]^T, bf16, two weight buffers alternated (each > L2)."""
    import torch
    import torch.nn.functional as F

    g = torch.Generator(device=device).manual_seed(11)
    ws = [torch.randn(r, k, generator=g, device=device, dtype=torch.bfloat16) for _ in range(2)]
    x = torch.randn(n, k, generator=g, device=device, dtype=torch.bfloat16)
    for i in range(3):
        F.linear(x, ws[i % 2])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for i in range(iters):
        F.linear(x, ws[i % 2])
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / iters
    del ws, x
    torch.cuda.empty_cache()
    return us


def committed_traffic(model, B, H, E):
    """Per-launch DRAM bytes of the fc2 phase from the committed ncu summary, or None.

    profiles/fc2_phase_traffic.txt holds lines ``<model>:B<b>:H<h>:E<e> <bytes> ...``.
    """
    path = os.path.join(ROOT, "profiles", "fc2_phase_traffic.txt")
    key = f"{model}:B{B}:H{H}:E{E}"
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == key:
                    return float(parts[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"dd_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- distributed
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------- model construction
def build_modules(H, G, E, V, device, seed):
    import torch
    import torch.nn as nn

    class DraftHead(nn.Module):
        def __init__(self):
            super().__init__()
            self.prefix_gru = nn.GRU(H, G, num_layers=1, batch_first=True, bias=False, device=device,
                                     dtype=torch.bfloat16)
            self.embed_proj = nn.Sequential(
                nn.Linear(H + G, E, bias=False, device=device, dtype=torch.bfloat16), nn.SiLU(),
                nn.Linear(E, V, bias=False, device=device, dtype=torch.bfloat16))

    class Target(nn.Module):
        def __init__(self):
            super().__init__()
            self.model = nn.Module()
            self.model.embed_tokens = nn.Embedding(V, H, device=device, dtype=torch.bfloat16)
            self.lm_head = nn.Linear(H, V, bias=False, device=device, dtype=torch.bfloat16)

    g = torch.Generator(device=device).manual_seed(seed)
    draft, target = DraftHead(), Target()
    with torch.no_grad():
        for p in list(draft.parameters()) + [target.lm_head.weight]:
            p.normal_(0.0, 0.02, generator=g)
        target.model.embed_tokens.weight.normal_(0.0, 1.0, generator=g)
    return draft.eval(), target.eval()


# ---------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    from domino_b200 import DraftCorrectionGraphRunner, _lib

    from domino_b200.parallel import max_over_ranks, shard_rows

    H, G, E, V, S, P = shapes(args)
    B = args.batch
    if args.global_batch is not None:
        B = shard_rows(args.global_batch, world, rank)[1]
        if B < 1:
            raise SystemExit(f"--global-batch {args.global_batch} leaves rank {rank} without rows")
    K = S + P
    sharded = args.vocab_shard and world > 1
    # Vocab shards must hold the same model and see the same requests.
    wseed = args.seed if sharded else args.seed + 17 * rank
    draft, target = build_modules(H, G, E, V, device, wseed)
    runner = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P + 1, device, use_graph=False,
                                        vocab_shard=sharded)
    V_local = runner.vocab_end - runner.vocab_begin
    lib = _lib.load()

    # Synthetic inputs: a pool of blocks; the target agrees with the draft on
    # the first k ~ U{0..S} positions (the path is deterministic, so a first
    # pass gives the draft tokens the posterior is built from).
    n_pool = 8
    g = torch.Generator(device=device).manual_seed(args.seed + 1000 + (0 if sharded else rank))
    ph_pool = [torch.randn(B, K, H, generator=g, device=device).to(torch.bfloat16) for _ in range(n_pool)]
    last_pool = [torch.randint(0, V, (B,), generator=g, device=device) for _ in range(n_pool)]
    post_pool, kk = [], []
    for i in range(n_pool):
        verify, _ = runner.draft_block(last_pool[i], ph_pool[i])
        k = torch.randint(0, S + 1, (B,), generator=g, device=device)
        post = torch.randint(0, V, (B, K + 1), generator=g, device=device)
        pos = torch.arange(K + 1, device=device).unsqueeze(0)
        agree = pos < (P + k).unsqueeze(1)
        shifted = torch.cat([verify[:, 1:], verify[:, -1:]], 1)
        post = torch.where(agree, shifted, torch.where(post == shifted, (post + 1) % V, post))
        post_pool.append(post)
        kk.append(k)
    torch.cuda.synchronize()
    base_buf = torch.empty(B, K, V_local, dtype=torch.bfloat16, device=device)

    def step(i):
        verify, _ = runner.draft_block(last_pool[i], ph_pool[i], base_buf)
        return runner.accept(verify, post_pool[i])

    # ---- value: device-resident inputs
    for i in range(args.warmup):
        step(i % n_pool)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    # All ranks leave the barrier together (vocab shards wait on one another).
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record()
    hist = [0] * (S + 2)
    accs = []
    for i in range(args.steps):
        acc, _ = step(i % n_pool)
        accs.append(acc)
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    for a in accs[: n_pool]:
        for x in a.tolist():
            hist[min(x + 1, S + 1)] += 1

    # ---- e2e: pinned host inputs, H2D + D2H inside the timed region
    ph_host = [t.cpu().pin_memory() for t in ph_pool]
    last_host = [t.cpu().pin_memory() for t in last_pool]
    post_host = [t.cpu().pin_memory() for t in post_pool]
    ph_dev = torch.empty_like(ph_pool[0])
    last_dev = torch.empty_like(last_pool[0])
    post_dev = torch.empty_like(post_pool[0])
    verify_host = torch.empty(B, K + 1, dtype=torch.long).pin_memory()
    acc_host = torch.empty(B, dtype=torch.int32).pin_memory()
    bonus_host = torch.empty(B, dtype=torch.long).pin_memory()

    def e2e_step(i):
        ph_dev.copy_(ph_host[i], non_blocking=True)
        last_dev.copy_(last_host[i], non_blocking=True)
        post_dev.copy_(post_host[i], non_blocking=True)
        verify, _ = runner.draft_block(last_dev, ph_dev, base_buf)
        acc, bonus = runner.accept(verify, post_dev)
        verify_host.copy_(verify, non_blocking=True)
        acc_host.copy_(acc, non_blocking=True)
        bonus_host.copy_(bonus, non_blocking=True)

    for i in range(min(args.warmup, 3)):
        e2e_step(i % n_pool)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev2.record()
    for i in range(args.steps):
        e2e_step(i % n_pool)
    ev3.record()
    torch.cuda.synchronize()
    ms_e2e = ev2.elapsed_time(ev3)
    clk = clocks.stop() if rank == 0 else None
    h2d = ph_pool[0].numel() * 2 + B * 8 + B * (K + 1) * 8
    d2h = B * (K + 1) * 8 + B * 4 + B * 8

    # ---- per-launch timing (events around every launch; separate loop)
    lib.dd_set_timing(runner._h, 1)
    n_timed_blocks = 3
    for i in range(n_timed_blocks):
        step(i % n_pool)
    torch.cuda.synchronize()
    kinds = (ctypes.c_int32 * 4096)()
    durs = (ctypes.c_float * 4096)()
    n = _lib.check(lib.dd_read_timing(runner._h, kinds, durs, 4096), runner._h, "dd_read_timing")
    lib.dd_set_timing(runner._h, 0)
    per_kind = {}
    for i in range(n):
        per_kind.setdefault(_lib.PHASES.get(kinds[i], str(kinds[i])), []).append(durs[i])
    launches_per_step = n / n_timed_blocks + 1  # + the accept kernel
    status = runner.status()

    # ---- reduce over ranks: the slowest rank's time; rows summed
    ms, ms_e2e, status_f = max_over_ranks([ms, ms_e2e, float(status)], device=device)
    # After the timed region, on more than one rank with request batches: the
    # vocab-sharded path on the same ranks (every rank takes part).
    shard_check = vocab_shard_check(device, world, rank) if (world > 1 and not sharded) else None
    status = int(status_f)
    rows_total = B * world
    if sharded:
        rows_total = B  # every rank drafts the same rows
    elif world > 1:
        rt = torch.tensor([B], dtype=torch.int64, device=device)
        dist.all_reduce(rt)
        rows_total = int(rt.item())

    if rank == 0:
        tokens = rows_total * S * args.steps
        value = tokens / (ms / 1e3)
        e2e_value = tokens / (ms_e2e / 1e3)
        peak, peak_src = measured_peak_hbm()
        fc2_ms = statistics.mean(per_kind.get("fc2", [float("nan")]))
        fc2_b = fc2_bytes(B, E, V_local)
        achieved = fc2_b / (fc2_ms / 1e3) / 1e9
        step_b = algorithmic_bytes(B, H, G, E, V, S, P) - (V - V_local) * (H + S * E) * 2  # this rank's weights
        step_ms = ms / args.steps
        traffic = committed_traffic(args.model, B, H, E)
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "draft tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(step_ms, 4),
            "us_per_block": round(step_ms * 1e3, 1),
            "per_gpu_value": round(value / world, 2),
            "higher_is_better": True,
            "scaling": "strong" if (args.global_batch is not None or sharded) else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: seeded random-init weights N(0,0.02), hidden states N(0,1), "
                    "target tokens = draft tokens for the first k~U{0..15} positions",
            "config": bench_config(args, B, rows_total, world, sharded, H, G, E, V, S, P),
            "roofline": {
                "bound": "hbm", "kernel": "fc2 phase (gemv_stream_kernel PH_FC2)",
                "achieved": round(achieved, 1), "peak": peak, "peak_source": peak_src, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "algorithmic_bytes_per_launch": fc2_b, "avg_launch_ms": round(fc2_ms, 4),
            },
            "step_roofline": {
                "algorithmic_bytes_per_step": step_b,
                "achieved_gbs": round(step_b / (step_ms / 1e3) / 1e9, 1),
                "frac": round(step_b / (step_ms / 1e3) / 1e9 / peak, 4),
            },
            "phase_ms": {k: round(statistics.mean(v), 4) for k, v in sorted(per_kind.items())},
            "phase_launches_per_block": {k: len(v) / n_timed_blocks for k, v in sorted(per_kind.items())},
            "e2e": {"value": round(e2e_value, 2), "unit": "draft tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e / args.steps, 4)},
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "accept_hist": hist,
            "device_status": status,
            "clocks": clk,
        }
        if shard_check is not None:
            line["vocab_shard_check"] = shard_check
        if world == 1:
            line["verify_roofline"] = measure_verify(device, V, peak)
            # The z / lm_head pass: tensor-bound once its passes are wide; its
            # FLOPs against the measured cuBLAS peaks and against cuBLAS on
            # the identical GEMM shape (the same rows per pass).
            rows = B * K
            n_pass, passes = zlm_passes(rows)
            zlm_us = statistics.mean(per_kind.get("zlm", [float("nan")])) * 1e3
            flops = 2.0 * rows * H * (V_local + E) / passes  # valid rows only
            burst, sustained, tf_src = measured_peak_tflops()
            tflops = flops / (zlm_us / 1e6) / 1e12
            wbytes = (V_local + E) * H * 2 + rows * (H + V_local + E) * 2 / passes  # weights + X + outputs
            gbs = wbytes / (zlm_us / 1e6) / 1e9
            cublas_us = measure_cublas_linear(device, n_pass, H, V_local + E)
            tensor = n_pass > 64  # wide passes: the tensor pipe binds; narrow ones stream the weights
            line["zlm_roofline"] = {
                "bound": "tensor" if tensor else "hbm",
                "kernel": "z / lm_head pass (gemv_stream_kernel PH_ZLM)",
                "gemm": f"[{n_pass} x {H}] . [{H} x {V_local + E}]", "passes_per_block": passes,
                "flops_per_launch": flops, "algorithmic_bytes_per_launch": int(wbytes),
                "avg_launch_us": round(zlm_us, 1), "tflops": round(tflops, 1), "gbs": round(gbs, 1),
                "achieved": round(tflops if tensor else gbs, 1), "unit": "TFLOP/s" if tensor else "GB/s",
                "peak": burst if tensor else peak, "peak_source": tf_src if tensor else peak_src,
                "frac": round(tflops / burst if tensor else gbs / peak, 4),
                "frac_of_sustained_tflops": round(tflops / sustained, 4),
                "cublas_same_gemm_us": round(cublas_us, 1), "cublas_over_ours": round(cublas_us / zlm_us, 3),
            }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, draft, target, ph_pool[0], last_pool[0], budget_s=30.0)
        print(json.dumps(line), flush=True)
    runner.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def vocab_shard_check(device, world, rank, seed=7, B=4, S=15, H=512, E=1024, V=151936):
    """The vocab-sharded draft block across all `world` ranks of this job (fc2
    and lm_head rows split, per-step argmax exchanged over NVLink inside the
    kernels) on one small head with the full vocabulary, every rank holding the
    same weights and inputs: whether every rank drafts the same tokens, how many
    equal the unsharded runner's (rank 0; the shards split the fp32 sums at
    other points, so a near-tie may go either way), the status words, and the
    sharded block's time (CUDA events, max over ranks)."""
    import torch
    import torch.distributed as dist

    from domino_b200 import DraftCorrectionGraphRunner
    from domino_b200.parallel import max_over_ranks

    draft, target = build_modules(H, H, E, V, device, seed)
    r = DraftCorrectionGraphRunner(draft, target, B, S, H, H, V, 1, device, use_graph=False, vocab_shard=True)
    g = torch.Generator(device=device).manual_seed(seed + 1)
    ph = torch.randn(B, S, H, generator=g, device=device).to(torch.bfloat16)
    last = torch.randint(0, V, (B,), generator=g, device=device)
    for _ in range(2):
        verify, _ = r.draft_block(last, ph)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    a.record()
    for _ in range(5):
        verify, _ = r.draft_block(last, ph)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / 5
    status = r.status()
    gathered = [torch.empty_like(verify) for _ in range(world)]
    dist.all_gather(gathered, verify)
    same = all(torch.equal(gathered[0], t) for t in gathered)
    us, status_f = max_over_ranks([us, float(status)], device=device)
    r.close()
    out = None
    if rank == 0:
        ref = DraftCorrectionGraphRunner(draft, target, B, S, H, H, V, 1, device, use_graph=False)
        v1, _ = ref.draft_block(last, ph)
        out = {"ranks": world, "head": f"H=G={H} E={E} V={V}, batch {B}, block {S + 1}",
               "tokens_equal_across_ranks": bool(same),
               "fraction_equal_to_unsharded": round(float((v1 == verify).float().mean()), 4),
               "status_max": int(status_f), "us_per_block_sharded": round(us, 1)}
        ref.close()
    dist.barrier()
    return out


def measure_verify(device, V, peak, B=16, K1=16, iters=20):
    """Device time of the fused target verify + acceptance (dd_verify_accept)
    over [B, K1, V] bf16 logits, rotating through four buffers (4 x 78 MB at
    the default shape, more than L2), one CUDA-event pair around each launch."""
    import torch

    from domino_b200 import DraftCorrectionGraphRunner

    draft, target = build_modules(64, 64, 64, V, device, seed=5)
    r = DraftCorrectionGraphRunner(draft, target, B, 15, 64, 64, V, 1, device, use_graph=False)
    g = torch.Generator(device=device).manual_seed(7)
    logits = [torch.randn(B, K1, V, generator=g, device=device).to(torch.bfloat16) for _ in range(4)]
    verify = torch.randint(0, V, (B, K1), generator=g, device=device)
    for i in range(3):
        r.verify_accept(logits[i % 4], verify)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(evs):
        a.record()
        r.verify_accept(logits[i % 4], verify)
        b.record()
    torch.cuda.synchronize()
    us = statistics.mean(a.elapsed_time(b) for a, b in evs) * 1e3
    nbytes = B * K1 * V * 2
    r.close()
    return {"kernel": "verify_accept_kernel (dd_verify_accept)", "logits": f"[{B}, {K1}, {V}] bf16",
            "algorithmic_bytes_per_launch": nbytes, "avg_launch_us": round(us, 2),
            "achieved": round(nbytes / (us / 1e6) / 1e9, 1), "peak": peak, "unit": "GB/s",
            "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4),
            "l2": "four logits buffers rotated (4 x the bytes above > 126 MB L2)"}


# ---------------------------------------------------------------- CPU leg
def cpu_head(draft, target):
    """Host copies of the head for the CPU leg (oracle/torch_branch.py: the
    reference's PyTorch-branch op sequence in torch CPU kernels).  The
    one-time W_ih table is built where the modules live (the GPU) and copied."""
    import torch
    import torch.nn.functional as F

    from oracle import torch_branch as TB

    gru = draft.prefix_gru
    with torch.inference_mode():
        table = F.linear(target.model.embed_tokens.weight, gru.weight_ih_l0,
                         gru.bias_ih_l0 if gru.bias else None).cpu()
    return TB.head_from_modules(draft, target, table=table)


def cpu_block(head, ph, last, P):
    """One block of the CPU leg: lm_head, pure-draft prefix, rollout (code/dflash.py:424-439)."""
    from oracle import torch_branch as TB

    return TB.draft_block(head, last, ph, P)


def cpu_baseline(args, draft, target, ph, last, budget_s):
    """Time the CPU leg on this host's cores on blocks of the same workload."""
    import torch

    H, G, E, V, S, P = shapes(args)
    threads = host_threads()
    head = cpu_head(draft, target)
    ph_c, last_c = ph.cpu(), last.cpu()
    cpu_block(head, ph_c, last_c, P)  # warm-up
    # A bounded sample: whole blocks until about a third of the budget (10 s of
    # the default 30 s) has passed, at least one block and at most 64.
    blocks, t0 = 0, time.perf_counter()
    while True:
        cpu_block(head, ph_c, last_c, P)
        blocks += 1
        if time.perf_counter() - t0 > budget_s / 3 or blocks >= 64:
            break
    dt = time.perf_counter() - t0
    return {
        "value": round(blocks * args.batch * S / dt, 4), "unit": "draft tokens/s", "cores": threads,
        "kind": "port", "threads": f"torch CPU, {torch.get_num_threads()} threads",
        "sample": f"{blocks} full block(s) of the same workload (batch {args.batch}, {S} draft tokens each) "
                  f"through oracle/torch_branch.py (the reference's PyTorch-branch op sequence, bf16 torch CPU "
                  f"kernels), {dt:.1f} s",
    }


def host_threads() -> int:
    """Use every host thread for the CPU leg (torchrun sets OMP_NUM_THREADS=1)."""
    import torch

    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(n)
    except Exception:
        pass
    return n


def run_reference(args):
    """The reference arm: the reference's PyTorch-branch op sequence
    (oracle/torch_branch.py) on this host's cores, on the same workload,
    config, steps and warm-up as our arm at this N.  Rank 0 alone runs it; the
    other ranks exit without work."""
    world, rank, local = dist_env()
    if rank != 0:
        return
    threads = host_threads()
    import torch

    from domino_b200.parallel import shard_rows

    H, G, E, V, S, P = shapes(args)
    B = args.batch
    sharded = args.vocab_shard and world > 1
    if args.global_batch is not None:
        B = shard_rows(args.global_batch, world, 0)[1]
        rows_total = args.global_batch
    elif sharded:
        rows_total = B
    else:
        rows_total = B * world
    K = S + P
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    # Weights are generated on the GPU only for speed; everything timed runs on the host.
    draft, target = build_modules(H, G, E, V, dev, args.seed)
    head = cpu_head(draft, target)
    del draft, target
    g = torch.Generator().manual_seed(args.seed)
    blocks = [(torch.randn(rows_total, K, H, generator=g).to(torch.bfloat16),
               torch.randint(0, V, (rows_total,), generator=g)) for _ in range(2)]
    t0 = time.perf_counter()
    cpu_block(head, blocks[0][0], blocks[0][1], P)
    t_block = time.perf_counter() - t0
    # A bounded sample: all requested steps unless they would take longer
    # than the budget (then as many whole blocks as fit).
    n_steps = max(1, min(args.steps, int(args.cpu_budget_s / max(t_block, 1e-3))))
    n_warm = max(0, args.warmup - 1)  # the sizing block above was the first warm-up step
    for i in range(n_warm):
        cpu_block(head, *blocks[i % 2], P)
    t0 = time.perf_counter()
    for i in range(n_steps):
        cpu_block(head, *blocks[i % 2], P)
    dt = time.perf_counter() - t0
    value = n_steps * rows_total * S / dt
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "draft tokens/s",
        "n_gpus": world,
        "steps": n_steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / n_steps * 1e3, 2),
        "higher_is_better": True,
        "scaling": "strong" if (args.global_batch is not None or sharded) else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded random-init weights N(0,0.02), hidden states N(0,1), "
                "target tokens = draft tokens for the first k~U{0..15} positions",
        "config": bench_config(args, B, rows_total, world, sharded, H, G, E, V, S, P),
        "cpu_baseline": {"value": round(value, 4), "unit": "draft tokens/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{n_steps} whole block(s) of all {rows_total} rows (of {args.steps} requested; "
                                   f"capped at ~{args.cpu_budget_s:.0f} s) through oracle/torch_branch.py (the "
                                   "reference's PyTorch-branch op sequence, code/kernel/domino.py:374-431, in bf16 "
                                   "torch CPU kernels; its tokens equal the reference's), all host threads, rank 0 "
                                   "only"},
        "e2e": {"value": round(value, 4), "unit": "draft tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- end-to-end loop
def _random_stack(cls, cfg, device, seed):
    """A stack module built on the device in bf16 with seeded N(0, 0.02) weights (norms 1)."""
    import torch

    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            m = cls(cfg)
    finally:
        torch.set_default_dtype(prev)
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("norm.weight"):
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=g)
    return m.eval()


def run_spec_loop(args):
    """The end-to-end synthetic spec-decode workload: per GPU, ``--requests``
    requests (default 2) of ``--prompt-len`` random ids, ``--new-tokens``
    greedy tokens in blocks of 16, a random-init Qwen3-8B-shaped target (36
    layers, H 4096, 32 q / 8 kv heads) verifying a DFlash drafter with the
    Qwen3-8B-shaped Domino head.  One process per GPU, each with its own
    requests (weak scaling); times are CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist

    from domino_b200 import DraftCorrectionGraphRunner
    from domino_b200.parallel import max_over_ranks
    from domino_b200.spec_decode import spec_generate
    from domino_b200.stack import DFlashBackbone, StackConfig, TargetLM, build_target_layer_ids

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=600),
                                device_id=device)
    H, G, E, V, S, P = shapes(args)
    B = args.requests
    tcfg = StackConfig(vocab_size=V, hidden_size=H, intermediate_size=3 * H, num_hidden_layers=36,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=H // 32, rope_theta=1e6)
    dcfg = StackConfig(vocab_size=V, hidden_size=H, intermediate_size=3 * H, num_hidden_layers=args.draft_layers,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=H // 32, rope_theta=1e6,
                       block_size=args.block, target_layer_ids=build_target_layer_ids(36, args.draft_layers),
                       mask_token_id=V - 1, emb_dim=E, gru_hidden_dim=G, pure_draft_prefix_len=P)
    target = _random_stack(TargetLM, tcfg, device, args.seed)
    draft = _random_stack(DFlashBackbone, dcfg, device, args.seed + 1)
    runner = DraftCorrectionGraphRunner(draft, target, B, S, H, G, V, P + 1, device, use_graph=False)
    g = torch.Generator().manual_seed(args.seed + 100 + rank)
    prompts = [torch.randint(0, V - 1, (args.prompt_len,), generator=g) for _ in range(B)]
    spec_generate(draft, target, runner, prompts, 64)  # warm-up
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    res = spec_generate(draft, target, runner, prompts, args.new_tokens, time_blocks=True)
    clk = clocks.stop() if rank == 0 else None
    status = runner.status()
    drafted = res.blocks * B * S
    generated = sum(res.num_output_tokens)
    decode_ms, draft_ms, verify_ms, status_f = max_over_ranks([res.decode_ms, res.draft_ms, res.verify_ms,
                                                               float(status)], device=device)
    sums = torch.tensor([drafted, generated, res.blocks], dtype=torch.float64, device=device)
    hist = torch.zeros(args.block + 2, dtype=torch.float64, device=device)
    for accs in res.acceptance_lengths:
        for a in accs:
            hist[min(a, args.block + 1)] += 1
    if world > 1:
        dist.all_reduce(sums)
        dist.all_reduce(hist)
    if rank == 0:
        drafted_all, generated_all, blocks_all = (float(x) for x in sums.tolist())
        line = {
            "metric": "end-to-end spec decode: draft tokens/s and generated tokens/s (CUDA events)",
            "value": round(drafted_all / (draft_ms / 1e3), 2), "unit": "draft tokens/s",
            "generated_tokens_per_s": round(generated_all / (decode_ms / 1e3), 2),
            "n_gpus": world, "requests_per_gpu": B, "higher_is_better": True, "scaling": "weak",
            "dtype": "bf16", "data": "synthetic: random-init Qwen3-8B-shaped target and drafter, random prompt ids",
            "config": {"workload": f"spec decode, {B} requests/GPU, prompt {args.prompt_len}, {args.new_tokens} new "
                                   f"tokens, block {args.block}; target Qwen3-8B-shaped (36 layers, H={H}, 32 q / 8 "
                                   f"kv heads); drafter {args.draft_layers} DFlash layers + Domino head (E={E}, G={G})",
                       "parallelism": f"dp{world} (requests sharded, no collective)"},
            "decode_ms": round(decode_ms, 1), "draft_ms": round(draft_ms, 1), "verify_ms": round(verify_ms, 1),
            "blocks_per_gpu": res.blocks,
            "ms_per_block": round(decode_ms / res.blocks, 3),
            "draft_ms_per_block": round(draft_ms / res.blocks, 3),
            "verify_ms_per_block": round(verify_ms / res.blocks, 3),
            "accept_len_hist": [int(x) for x in hist.tolist()],
            "mean_accept_len": round(sum(i * x for i, x in enumerate(hist.tolist())) / max(1.0, sum(hist.tolist())), 4),
            "device_status": int(status_f), "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    runner.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.spec_loop:
        run_spec_loop(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
