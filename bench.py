"""Benchmark: ragged paged-attention decode on B200 (tok/s and achieved HBM bandwidth).

Workload (per GPU): the batch-64 decode configuration — 64 sequences, one query token each,
contexts uniform in [128, 4096], Qwen2.5-3B GQA geometry (16 query heads, 2 KV heads,
head_dim 128, scale 1/sqrt(128)), page size 16, pool = total pages x 1.1 + 8 scratch pages,
block tables scattered by a seeded permutation, bf16 N(0,1) data.  One step = append the 64
new K/V rows (Cache.write) + ragged_attention_direct over the batch.

Multi-GPU (torchrun, one process per GPU): requests are sharded by context length (LPT) so
every rank holds its requests' pages; no collective on the data path (weak scaling: 64
requests per GPU).  Timing is on the device with CUDA events, max over ranks.

L2: each rank keeps R independent batches (own pool and tables, > 4x L2 in total) and
rotates through them, so no step finds its pages in the 126 MB L2.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ragged paged-attn decode tok/s & achieved HBM TB/s (% peak), 1/2/4/8 B200"
BATCH = 64
CTX_LO, CTX_HI = 128, 4096
HEADS, KV_HEADS, HEAD_DIM = 16, 2, 128
SCALE = HEAD_DIM ** -0.5
WORKLOAD = ("decode batch 64/GPU, ctx U[128,4096], 16q/2kv heads, d128, page 16, "
            "pool = pages x 1.1 + 8, scattered block tables, bf16 N(0,1)")
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4000)
    p.add_argument("--warmup", type=int, default=200)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--replicas", type=int, default=4, help="batches rotated to defeat L2")
    p.add_argument("--graph-steps", type=int, default=100, help="steps per captured graph")
    p.add_argument("--e2e-steps", type=int, default=200)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--seed", type=int, default=2024)
    return p.parse_args()


def global_lengths(world, seed):
    from shardserve_b200.workloads import uniform_lengths

    return uniform_lengths(BATCH * world, CTX_LO, CTX_HI, seed)


def rank_lengths(world, rank, seed):
    from shardserve_b200.sharding import shard_requests

    lengths = global_lengths(world, seed)
    shard = shard_requests(lengths, world)[rank]
    return [lengths[i] for i in shard]


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons every 20 ms (read-only queries)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.monotonic(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = []
        for ts, line in self.samples:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((ts, float(parts[1]), float(parts[2]), parts))
            except ValueError:
                continue
        inside = [r for r in rows if t0 <= r[0] <= t1]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i in range(4) if r[3][5 + i] == "Active"})
        return {"sm_mhz": statistics.median(r[1] for r in use), "sm_max_mhz": max(r[2] for r in use),
                "reasons": reasons, "samples": len(inside), "samples_outside_region": len(rows) - len(inside)}


# ---------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    """Reference arm: the CPU restatement of the reference attention path (the reference is
    pure Python/PyTorch and cannot run here), timed on this host's cores, rank 0 only."""
    if rank != 0:
        return
    import numpy as np
    import torch

    import oracle

    threads = oracle.host_threads()
    torch.set_num_threads(threads)
    lengths = rank_lengths(world, 0, args.seed)
    b = _cpu_batch(lengths, args.seed)
    # A step is one decode token per host thread, fewer when K + W steps of that size would
    # not finish in about two minutes (the arm must end within a few minutes for any K).
    t0 = time.perf_counter()
    oracle.ragged_attention(b["q"][:1], b["kp"], b["vp"], b["bt"][:1], np.zeros(1, np.int32),
                            b["pos"][:1], SCALE)
    t_tok = time.perf_counter() - t0
    budget = 120.0 / max(1, args.steps + args.warmup)
    per_step = int(max(1, min(threads, len(lengths), budget / max(t_tok, 1e-6))))

    def step(i):
        sel = [(i * per_step + j) % len(lengths) for j in range(per_step)]
        oracle.kv_append(b["kp"], b["vp"], b["kn"][sel], b["vn"][sel], b["slots"][sel])
        oracle.ragged_attention(b["q"][sel], b["kp"], b["vp"], b["bt"], b["seq"][sel],
                                b["pos"][sel], SCALE, threads=per_step)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = time.perf_counter() - t0
    value = args.steps * per_step / dt
    sample = (f"{per_step} decode tokens per step (one per host thread), rotating over the "
              f"{len(lengths)}-token batch; numpy port of Cache.write + the attention path")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "step": sample},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": per_step, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _cpu_batch(lengths, seed):
    import numpy as np

    rng = np.random.default_rng(seed)
    pages = [math.ceil(L / 16) for L in lengths]
    data_pages = int(math.ceil(sum(pages) * 1.1))
    N = data_pages + 8
    perm = rng.permutation(data_pages).astype(np.int32)
    W = max(pages)
    bt = np.zeros((len(lengths), W), np.int32)
    off = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[off:off + n]
        off += n
    pos = np.asarray([L - 1 for L in lengths], np.int64)
    seq = np.arange(len(lengths), dtype=np.int32)
    slots = bt[seq, pos // 16].astype(np.int64) * 16 + pos % 16
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)
    import oracle

    r = oracle.bf16_round
    return dict(kp=r(f(N, 16, KV_HEADS, HEAD_DIM)), vp=r(f(N, 16, KV_HEADS, HEAD_DIM)),
                q=r(f(len(lengths), HEADS, HEAD_DIM)), kn=r(f(len(lengths), KV_HEADS, HEAD_DIM)),
                vn=r(f(len(lengths), KV_HEADS, HEAD_DIM)), bt=bt, seq=seq, pos=pos, slots=slots)


def cpu_baseline(args, lengths):
    """The oracle (numpy port of the reference path) on a bounded sample, all host threads."""
    import oracle

    threads = oracle.host_threads()
    b = _cpu_batch(lengths, args.seed)
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < args.cpu_seconds:
        oracle.kv_append(b["kp"], b["vp"], b["kn"], b["vn"], b["slots"])
        oracle.ragged_attention(b["q"], b["kp"], b["vp"], b["bt"], b["seq"], b["pos"], SCALE,
                                threads=threads)
        done += len(lengths)
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{done // len(lengths)} full passes over this rank's {len(lengths)}-token "
                      f"batch in {dt:.1f} s (numpy, {threads} threads)"}


# ---------------------------------------------------------------------------------------
def run_ours(args, rank, world, dist):
    import torch

    import shardserve_b200 as sb
    from shardserve_b200 import kernel as K
    from shardserve_b200.workloads import append_bytes, attention_bytes, decode_batch

    dev = torch.device("cuda", torch.cuda.current_device())
    lengths = rank_lengths(world, rank, args.seed)
    T = len(lengths)
    R = max(1, args.replicas)
    batches = [decode_batch(lengths, HEADS, KV_HEADS, HEAD_DIM, seed=args.seed + 1000 * rank + r,
                            device=dev) for r in range(R)]

    def step(b):
        sb.kv_append(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots)
        return sb.ragged_attention_direct(b.q, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                          b.positions, SCALE)

    # Warm the workspace and check the fast path is the one that runs.
    for b in batches:
        step(b)
    torch.cuda.synchronize()
    assert K.last_attention_path() == 1, "attention did not take the TMA tensor-core path"
    assert K.device_errors(dev) == 0

    S = max(R, (args.graph_steps // R) * R)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    outs = []
    with torch.cuda.stream(stream):
        g_full = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_full, stream=stream):
            for i in range(S):
                outs.append(step(batches[i % R]))
        g_attn = torch.cuda.CUDAGraph()
        # external=True: the records become event-record nodes of the graph, so each replay
        # timestamps every attention launch on the stream it runs on.
        ev = [(torch.cuda.Event(enable_timing=True, external=True),
               torch.cuda.Event(enable_timing=True, external=True)) for _ in range(S)]
        with torch.cuda.graph(g_attn, stream=stream):
            for i in range(S):
                b = batches[i % R]
                ev[i][0].record(stream)
                sb.ragged_attention_direct(b.q, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                           b.positions, SCALE)
                ev[i][1].record(stream)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    reps_w = max(1, math.ceil(args.warmup / S))
    reps = max(1, math.ceil(args.steps / S))
    steps = reps * S
    clocks = ClockSampler(dev.index)
    clocks.start()
    time.sleep(0.3)
    with torch.cuda.stream(stream):
        for _ in range(reps_w):
            g_full.replay()
    barrier()
    # ---- timed region: exactly `steps` steps (append + attention) ----------------------
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.monotonic()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g_full.replay()
        e1.record(stream)
    barrier()
    t_wall1 = time.monotonic()
    ms_rank = e0.elapsed_time(e1)
    # ---- attention kernel alone, one CUDA-event pair per launch --------------------------
    with torch.cuda.stream(stream):
        g_attn.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        g_attn.replay()
    torch.cuda.synchronize()
    kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    clocks.stop()
    ms = max_over_ranks(ms_rank)
    kernel_ms = max_over_ranks(kernel_ms)
    tok_all = torch.tensor([float(T)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(tok_all)
    tokens_per_step = float(tok_all.item())
    value = tokens_per_step * steps / (ms / 1e3)

    # ---- end to end through the public API with host buffers ---------------------------
    e2e = run_e2e(args, batches[0], dev, dist, barrier, max_over_ranks, tok_all.item())

    abytes = attention_bytes(lengths, HEADS, KV_HEADS, HEAD_DIM)
    peak, peak_kind = peaks()
    achieved = abytes / (kernel_ms / 1e3) / 1e9
    traffic = traffic_from_profile(abytes)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": reps_w * S, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens_per_gpu_step": T,
                   "parallelism": f"request-sharded x{world} (LPT by context), no collective",
                   "l2": f"{R} rotating batches of ~{abytes / 1e6:.0f} MB each per GPU (> L2)",
                   "graph": f"{S} steps per CUDA graph, {reps} replays"},
        "hbm_tbs": achieved / 1e3,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "decode_attention_kernel<128,2>",
                     "kernel_us": kernel_ms * 1e3, "algorithmic_bytes": abytes,
                     "peak_kind": f"{peak_kind} copy bandwidth"},
        "append_bytes": append_bytes(T, KV_HEADS, HEAD_DIM),
        "e2e": e2e,
        "gpu_launches": 2 * steps,
        "clocks": clocks.summary(t_wall0, t_wall1),
    }
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_baseline(args, lengths)
    elif rank == 0:
        line["cpu_baseline"] = None
    del g_full, g_attn
    return line


def run_e2e(args, b, dev, dist, barrier, max_over_ranks, tokens_all):
    """Per step: pinned host -> device copies of q, new K/V rows, positions, sequence ids,
    block tables and slots; Cache.write + ragged_attention_direct through the public API;
    device -> pinned host copy of the output; stream synchronise (the reference runtime reads
    its results back every iteration, runtime.py:156)."""
    import torch

    import shardserve_b200 as sb

    host = {k: getattr(b, k).cpu().pin_memory() for k in
            ("q", "k_new", "v_new", "positions", "seq_ids", "block_tables", "slots")}
    dev_buf = {k: torch.empty_like(getattr(b, k)) for k in host}
    out_host = torch.empty(b.q.shape, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()
    stream = torch.cuda.current_stream(dev)

    def one():
        for k, t in host.items():
            dev_buf[k].copy_(t, non_blocking=True)
        sb.kv_append(b.k_pool, b.v_pool, dev_buf["k_new"], dev_buf["v_new"], dev_buf["slots"])
        out = sb.ragged_attention_direct(dev_buf["q"], b.k_pool, b.v_pool, dev_buf["block_tables"],
                                         dev_buf["seq_ids"], dev_buf["positions"], SCALE)
        out_host.copy_(out, non_blocking=True)
        stream.synchronize()

    for _ in range(20):
        one()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        one()
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    return {"value": tokens_all * args.e2e_steps / (ms / 1e3), "unit": "tok/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms / args.e2e_steps,
            "api": "shardserve_b200.kv_append + ragged_attention_direct, eager, per-step sync"}


def traffic_from_profile(abytes):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "decode_attention_batch64.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist_mod

        torch.cuda.set_device(local)
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        dist = dist_mod
    else:
        torch.cuda.set_device(0)
    try:
        line = run_ours(args, rank, world, dist)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
