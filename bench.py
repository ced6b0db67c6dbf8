"""Benchmark of the FOLD draft-step hot path: side-cache append + rotated far read + merge.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl fold|reference]

One step is one drafter layer's draft step: append the tokens accepted by the previous step
(1..B, drawn from the seed) to the side cache, read the far memory with the query rotated to the
shared far position (split-KV, fused rotation), and merge with the window read by LSE. With N
ranks (torchrun) the side cache is partitioned by contiguous position chunks; each rank reads its
chunk, combines its splits, the per-rank partials are all-gathered over NCCL and merged.

Workloads (synthetic, seeded; random-init drafter shapes):
  2 (default): Llama-3.1-8B drafter, 32 q / 8 kv heads, hd 128, B 10, context 131072, W 2048,
     alpha 2, K/V N(0,1) with 4 outlier channels per head x8, theta 5e5.
  3: Qwen3-8B drafter, 32/8, hd 128, B 8, context 32768, W 2048, theta 1e6.
  4: 16/4 heads, hd 256, B 16, context 262144, W 4096.
  5: 16/8 heads, hd 256, B 8, context 262144, W 4096.
The window read's (o, lse) are synthetic inputs resident in HBM (that read is not part of this
path). The side cache (0.5-2 GB) is far larger than L2 (126 MB), so no flush is needed between
steps.

Prints one JSON line (rank 0). value = microseconds per draft step (max over ranks, CUDA events).
--impl reference times the CPU oracle port of the same step on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    2: dict(name="llama3.1-8b-drafter-128k", hq=32, hkv=8, hd=128, B=10, ctx=131072, W=2048, theta=5e5, outliers=4),
    3: dict(name="qwen3-8b-drafter-32k", hq=32, hkv=8, hd=128, B=8, ctx=32768, W=2048, theta=1e6, outliers=0),
    4: dict(name="hd256-16q4kv-262k", hq=16, hkv=4, hd=256, B=16, ctx=262144, W=4096, theta=1e6, outliers=0),
    5: dict(name="hd256-16q8kv-262k", hq=16, hkv=8, hd=256, B=8, ctx=262144, W=4096, theta=1e6, outliers=0),
}
ALPHA = 2.0
METRIC = "us/draft-step (FOLD far-read + merge)"


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="fold", choices=["fold", "reference", "fa4"],
                    help="fold: this library; reference: the CPU implementation of the path; fa4: the "
                         "reference's own GPU path (its Triton rotation and merge with FlashAttention-4) alone")
    ap.add_argument("--no-fa4", action="store_true", help="skip timing the reference's GPU path beside the step")
    ap.add_argument("--no-fp8", action="store_true", help="skip the leg with the fp8 side cache")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--splits", type=int, default=0, help="far-read splits per KV head (0: one CTA per SM)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch the timed steps from Python, not as a CUDA graph")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1: how the per-rank partials meet (peer-to-peer kernel, or NCCL all-gather + merge)")
    ap.add_argument("--fused", action="store_true",
                    help="run the far read and the merge (or the peer exchange) as one cooperative kernel instead "
                         "of two launches")
    return ap.parse_args()


# ------------------------------------------------------------------------------ clocks sampler
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""
    # started 0.3 s before the work so that the first samples already see the load

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), active=parts[4], hw=parts[5],
                                 hw_thermal=parts[6], sw_thermal=parts[7], power_cap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return None
        loaded = [r for r in rows if r["sm"] > 0.5 * r["max"]] or rows
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"), ("power_cap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------------------ workload
def plan_steps(cfg, total_steps, seed):
    """Accepted tokens per step (1..B uniform from the seed) and the committed context H of each
    step; the first step sees a context of exactly cfg['ctx'] positions (H0 = ctx - B)."""
    import numpy as np

    rng = np.random.default_rng(seed + 1)
    acc = rng.integers(1, cfg["B"] + 1, size=total_steps)
    H = np.empty(total_steps, dtype=np.int64)
    H[0] = cfg["ctx"] - cfg["B"]
    for i in range(1, total_steps):
        H[i] = H[i - 1] + acc[i - 1]
    return acc, H


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(cfg_id):
    """DRAM bytes per far-read launch from the committed ncu summary of this workload, if any."""
    f = ROOT / "profiles" / f"far_read_config{cfg_id}.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


# ------------------------------------------------------------------------------ CPU legs
def cpu_step_oracle(cfg, H, q, k, v, o_l, lse_l, inv_freq):
    """The oracle's far query + far read + merge of one step (float64 numpy)."""
    from oracle import fold_oracle as fo

    W, B = cfg["W"], cfg["B"]
    qf = fo.bf16_round(fo.far_query(q, H, inv_freq, W + B))
    lim = fo.far_row_limits(H, W, B, B)
    L = int(lim.max())
    o_f, lse_f = fo.far_read(qf, k[:L], v[:L], lim, cfg["hd"] ** -0.5 * ALPHA)
    return fo.merge(o_l, lse_l, o_f, lse_f, H, W, B, ALPHA)


def cpu_inputs(cfg, seed, max_keys):
    import numpy as np

    rng = np.random.default_rng(seed + 7)
    L = max_keys
    # a 4096-row block of N(0,1) keys/values tiled to the context: the oracle's cost does not
    # depend on the values, and generating 10^8 normals would dominate the sample
    reps = -(-L // 4096)
    k = np.tile(rng.standard_normal((4096, cfg["hkv"], cfg["hd"])), (reps, 1, 1))[:L]
    v = np.tile(rng.standard_normal((4096, cfg["hkv"], cfg["hd"])), (reps, 1, 1))[:L]
    q = rng.standard_normal((cfg["B"], cfg["hq"], cfg["hd"])).astype(np.float64)
    o_l = rng.standard_normal((cfg["B"], cfg["hq"], cfg["hd"]))
    lse_l = rng.standard_normal((cfg["hq"], cfg["B"])) + 5.0
    return q, k, v, o_l, lse_l


def cpu_baseline(cfg, seed, budget_s=15.0, max_steps=50):
    """Times the oracle port on the host cores: whole steps of the workload until ~budget_s."""
    from oracle import fold_oracle as fo

    acc, H = plan_steps(cfg, max_steps, seed)
    q, k, v, o_l, lse_l = cpu_inputs(cfg, seed, int(H.max()))
    f = fo.inv_freq(cfg["theta"], cfg["hd"])
    cpu_step_oracle(cfg, int(H[0]), q, k, v, o_l, lse_l, f)  # warm-up
    times = []
    t_all = time.perf_counter()
    for i in range(max_steps):
        t0 = time.perf_counter()
        cpu_step_oracle(cfg, int(H[i]), q, k, v, o_l, lse_l, f)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    us = 1e6 * statistics.mean(times)
    out = dict(value=us, unit="us/draft-step", cores=os.cpu_count() or 1, kind="port",
               sample=f"{len(times)} whole draft steps of the {cfg['name']} workload (float64 numpy oracle: "
                      f"far query + far read + merge, BLAS threads = {os.cpu_count()})")
    try:  # the same step on one thread (one step: it takes seconds)
        from threadpoolctl import threadpool_limits

        with threadpool_limits(limits=1):
            t0 = time.perf_counter()
            cpu_step_oracle(cfg, int(H[0]), q, k, v, o_l, lse_l, f)
            out["value_1_thread"] = 1e6 * (time.perf_counter() - t0)
    except ImportError:
        pass
    return out


# ------------------------------------------------------------------------------ GPU arm
def run_gpu(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from fold_b200 import kernels
    from fold_b200.rope import default_inv_freq, rope_table
    from fold_b200.shard import PeerExchange, ShardPlan, unpack_partials

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=30), device_id=dev)
    cfg = CONFIGS[args.config]
    hq, hkv, hd, B, W = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["B"], cfg["W"]
    total = args.warmup + args.steps
    acc, H = plan_steps(cfg, total, args.seed)
    length = int(H[-1] + acc[-1]) + B  # every position any step appends or reads
    plan = ShardPlan.for_far(length, W, B, world, rank)
    pos_lo, held = plan.pos_lo, plan.held
    pages = -(-max(held, 1) // 256) + 1

    # ---- side cache: the committed context before the first step, N(0,1) (+ outlier channels)
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed * 1000 + rank)
    side = torch.empty((pages, hkv, 256, 2 * hd), device=dev, dtype=torch.bfloat16)
    side.normal_(generator=gen)
    if cfg["outliers"]:
        ch = torch.randperm(hd, generator=torch.Generator().manual_seed(args.seed))[: cfg["outliers"]]
        cols = torch.cat((ch, ch + hd)).to(dev)
        side[..., cols] *= 8.0
    # accepted tokens of every step (K and V before RoPE), appended at their positions
    max_acc = int(acc.max())
    new_k = torch.randn((total, max_acc, hkv, hd), device=dev, dtype=torch.bfloat16, generator=gen)
    new_v = torch.randn((total, max_acc, hkv, hd), device=dev, dtype=torch.bfloat16, generator=gen)
    new_pos = torch.zeros((total, max_acc), device=dev, dtype=torch.int64)
    for i in range(total):
        new_pos[i, : acc[i]] = torch.arange(int(H[i]), int(H[i]) + int(acc[i]))
    q_all = torch.randn((total, B, hq, hd), device=dev, dtype=torch.bfloat16, generator=gen)
    seq_all = torch.from_numpy((H + B).astype(np.int32)).to(dev)
    qsl = torch.tensor([0, B], dtype=torch.int32, device=dev)
    o_l = torch.randn((B, hq, hd), device=dev, dtype=torch.bfloat16, generator=gen)
    lse_l = (torch.randn((hq, B), device=dev, generator=gen) + 5.0).float()
    out = torch.empty((B, hq, hd), device=dev, dtype=torch.bfloat16)
    inv = default_inv_freq(cfg["theta"], hd, dev)
    table = rope_table(inv, length + W + B + 1, dev)
    splits = args.splits or kernels.default_splits(hkv)
    o_part = torch.empty((splits, B, hq, hd), device=dev, dtype=torch.float32)
    lse_part = torch.empty((splits, hq, B), device=dev, dtype=torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    per = B * hq * hd + hq * B
    send = torch.empty(per, device=dev, dtype=torch.float32)
    recv = torch.empty(world * per, device=dev, dtype=torch.float32)
    o_mine, lse_mine = send[: B * hq * hd].view(B, hq, hd), send[B * hq * hd:].view(hq, B)
    scale = hd ** -0.5 * ALPHA
    stream = torch.cuda.current_stream(dev)
    # --fused: the far read ends with the exchange (of one rank at N = 1) and the merge in one cooperative
    # launch; otherwise the far read and the merge (or the peer exchange kernel) are two launches
    fused = args.exchange == "p2p" and args.fused
    # at N > 1 both data planes are built: the step runs the chosen one, the other is timed beside it
    peer = PeerExchange(n=B, hq=hq, hd=hd, device=dev) if world > 1 or fused else None
    comm = 0
    if world > 1:
        dist.barrier(device_ids=[local])  # the NCCL communicator exists from here on
        comm = int(dist.group.WORLD._get_backend(dev)._comm_ptr())

    def far(i):
        kernels.far_read(q_all[i], qsl, seq_all[i: i + 1], side, o_part, lse_part, window=W, block=B,
                         far_distance=W + B, softmax_scale=scale, table=table, pos_lo=pos_lo, capacity=length, err=err)

    def append(i):
        a = int(acc[i - 1]) if i > 0 else 0
        if a:  # tokens accepted by the previous step become committed context
            kernels.append(new_k[i - 1, :a], new_v[i - 1, :a], new_pos[i - 1, :a], new_pos[i - 1, :a], side,
                           pos_lo=pos_lo, skip_foreign=world > 1, err=err)

    def step(i, exchange=args.exchange):
        append(i)
        seq = seq_all[i: i + 1]
        if fused:
            kernels.far_read_exchange(peer.handle, q_all[i], qsl, seq, side, o_part, lse_part, o_l, lse_l, out,
                                      window=W, block=B, far_distance=W + B, softmax_scale=hd ** -0.5, alpha=ALPHA,
                                      table=table, pos_lo=pos_lo, capacity=length, err=err)
            return
        far(i)
        if world == 1:
            kernels.merge(o_l, lse_l, o_part, lse_part, out, qsl, seq, window=W, block=B, alpha=ALPHA)
        elif exchange == "p2p":
            peer.merge(o_part, lse_part, o_l, lse_l, out, qsl, seq, window=W, block=B, alpha=ALPHA, err=err)
        else:  # combine + ncclAllGather (fold_allgather_partials), then the merge of the world's partials
            o_all, lse_all = kernels.allgather_partials(comm, o_part, lse_part, send, recv)
            kernels.merge(o_l, lse_l, o_all, lse_all, out, qsl, seq, window=W, block=B, alpha=ALPHA)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    align_buf = torch.zeros(1, device=dev)

    def align():
        """N > 1: a one-float all-reduce enqueued on the timing stream right before the start event,
        so that every rank's timed region starts when the collective completes on the devices, not
        when each host process gets past its barrier (host skew would count in the max over ranks)."""
        if world > 1:
            dist.all_reduce(align_buf)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # The K timed steps run as one CUDA graph (the drafter step runs inside vLLM's CUDA graphs);
    # --eager launches them one by one from Python instead.
    graph = None
    if not args.eager:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for j in range(args.steps):
                step(args.warmup + j)
        torch.cuda.synchronize()

    def timed_steps():
        if graph is not None:
            graph.replay()
        else:
            for j in range(args.steps):
                step(args.warmup + j)

    # A short untimed run of the same steps precedes the timed region so that nvidia-smi (100 ms
    # samples) sees the load. Its length is decided on rank 0 and shared, so that every rank issues
    # the same collectives.
    pre = 0
    if graph is not None:
        t0 = time.perf_counter()
        graph.replay()
        torch.cuda.synchronize()
        pre = max(1, min(50, int(0.2 / max(time.perf_counter() - t0, 1e-4))))
    if world > 1:
        n_pre = torch.tensor([pre], device=dev, dtype=torch.int64)
        dist.broadcast(n_pre, src=0)
        pre = int(n_pre.item())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        for _ in range(pre):
            graph.replay()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        align()
        e0.record(stream)
        timed_steps()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # The far-read kernel alone (roofline): the same K launches back to back, timed with events
    # around one replay of a graph that holds only them.
    far_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(far_graph):
        for j in range(args.steps):
            far(args.warmup + j)
    far_graph.replay()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    far_graph.replay()
    f1.record(stream)
    torch.cuda.synchronize()
    far_ms = f0.elapsed_time(f1) / args.steps
    # The same graph again after ~0.3 s of back-to-back replays: under sustained load the board
    # reaches its power cap and lowers the SM clock.
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.3:
        far_graph.replay()
        torch.cuda.synchronize()
    f0.record(stream)
    far_graph.replay()
    f1.record(stream)
    torch.cuda.synchronize()
    far_sustained_ms = f0.elapsed_time(f1) / args.steps
    del far_graph
    fused_ms = None
    if fused:  # the far read that ends with the merge (exchange) alone, timed as the far read above
        fg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(fg):
            for j in range(args.steps):
                i = args.warmup + j
                kernels.far_read_exchange(peer.handle, q_all[i], qsl, seq_all[i: i + 1], side, o_part, lse_part, o_l,
                                          lse_l, out, window=W, block=B, far_distance=W + B, softmax_scale=hd ** -0.5,
                                          alpha=ALPHA, table=table, pos_lo=pos_lo, capacity=length, err=err)
        fg.replay()
        torch.cuda.synchronize()
        f0.record(stream)
        fg.replay()
        f1.record(stream)
        torch.cuda.synchronize()
        fused_ms = f0.elapsed_time(f1) / args.steps
        del fg
    # N > 1: the same steps with the other data plane (peer exchange or NCCL all-gather), timed
    # the same way (graph of K steps after the same untimed passes, barrier, max over ranks)
    alt, alt_ms = None, 0.0
    if world > 1 and not fused:
        alt = "nccl" if args.exchange == "p2p" else "p2p"
        for j in range(args.warmup):
            step(j, alt)
        torch.cuda.synchronize()
        alt_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(alt_graph):
            for j in range(args.steps):
                step(args.warmup + j, alt)
        alt_graph.replay()
        for _ in range(pre):
            alt_graph.replay()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        align()
        f0.record(stream)
        alt_graph.replay()
        f1.record(stream)
        torch.cuda.synchronize()
        alt_ms = f0.elapsed_time(f1)
        del alt_graph
    window = run_window(args, cfg, dev, stream, H, q_all, seq_all, qsl, side, table, pos_lo, out, length, err,
                        append) if world == 1 else None
    fp8 = None
    if world == 1 and args.impl == "fold" and not args.no_fp8:
        fp8 = run_fp8(args, cfg, dev, stream, side, H, acc, q_all, seq_all, qsl, new_k, new_v, new_pos, o_l, lse_l,
                      out, table, length, splits, err)
    fa4 = None
    if world == 1 and (args.impl == "fa4" or not args.no_fa4):
        fa4 = run_fa4(args, cfg, dev, stream, side, q_all, seq_all, qsl, new_k, new_v, new_pos, acc, o_l, lse_l,
                      length, inv)
    # every rank takes part in the reduction before any rank may raise (same collectives everywhere)
    t = torch.tensor([ms, far_ms, far_sustained_ms, float(err.item()), alt_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, far_ms, far_sustained_ms, alt_ms = float(t[0]), float(t[1]), float(t[2]), float(t[4])
    if int(t[3]):
        raise RuntimeError(f"device error word {int(t[3])} on some rank")
    us_step = 1000.0 * ms / args.steps

    # algorithmic bytes of one far-read launch on this rank: its K/V rows + q + partials
    far_keys = [min(max(int(H[args.warmup + j]) - W, 0), pos_lo + held) - pos_lo for j in range(args.steps)]
    kv_bytes = statistics.mean(max(f, 0) for f in far_keys) * hkv * 2 * hd * 2
    part_bytes = splits * (B * hq * hd + hq * B) * 4
    alg = kv_bytes + B * hq * hd * 2 + part_bytes
    hbm_peak, peak_kind = peaks()
    # the far read as it runs inside the step: K launches back to back after 0.3 s of load, when
    # the board sits at its power cap (the burst figure is kept beside it)
    achieved = alg / (far_sustained_ms * 1e-3) / 1e9
    achieved_burst = alg / (far_ms * 1e-3) / 1e9
    traffic = profile_traffic(args.config) if world == 1 else None

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, cfg, dev, side, table, H, acc, pos_lo, length, splits, world, rank, local,
                      peer if fused else None)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(us_step, 3),
            "unit": "us/draft-step",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 6),
            "higher_is_better": False,
            "scaling": "strong",  # one context, its far memory split over the ranks
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) K/V/Q, random-init drafter shapes)",
            "config": {"workload": cfg["name"], "context": cfg["ctx"], "window": W, "block": B, "heads_q": hq,
                       "heads_kv": hkv, "head_dim": hd, "alpha": ALPHA, "splits": splits,
                       "parallelism": f"seq-shard{world}" if world > 1 else "single",
                       "step_kernels": ("append + far read ending with the merge in one cooperative kernel" if fused
                                        and world == 1 else "append + far read ending with the peer exchange and the "
                                        "merge in one cooperative kernel" if fused else "append + far read + merge"
                                        if world == 1 else "append + far read + peer exchange kernel"
                                        if args.exchange == "p2p" else "append + far read + combine and "
                                        "ncclAllGather (fold_allgather_partials) + merge"),
                       "exchange": None if world == 1 else (
                           "peer-to-peer (NVLink stores of self-validating lines, combine and merge fused)"
                           if args.exchange == "p2p" else "NCCL all-gather"),
                       "timing": "eager launches" if args.eager else "CUDA graph of the K timed steps",
                       "l2": "inputs larger than L2 (side cache %.0f MB per GPU)" % (side.numel() * 2 / 1e6)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                         "kernel": "far_read_kernel", "kernel_us": round(far_sustained_ms * 1000, 3),
                         "kernel_timing": "sustained: the far read alone, one graph of K launches timed after 0.3 s "
                                          "of back-to-back replays (the power-capped clock of the step)",
                         "kernel_us_sustained": round(far_sustained_ms * 1000, 3),
                         "kernel_us_burst": round(far_ms * 1000, 3),
                         "achieved_burst": round(achieved_burst, 1),
                         "frac_burst": round(achieved_burst / hbm_peak, 4),
                         "fused_kernel_us": None if fused_ms is None else round(fused_ms * 1000, 3),
                         "algorithmic_bytes": int(alg), "traffic": traffic},
            "gpu_launches": args.steps * (2 if fused else 3 if world == 1 or args.exchange == "p2p" else 5),
            "clocks": clocks.summary(),
            "e2e": e2e,
        }
        if window is not None:
            line["window_read"] = window
        if fp8 is not None:
            line["fp8_side_cache"] = fp8
        if fa4 is not None:
            line["reference_gpu_path"] = fa4
        if args.impl == "fa4":  # the reference's GPU path as its own line
            ok = "us_per_step" in fa4
            line = {"impl": "fa4", "metric": METRIC, "value": fa4.get("us_per_step"), "unit": "us/draft-step",
                    "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(fa4["us_per_step"] / 1000, 6) if ok else None, "higher_is_better": False,
                    "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": line["data"],
                    "config": line["config"], "reference_gpu_path": fa4}
            if not ok:
                line = {"impl": "fa4", "unavailable": fa4.get("unavailable")}
        if alt is not None:
            line["exchange_alternative"] = {
                "exchange": alt, "us_per_step": round(1000.0 * alt_ms / args.steps, 3),
                "how": ("append + far read + combine and ncclAllGather of the per-rank partials "
                        "(fold_allgather_partials) + merge" if alt == "nccl" else
                        "append + far read + peer exchange kernel"),
                "timing": "the same K steps as one CUDA graph, same untimed passes, max over ranks"}
        if not args.no_cpu and world == 1:
            line["cpu_baseline"] = cpu_baseline(cfg, args.seed)
        print(json.dumps(line), flush=True)
    del graph
    if peer is not None:
        peer.close()
    if world > 1:
        dist.destroy_process_group()


def run_fa4(args, cfg, dev, stream, side, q_all, seq_all, qsl, new_k, new_v, new_pos, acc, o_l, lse_l, length, inv):
    """The reference's own GPU path for the same steps (fold/attention.py:162-172, 260-265): the
    side-cache scatter of _wrap_context_kv in torch, its Triton far_query, FlashAttention-4 over the
    side cache (paged, causal, seqused_k = far_len, num_splits = max(16, 64 // Hkv)) and its
    Triton merge, from the unmodified reference package installed under baseline/_ref and vLLM's
    flash_attn_varlen_func(fa_version=4). Timed like the step: one CUDA graph of K steps after
    0.3 s of load, CUDA events. Returns the result dict, or {"unavailable": why}."""
    import torch

    try:
        ref_path = ROOT / "baseline" / "_ref"
        if not (ref_path / "fold" / "kernels.py").exists():
            return {"unavailable": "the reference is not installed under baseline/_ref"}
        if str(ref_path) not in sys.path:
            sys.path.insert(0, str(ref_path))
        from fold.kernels import far_query, merge  # noqa: PLC0415
        from vllm.vllm_flash_attn import fa_version_unsupported_reason, flash_attn_varlen_func  # noqa: PLC0415
        why = fa_version_unsupported_reason(4)
        if why:
            return {"unavailable": f"FlashAttention-4: {why}"}
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        return {"unavailable": f"{type(e).__name__}: {e}"}
    hq, hkv, hd, B, W = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["B"], cfg["W"]
    pages = side.shape[0]
    side_table = torch.arange(pages, device=dev, dtype=torch.int32)[None]
    far_len = torch.zeros(1, device=dev, dtype=torch.int32)
    fk, fv = side.transpose(1, 2).split(hd, dim=-1)
    out = torch.empty((B, hq * hd), device=dev, dtype=torch.bfloat16)
    splits = max(16, 64 // hkv)
    scale = hd ** -0.5 * ALPHA

    def append(i):
        a = int(acc[i - 1]) if i > 0 else 0
        if a:
            pos = new_pos[i - 1, :a]
            pg, off = torch.div(pos, 256, rounding_mode="floor"), pos % 256
            side[pg, :, off, :hd] = new_k[i - 1, :a]
            side[pg, :, off, hd:] = new_v[i - 1, :a]

    def far(i, qf):
        return flash_attn_varlen_func(q=qf, k=fk, v=fv, cu_seqlens_q=qsl, max_seqlen_q=B, seqused_k=far_len,
                                      max_seqlen_k=length, softmax_scale=scale, causal=True, block_table=side_table,
                                      return_softmax_lse=True, fa_version=4, num_splits=splits)

    def step(i):
        append(i)
        seq = seq_all[i: i + 1]
        qf = far_query(q_all[i], qsl, seq, inv, far_len, far_distance=W + B, window=W, block=B)
        out_f, lse_f = far(i, qf)
        merge(o_l, lse_l, out_f, lse_f, out.view(B, hq, hd), qsl, seq, window=W, block=B, alpha=ALPHA)

    try:
        t_first = time.perf_counter()
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        first_s = time.perf_counter() - t_first
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def graph_of(fn):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for j in range(args.steps):
                    fn(args.warmup + j)
            g.replay()
            torch.cuda.synchronize()
            return g

        def timed(g, sustained):
            if sustained:
                t0 = time.perf_counter()
                while time.perf_counter() - t0 < 0.3:
                    g.replay()
                    torch.cuda.synchronize()
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            return 1000.0 * e0.elapsed_time(e1) / args.steps

        qf_fixed = far_query(q_all[args.warmup], qsl, seq_all[args.warmup: args.warmup + 1], inv, far_len,
                             far_distance=W + B, window=W, block=B)
        gf = graph_of(lambda i: far(i, qf_fixed))
        far_burst = timed(gf, False)
        far_sustained = timed(gf, True)
        del gf
        gs = graph_of(step)
        us = timed(gs, True)
        del gs
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        return {"unavailable": f"{type(e).__name__}: {e}"}
    return {"us_per_step": round(us, 3), "unit": "us/draft-step",
            "far_read_us_sustained": round(far_sustained, 3), "far_read_us_burst": round(far_burst, 3),
            "first_calls_s": round(first_s, 1), "splits": splits,
            "path": "reference GPU path: torch side-cache scatter + Triton far_query + FlashAttention-4 far read "
                    "(vllm.vllm_flash_attn, fa_version=4) + Triton merge, unmodified from baseline/_ref",
            "timing": "one CUDA graph of K steps after 0.3 s of back-to-back replays (sustained), CUDA events; "
                      "the far read alone likewise, burst and sustained"}


def run_fp8(args, cfg, dev, stream, side, H, acc, q_all, seq_all, qsl, new_k, new_v, new_pos, o_l, lse_l, out,
            table, length, splits, err):
    """The same steps with the fp8 side cache (FoldWorkspace side_format "fp8"): the bf16 side
    cache is quantised into it once (per-KV-head scales amax / 448), then each step appends the
    accepted tokens with fold_append_fp8, reads the far memory with fold_far_read_fp8 and merges.
    Timed like the headline step (one CUDA graph of K steps after 0.3 s of load); the far read
    alone likewise, burst and sustained."""
    import torch

    from fold_b200 import kernels

    hq, hkv, hd, B, W = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["B"], cfg["W"]
    if hd != kernels.FP8_HEAD_DIM:
        return None
    pages = side.shape[0]
    side8 = torch.zeros(kernels.fp8_side_shape(pages, hkv), device=dev, dtype=torch.uint8)
    ks = (side[..., :hd].abs().amax(dim=(0, 2, 3)).float() / 448.0).contiguous()
    vs = (side[..., hd:].abs().amax(dim=(0, 2, 3)).float() / 448.0).contiguous()
    for a in range(0, (pages - 1) * 256, 16384):
        pos = torch.arange(a, min(a + 16384, (pages - 1) * 256), device=dev)
        k, v = kernels.gather(side, pos)
        kernels.append_fp8(k, v, pos, pos, side8, ks, vs)
    o_part = torch.empty((splits, B, hq, hd), device=dev, dtype=torch.float32)
    lse_part = torch.empty((splits, hq, B), device=dev, dtype=torch.float32)
    scale = hd ** -0.5 * ALPHA

    def far(i):
        kernels.far_read_fp8(q_all[i], qsl, seq_all[i: i + 1], side8, ks, vs, o_part, lse_part, window=W, block=B,
                             far_distance=W + B, softmax_scale=scale, table=table, capacity=length, err=err)

    def step(i):
        a = int(acc[i - 1]) if i > 0 else 0
        if a:
            kernels.append_fp8(new_k[i - 1, :a], new_v[i - 1, :a], new_pos[i - 1, :a], new_pos[i - 1, :a], side8, ks,
                               vs, err=err)
        far(i)
        kernels.merge(o_l, lse_l, o_part, lse_part, out, qsl, seq_all[i: i + 1], window=W, block=B, alpha=ALPHA)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def graph_of(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for j in range(args.steps):
                fn(args.warmup + j)
        g.replay()
        torch.cuda.synchronize()
        return g

    def timed(g, sustained):
        if sustained:
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < 0.3:
                g.replay()
                torch.cuda.synchronize()
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return 1000.0 * e0.elapsed_time(e1) / args.steps

    gf = graph_of(far)
    burst, sustained = timed(gf, False), timed(gf, True)
    del gf
    gs = graph_of(step)
    us = timed(gs, True)
    del gs
    far_keys = statistics.mean(max(min(int(H[args.warmup + j]) - W, length), 0) for j in range(args.steps))
    alg = far_keys * hkv * 2 * hd + B * hq * hd * 2 + splits * (B * hq * hd + hq * B) * 4
    hbm_peak, peak_kind = peaks()
    return {"us_per_step": round(us, 3), "unit": "us/draft-step", "far_read_us_sustained": round(sustained, 3),
            "far_read_us_burst": round(burst, 3), "algorithmic_bytes": int(alg),
            "achieved_gbs": round(alg / (sustained * 1e-6) / 1e9, 1), "peak": hbm_peak, "peak_kind": peak_kind,
            "frac": round(alg / (sustained * 1e-6) / 1e9 / hbm_peak, 4),
            "side_cache_bytes": int(side8.numel()), "kernel": "far_read_kernel<FarCfg<128, nt, 128, 4, fp8>>",
            "how": "append_fp8 + far_read_fp8 + merge of the same steps, e4m3 K and V^T with per-KV-head scales "
                   "(amax / 448); one CUDA graph of K steps after 0.3 s of load (sustained); far read alone burst "
                   "and sustained"}


def run_window(args, cfg, dev, stream, H, q_all, seq_all, qsl, side, table, pos_lo, out, length, err, append):
    """The window (exact-position) read, which the headline step takes as an input, measured on
    its own (16 splits per KV head) and inside the whole draft step: append + one launch in which
    each KV head's blocks (one per SM in all) share the far and window reads, split per step from
    the device-side lengths + merge of both split sets (with a tcgen05 far read, the two reads as
    two launches, as FoldAttention does). The drafter's paged cache (block size 16, shuffled blocks) holds every position a step's
    window reaches; each split reads a contiguous part of the window [H - W - B + 1, H + B)."""
    import numpy as np
    import torch

    from fold_b200 import kernels

    hq, hkv, hd, B, W = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["B"], cfg["W"]
    bs, wsplits = 16, 16
    lo = max(int(H[args.warmup]) - W - B - 256, 0) // bs  # first logical block any timed step's tiles touch
    nbl = -(-length // bs)
    rng = np.random.default_rng(args.seed + 5)
    table_np = np.zeros((1, nbl), dtype=np.int32)
    table_np[0, lo:] = rng.permutation(nbl - lo)
    block_table = torch.from_numpy(table_np).to(dev)
    kv = torch.randn((nbl - lo, hkv, bs, 2 * hd), device=dev, dtype=torch.bfloat16)
    kc, vc = kernels.paged_planes(kv, hd)
    wo = torch.empty((wsplits, B, hq, hd), device=dev, dtype=torch.float32)
    wl = torch.empty((wsplits, hq, B), device=dev, dtype=torch.float32)
    scale = hd ** -0.5
    fsplits = max(kernels.default_splits(hkv), 2)  # blocks per KV head, shared by the two reads
    far_parts = (torch.empty((fsplits, B, hq, hd), device=dev), torch.empty((fsplits, hq, B), device=dev))
    win_parts = (torch.empty((fsplits, B, hq, hd), device=dev), torch.empty((fsplits, hq, B), device=dev))
    plan = torch.zeros(1, device=dev, dtype=torch.int32)
    one_launch = not kernels.far_read_uses_tcgen05(hd, B, hq, hkv)  # as FoldAttention chooses
    ws = (W + B - 1, B - 1)

    def window(i):
        kernels.window_read(q_all[i], qsl, seq_all[i: i + 1], kc, vc, block_table, wo, wl, window_size=ws,
                            causal=False, softmax_scale=scale, err=err)

    def full_step(i):
        append(i)
        seq = seq_all[i: i + 1]
        if one_launch:
            kernels.step_read(q_all[i], q_all[i], qsl, seq, side, far_parts, kc, vc, block_table, win_parts, plan,
                              window=W, block=B, far_distance=W + B, softmax_scale=scale, alpha=ALPHA, window_size=ws,
                              causal=False, table=table, pos_lo=pos_lo, capacity=length, err=err)
            kernels.merge_partials(win_parts[0], win_parts[1], far_parts[0], far_parts[1], out, qsl, seq, window=W,
                                   block=B, alpha=ALPHA, plan=plan)
        else:  # tcgen05 far read, then the window read with its own splits
            kernels.far_read(q_all[i], qsl, seq, side, far_parts[0], far_parts[1], window=W, block=B,
                             far_distance=W + B, softmax_scale=scale * ALPHA, table=table, pos_lo=pos_lo,
                             capacity=length, err=err)
            window(i)
            kernels.merge_partials(wo, wl, far_parts[0], far_parts[1], out, qsl, seq, window=W, block=B, alpha=ALPHA)

    def graph_of(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for j in range(args.steps):
                fn(args.warmup + j)
        g.replay()
        torch.cuda.synchronize()
        return g

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def time_graph(g):
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return 1000.0 * e0.elapsed_time(e1) / args.steps

    wg = graph_of(window)
    w_us = time_graph(wg)
    del wg
    fg = graph_of(full_step)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.3:  # sustained, like the headline step
        fg.replay()
        torch.cuda.synchronize()
    f_us = time_graph(fg)
    del fg
    keys = statistics.mean(min(W + 2 * B - 1, int(H[args.warmup + j]) + B) for j in range(args.steps))
    alg = keys * hkv * 2 * hd * 2 + B * hq * hd * 2 + wsplits * (B * hq * hd + hq * B) * 4
    return {"kernel": "window_read_kernel", "us": round(w_us, 3), "splits": wsplits, "block_size": bs,
            "algorithmic_bytes": int(alg), "achieved_gbs": round(alg / (w_us * 1e-6) / 1e9, 1),
            "timing": "burst: K window reads back to back in one graph",
            "full_step_us": round(f_us, 3),
            "full_step": ("append + one launch in which the far and window reads share the KV heads' blocks "
                          f"({fsplits} per head, split per step)" if one_launch else "append + tcgen05 far read + "
                          f"window read ({wsplits} splits per KV head)") + " + merge of both split sets (no synthetic "
                         "window input), one graph of K steps, sustained"}


def run_e2e(args, cfg, dev, side, table, H, acc, pos_lo, length, splits, world, rank, local, peer):
    """The same steps through the public workspace API with pinned host inputs. Per step, the
    query, the K/V, positions and slots of the tokens the previous step accepted, and seq_len are
    copied host->device inside the timed region, and the merged output is read back device->host.

    The layer's calls (FoldWorkspace.append, read_far or ShardedFarMemory.step, the merge) are
    captured once in a CUDA graph per input buffer, as vLLM captures the drafter's forward, and
    replayed per step. A step's record has room for B accepted tokens. Rows past the accepted
    count carry slot -1, which the append sends to the dummy slot (fold/attention.py:262), so one
    graph serves every acceptance count."""
    import torch
    import torch.distributed as dist

    from fold_b200 import kernels
    from fold_b200.attention import FoldWorkspace
    from fold_b200.shard import ShardedFarMemory, ShardPlan

    hq, hkv, hd, B, W = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["B"], cfg["W"]
    total = args.warmup + args.steps
    fused = args.exchange == "p2p" and args.fused  # the data plane of the device-timed step
    dummy = torch.zeros((1, hkv, 16, 2 * hd), device=dev, dtype=torch.bfloat16)
    plan = ShardPlan.for_far(length, W, B, world, rank)
    ws = FoldWorkspace(dummy, W, B, length, inv_freq=torch.ones(hd // 2, device=dev), far_distance=W + B,
                       alpha=ALPHA, num_heads=hq, splits=splits, pos_lo=plan.pos_lo,
                       shard_len=plan.held if world > 1 else None)
    ws.side = side  # the same resident side cache as the kernel leg
    ws._table = table
    ws.partials(B, hq)  # allocated before capture
    sharded = ShardedFarMemory(plan, ws, exchange=args.exchange, peer=peer) if world > 1 else None
    gen = torch.Generator().manual_seed(args.seed + 99)
    max_acc = B
    # One pinned record per step, uploaded with one copy: the step's query, the K/V, positions and
    # slots of the tokens the previous step accepted, and the step's seq_len (fields 16-byte aligned).
    qb, kb = B * hq * hd * 2, max_acc * hkv * hd * 2
    off_k, off_v, off_pos = qb, qb + kb, qb + 2 * kb
    off_slot = off_pos + max_acc * 8
    off_seq = off_slot + max_acc * 8
    rec = (off_seq + 4 + 15) // 16 * 16
    h_in = torch.zeros((total, rec), dtype=torch.uint8)
    for i in range(total):
        h_in[i, :qb].view(torch.bfloat16).copy_(torch.randn(B * hq * hd, generator=gen))
        a = int(acc[i - 1]) if i > 0 else 0
        if a:
            h_in[i, off_k:off_k + a * hkv * hd * 2].view(torch.bfloat16).copy_(torch.randn(a * hkv * hd, generator=gen))
            h_in[i, off_v:off_v + a * hkv * hd * 2].view(torch.bfloat16).copy_(torch.randn(a * hkv * hd, generator=gen))
        pos = torch.full((max_acc,), -1, dtype=torch.int64)
        if a:
            pos[:a] = torch.arange(int(H[i - 1]), int(H[i - 1]) + a)
        h_in[i, off_pos:off_pos + max_acc * 8].view(torch.int64).copy_(pos.clamp_min(0))
        h_in[i, off_slot:off_slot + max_acc * 8].view(torch.int64).copy_(pos)
        h_in[i, off_seq:off_seq + 4].view(torch.int32).fill_(int(H[i]) + B)
    h_in = h_in.pin_memory()
    h_out = torch.empty((2, B, hq, hd), dtype=torch.bfloat16).pin_memory()
    qsl = torch.tensor([0, B], dtype=torch.int32, device=dev)
    o_l = torch.randn((B, hq, hd), device=dev, dtype=torch.bfloat16)
    lse_l = torch.randn((hq, B), device=dev) + 5.0
    scale = hd ** -0.5

    class Slot:
        """One device input record and output, with the captured step that reads and writes them."""

        def __init__(self):
            self.d_in = torch.zeros(rec, device=dev, dtype=torch.uint8)
            d = self.d_in
            self.q = d[:qb].view(torch.bfloat16).view(B, hq, hd)
            self.k = d[off_k:off_k + kb].view(torch.bfloat16).view(max_acc, hkv, hd)
            self.v = d[off_v:off_v + kb].view(torch.bfloat16).view(max_acc, hkv, hd)
            self.pos = d[off_pos:off_pos + max_acc * 8].view(torch.int64)
            self.slots = d[off_slot:off_slot + max_acc * 8].view(torch.int64)
            self.seq = d[off_seq:off_seq + 4].view(torch.int32)
            self.out = torch.empty((B, hq, hd), device=dev, dtype=torch.bfloat16)
            self.uploaded, self.computed, self.read = (torch.cuda.Event() for _ in range(3))
            self.graph = None

        def layer_step(self):
            ws.append(self.k, self.v, self.pos, self.slots)
            if peer is not None and sharded is None:
                peer.read_merge(ws, self.q, qsl, self.seq, scale, o_l, lse_l, self.out)
            elif sharded is not None and fused:
                sharded.step_merge(self.q, qsl, self.seq, scale, o_l, lse_l, self.out, fused=True)
            elif sharded is not None:  # far read, then the exchange of the step (peer or NCCL) and the merge
                o_all, lse_all = sharded.step(self.q, qsl, self.seq, scale)
                sharded.merge(o_l, lse_l, o_all, lse_all, self.out, qsl, self.seq)
            else:
                o_part, lse_part = ws.read_far(self.q, qsl, self.seq, scale)
                kernels.merge(o_l, lse_l, o_part, lse_part, self.out, qsl, self.seq, window=W, block=B, alpha=ALPHA)

    slots = (Slot(), Slot())
    compute = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # capture after one eager run of each (every rank captures the same collectives in the same order)
    for sl in slots:
        sl.d_in.copy_(h_in[0])
        sl.layer_step()
    torch.cuda.synchronize()
    for sl in slots:
        sl.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(sl.graph):
            sl.layer_step()
    torch.cuda.synchronize()

    def upload(i):
        sl = slots[i % 2]
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(sl.computed)  # step i-2 has finished reading this record
            sl.d_in.copy_(h_in[i], non_blocking=True)
            sl.uploaded.record(up)

    def step(i, last):
        sl = slots[i % 2]
        compute.wait_event(sl.uploaded)
        if i >= 2:
            compute.wait_event(sl.read)  # step i-2's output has been read back
        sl.graph.replay()
        sl.computed.record(compute)
        if i + 1 < last:
            upload(i + 1)
        with torch.cuda.stream(down):
            down.wait_event(sl.computed)
            h_out[i % 2].copy_(sl.out, non_blocking=True)
            sl.read.record(down)

    def run(first, last):
        upload(first)
        for i in range(first, last):
            step(i, last)
        compute.wait_stream(down)

    def run_serial(first, last):
        """One step after the other as a drafter must take them (step i + 1's query depends on
        step i's output): upload, replay, read back, each ordered after the last on one stream,
        so no copy overlaps any step's compute."""
        sl = slots[0]
        for i in range(first, last):
            sl.d_in.copy_(h_in[i], non_blocking=True)
            sl.graph.replay()
            h_out[0].copy_(sl.out, non_blocking=True)

    def timed(fn):
        """fn(warmup + ...) steps timed with events on the compute stream after untimed passes
        (the same sustained load and power-capped clock as the device-timed step; rank 0's pass
        count), max over ranks."""
        fn(0, args.warmup)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fn(args.warmup, total)
        torch.cuda.synchronize()
        pre = torch.tensor([max(0, min(20, int(0.3 / max(time.perf_counter() - t0, 1e-4))))], device=dev)
        if world > 1:
            dist.broadcast(pre, src=0)
        for _ in range(int(pre.item())):
            fn(args.warmup, total)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
            dist.all_reduce(torch.zeros(1, device=dev))  # device-aligned start (see align() above)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        fn(args.warmup, total)
        e1.record(compute)
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return 1000.0 * float(ms) / args.steps

    us_serial = timed(run_serial)
    us_pipelined = timed(run)
    for sl in slots:
        sl.graph = None  # graphs that hold collectives go before the process group
    torch.cuda.synchronize()
    if sharded is not None and sharded.peer is not None and sharded.peer is not peer:
        sharded.peer.close()
    api = ("FoldWorkspace.append + " + (
        "PeerExchange.read_merge (far read + merge in one cooperative kernel)" if peer is not None and
        sharded is None else "ShardedFarMemory.step_merge (far read + peer exchange + merge in one "
        "cooperative kernel)" if sharded is not None and fused else
        f"ShardedFarMemory.step + merge ({args.exchange} exchange)" if sharded is not None
        else "FoldWorkspace.read_far + kernels.merge") + " (fold_b200 C-ABI), captured once per input buffer in a "
        "CUDA graph and replayed per step")
    return {"value": round(us_serial, 3), "unit": "us/draft-step",
            "h2d_bytes_per_step": rec, "d2h_bytes_per_step": B * hq * hd * 2,
            "api": api + "; per step, serially on one stream: one pinned host->device copy of the step's inputs, "
                         "the replay, one device->host copy of its output, then the next step's copy",
            "pipelined": {"value": round(us_pipelined, 3), "unit": "us/draft-step",
                          "how": "the same steps with the copies on their own streams, double-buffered so that "
                                 "step i + 1's upload and step i - 1's read-back overlap step i (throughput of "
                                 "independent steps, not a draft-step latency)"}}


# ------------------------------------------------------------------------------ reference arm
def port_step_heads(cfg, H, q, k, v, o_l, lse_l, inv_freq, kv_heads):
    """The oracle port's far query + far read + merge of one step, restricted to the given KV
    heads and their query heads (query heads are independent)."""
    G = cfg["hq"] // cfg["hkv"]
    qh = np.concatenate([np.arange(h * G, (h + 1) * G) for h in kv_heads])
    sub = dict(cfg, hq=len(qh), hkv=len(kv_heads))
    return cpu_step_oracle(sub, H, q[:, qh], k[:, kv_heads], v[:, kv_heads], o_l[:, qh], lse_l[qh], inv_freq)


def reference_module():
    """fold.reference of the reference package installed under baseline/_ref, or the import error."""
    path = ROOT / "baseline" / "_ref"
    if not (path / "fold" / "reference.py").exists():
        return None, "the reference is not installed under baseline/_ref"
    sys.path.insert(0, str(path))
    try:
        from fold import reference as ref  # noqa: PLC0415
        return ref, None
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        return None, f"import of fold.reference failed: {type(e).__name__}: {e}"


def time_fold_block(cfg, H, steps, warm, seed, budget_s=120.0):
    """The reference's own CPU implementation, fold.reference.fold_block (fold/reference.py:21-53),
    timed head-sliced: each step runs the whole draft block for one query head with its KV head
    (GQA expanded, as fold_block requires; heads are independent), and the figure is scaled to all
    query heads. Steps are the arm's own; if they do not fit the budget, every k-th is timed."""
    import torch

    ref, why = reference_module()
    if ref is None:
        return {"unavailable": why}
    hq, hkv, hd, B, W = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["B"], cfg["W"]
    G = hq // hkv
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(seed + 11)
    L = int(H.max())
    k_all = torch.randn((L, hkv, hd), generator=gen)
    v_all = torch.randn((L, hkv, hd), generator=gen)
    q_all = torch.randn((B, hq, hd), generator=gen)
    kb, vb = torch.randn((B, hkv, hd), generator=gen), torch.randn((B, hkv, hd), generator=gen)
    inv = torch.from_numpy((1.0 / (cfg["theta"] ** (np.arange(0, hd, 2) / hd))).astype(np.float32))

    def one(i):
        h = i % hq
        kv = h // G
        t = int(H[i])
        return ref.fold_block(q_all[:, h:h + 1], k_all[:t, kv:kv + 1], v_all[:t, kv:kv + 1], kb[:, kv:kv + 1],
                              vb[:, kv:kv + 1], window=W, alpha=ALPHA, inv_freq=inv, scale=hd ** -0.5)

    t0 = time.perf_counter()
    one(0)
    first = time.perf_counter() - t0
    every = max(1, int(np.ceil((steps + warm) * first / budget_s)))
    times = []
    for i in range(warm + steps):
        if i % every:
            continue
        t0 = time.perf_counter()
        one(i)
        if i >= warm:
            times.append(time.perf_counter() - t0)
    if not times:
        return {"unavailable": "no timed step fitted the budget"}
    out = {"value": round(1e6 * float(np.mean(times)) * hq, 1), "unit": "us/draft-step", "kind": "reference",
           "cores": torch.get_num_threads(),
           "sample": f"fold.reference.fold_block (baseline/_ref, unmodified) on one of the {hq} query heads per "
                     f"step (GQA expanded), {len(times)} timed steps of the {cfg['name']} workload"
                     + (f" (every {every}th step of the arm's {steps})" if every > 1 else "")
                     + f", scaled by {hq} heads; float64 inside, as the reference computes"}
    torch.set_num_threads(1)
    t0 = time.perf_counter()
    one(warm)
    out["value_1_thread"] = round(1e6 * (time.perf_counter() - t0) * hq, 1)
    torch.set_num_threads(os.cpu_count() or 1)
    return out


def run_reference(args):
    """The reference arm: the CPU implementation of the path on all host threads, over the arm's
    own steps and warm-up, on the GPU arm's workload and metric. `value` is the oracle port's far
    query + far read + merge (the work the GPU arm's metric counts; each step samples KV heads
    when the whole step would not fit the time budget, scaled to all heads). The reference's own
    fold_block (the whole FOLD block, local read and key rotation included) is timed beside it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    from oracle import fold_oracle as fo

    steps, warm = max(1, args.steps), max(0, args.warmup)
    hkv = cfg["hkv"]
    acc, H = plan_steps(cfg, steps + warm, args.seed)
    q, k, v, o_l, lse_l = cpu_inputs(cfg, args.seed, int(H.max()))
    f = fo.inv_freq(cfg["theta"], cfg["hd"])
    t0 = time.perf_counter()
    port_step_heads(cfg, int(H[0]), q, k, v, o_l, lse_l, f, [0])
    per_head = time.perf_counter() - t0
    budget = 120.0
    kv_sample = int(max(1, min(hkv, budget / max((steps + warm) * per_head, 1e-9))))
    times = []
    for i in range(warm + steps):
        heads = [(i * kv_sample + j) % hkv for j in range(kv_sample)]
        t0 = time.perf_counter()
        port_step_heads(cfg, int(H[i]), q, k, v, o_l, lse_l, f, heads)
        if i >= warm:
            times.append(time.perf_counter() - t0)
    us = 1e6 * float(np.mean(times)) * hkv / kv_sample
    cores = os.cpu_count() or 1
    sample = (f"{steps} draft steps of the {cfg['name']} workload after {warm} warm-up steps: float64 numpy port of "
              f"fold/reference.py's far query + far read + merge (BLAS on {cores} threads), "
              + ("all KV heads per step" if kv_sample == hkv else
                 f"{kv_sample} of {hkv} KV heads per step (with their query heads), scaled to {hkv}"))
    line = {"impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/draft-step",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": steps, "warmup": warm,
            "ms_per_step": round(us / 1000, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": cfg["name"], "context": cfg["ctx"], "window": cfg["W"], "block": cfg["B"],
                       "heads_q": cfg["hq"], "heads_kv": cfg["hkv"], "head_dim": cfg["hd"], "alpha": ALPHA},
            "cpu_baseline": {"value": round(us, 1), "unit": "us/draft-step", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(us, 1), "unit": "us/draft-step", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "reference_fold_block": time_fold_block(cfg, H, steps, warm, args.seed)}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        if args.impl == "fa4":
            args.no_e2e = args.no_cpu = True
        run_gpu(args)


if __name__ == "__main__":
    main()
