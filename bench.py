#!/usr/bin/env python
"""MLA decode benchmark -- prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload cfg1|cfg2|cfg3|cfg4]

Multi-GPU runs are launched by torchrun (one process per GPU, NCCL); RANK /
LOCAL_RANK / WORLD_SIZE come from the environment.

Workloads (seeded synthetic inputs with the BASELINE shapes; no dataset exists):
  cfg1 (default)  DeepSeek-V2 decode step, B=1 per GPU, H=128, L=8192, bf16.
                  N GPUs run N independent sequences (batch-sharded, weak scaling).
  cfg2            B=64 sequences, L_b ~ U[1024, 16384], sharded by batch (LPT) over GPUs.
  cfg3            B=1, L=131072, KV-range sharded over GPUs; per-head partials
                  (m, l, o_latent) are all-gathered with NCCL and merged.
  cfg4            B=256, L=4096 (DeepSeek-V3 shape), sharded by batch.

A step = Q absorption (q_nope @ W_UK) + split-KV latent attention over the cache
+ log-sum-exp combine + W_UV projection, i.e. one pass of the decode hot path.
The metric is the latent-cache bytes a step reads divided by the step time
(whole job: summed over GPUs, time = max over GPUs); the step time itself is
reported as ms_per_step / us_per_step. L2 is flushed (256 MiB write) before
every timed step because the config-1 inputs fit in the 126 MB L2.

Device-timed leg: each timed step is one replay of a CUDA graph captured from the
public call (latent_attn.functional.mla_decode, or the KV-range decoder with its
NCCL all-gather on several GPUs), so the events bracket the step's kernels rather
than the host's time to enqueue them (--eager launches it directly). The roofline's
decode-kernel time comes from a second loop of the same steps, each carrying the
library's kernel timer. Graphs that hold NCCL calls are released before the process
group is destroyed.
The end-to-end leg calls the public API every step, with the host copies inside.
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "latent-attn_b200"))

CACHE_ROW_BYTES = 576 * 2          # one packed [c_t | k_rope] row in bf16 (the per-position unit)
HBM_FALLBACK_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4"], default="cfg1")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch the device-timed steps directly, not from CUDA graphs")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return HBM_FALLBACK_GBS, "fallback (6.65 TB/s, earlier pool measurement)"


def ncu_traffic(workload, share=1.0):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary (a one-GPU launch
    over the whole workload), scaled by the share of the workload's cache rows this rank's launch
    decodes (the traffic grows in proportion to the rows); None without a summary."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        t = d.get(workload)
        return None if t is None else int(round(t * share))
    return None


# ----------------------------------------------------------------------------- workloads

def workload_spec(name):
    from latent_attn import synthetic
    if name == "cfg1":
        return dict(name=name, lens=[8192], sharding="batch-replica", desc=(
            "config 1: DeepSeek-V2 MLA decode, B=1 per GPU, H=128, L=8192, bf16"))
    if name == "cfg2":
        return dict(name=name, lens=synthetic.varlen_lengths(64, 1024, 16384, seed=0), sharding="batch",
                    desc="config 2: B=64 variable-length decode, L_b~U[1024,16384], H=128, bf16")
    if name == "cfg3":
        return dict(name=name, lens=[131072], sharding="kv-range",
                    desc="config 3: B=1, L=131072, H=128, bf16, KV-range sharded + NCCL combine")
    return dict(name=name, lens=[4096] * 256, sharding="batch",
                desc="config 4: B=256, L=4096, H=128 (DeepSeek-V3 MLA dims), bf16")


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu_id)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, begin):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((ts, float(parts[1]), float(parts[2]), parts))
            except ValueError:
                continue
        if not rows:
            return None
        inside = [r for r in rows if self.t0 and self.t1 and self.t0 - 0.06 <= r[0] <= self.t1 + 0.06]
        use = inside if inside else rows
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in use:
            for name, val in zip(names, r[3][5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[1] for r in use), "sm_max_mhz": max(r[2] for r in use),
                "reasons": sorted(reasons), "samples": len(use),
                "window": "timed region" if inside else "whole run (timed region shorter than the sampling period)"}


# ----------------------------------------------------------------------------- CPU oracle leg

def cpu_oracle_rate(lens, seconds, H=128):
    """Time the oracle's restatement of the reference's torch-CPU MLA decode
    (decompress-then-attend, fp32 numpy) on the workload's first sequence; returns
    (GB/s of latent cache, cores, sample description)."""
    import numpy as np
    from oracle import mla_oracle as O
    from latent_attn import synthetic
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [os.cpu_count() or 1])
    except Exception:  # pragma: no cover
        cores = os.cpu_count() or 1
    L = lens[0]
    inp = synthetic.baseline_inputs(num_heads=H, seq_lens=[L], seed=0)
    kv = inp.kv_cache.float().numpy()
    WK, WV = inp.W_UK.float().numpy(), inp.W_UV.float().numpy()
    qn, qr = inp.q_nope[0].float().numpy(), inp.q_rope[0].float().numpy()
    cos, sin = O.rope_tables(L, 64)
    # size the sample: full steps if they fit the budget, else a head subset
    t0 = time.perf_counter()
    O.naive_decode(kv, WK[:16 * 128], WV[:16 * 128], qn[:16], qr[:16], cos, sin, 16, 512, 128, 64, 128)
    est_full = (time.perf_counter() - t0) * H / 16
    heads = H if est_full < seconds / 3 else max(16, int(16 * (seconds / 3) / max(est_full * 16 / H, 1e-9)) // 16 * 16)
    heads = min(heads, H)
    n, t_total = 0, 0.0
    while t_total < seconds or n == 0:
        t0 = time.perf_counter()
        O.naive_decode(kv, WK[:heads * 128], WV[:heads * 128], qn[:heads], qr[:heads], cos, sin, heads, 512,
                       128, 64, 128)
        t_total += time.perf_counter() - t0
        n += 1
        if n >= 200:
            break
    per_step = t_total / n * (H / heads)
    gbs = L * CACHE_ROW_BYTES / per_step / 1e9
    sample = (f"{n} step(s) of the oracle's decompress-then-attend decode (numpy fp32, restating the reference's "
              f"torch_mla_reference) on B=1, L={L}, {heads} of {H} heads, scaled to {H} heads; "
              f"{per_step * 1e3:.1f} ms per full step")
    return gbs, cores, sample


# ----------------------------------------------------------------------------- reference arm

def json_stdout():
    """The real stdout, kept for the one JSON line; file descriptor 1 then goes to stderr, so whatever
    else libraries print there (NCCL's version banner on rank 0, for one) cannot add lines to it."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def run_reference(args, rank, out):
    if rank != 0:
        return
    spec = workload_spec(args.workload)
    budget = max(10.0, min(150.0, 8.0 * (args.steps + args.warmup)))
    gbs, cores, sample = cpu_oracle_rate(spec["lens"], budget)
    line = {
        "impl": "reference", "metric": "MLA decode latent-cache GB/s", "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": spec["desc"], "batch_per_gpu": 1, "seq_len": spec["lens"][0], "heads": 128},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ms_per_step": round(spec["lens"][0] * CACHE_ROW_BYTES / gbs / 1e6, 4),
    }
    print(json.dumps(line), file=out, flush=True)


# ----------------------------------------------------------------------------- main arm

def main():
    json_out = json_stdout()
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, json_out)
        return

    import torch
    import torch.distributed as dist
    from latent_attn import MLAConfig, synthetic, _lib
    from latent_attn.functional import mla_decode
    from latent_attn import _C
    from latent_attn.distributed import KVRangeDecoder, kv_range, lpt_shard

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    cfg = MLAConfig.deepseek_v2()
    spec = workload_spec(args.workload)
    lens_all = spec["lens"]

    # ---- this rank's share of the workload
    if spec["sharding"] == "batch-replica":
        my_lens = lens_all
        seed = 1000 + rank
    elif spec["sharding"] == "batch":
        my_lens = [lens_all[i] for i in lpt_shard(lens_all, world)[rank]]
        seed = 2000 + rank
    else:  # kv-range: contiguous slice of the single sequence
        L = lens_all[0]
        lo, hi = kv_range(L, world, rank)
        my_lens = [hi - lo]
        seed = 0
    if spec["sharding"] == "kv-range":
        full = synthetic.baseline_inputs(num_heads=128, seq_lens=lens_all, seed=seed)
        kv_host = full.kv_cache[lo:hi].contiguous()
        inp = full
        pos_offset = lo
    else:
        inp = synthetic.baseline_inputs(num_heads=128, seq_lens=my_lens, seed=seed)
        kv_host = inp.kv_cache
        pos_offset = 0
    B = inp.batch if spec["sharding"] != "kv-range" else 1
    kv = kv_host.to(dev)
    W_UK, W_UV = inp.W_UK.to(dev), inp.W_UV.to(dev)
    q_nope, q_rope = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    Lmax = max(lens_all) if spec["sharding"] == "kv-range" else max(my_lens)
    cos, sin = synthetic.build_rope_tables(max(lens_all), 64, device=dev)
    seq = offs = None
    if spec["sharding"] == "batch" and len(set(my_lens)) > 1:
        seq = torch.tensor(my_lens, dtype=torch.int32, device=dev)
        offs = torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev)
    out = torch.empty(B, 128, 128, dtype=torch.float32, device=dev)
    ws = torch.empty(1 << 28, dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    dims = (cfg.d_model, 512, 128, 64, 128, 128)
    bytes_per_step = sum(my_lens) * CACHE_ROW_BYTES

    if spec["sharding"] == "kv-range":
        sharded = KVRangeDecoder(cfg) if world > 1 else None

        def step(q_n=q_nope, q_r=q_rope, o=out, t=None):
            if sharded is not None:
                return sharded(kv, q_r, W_UV, cos, sin, pos_offset=pos_offset, q_nope=q_n, W_UK=W_UK, out=o,
                               workspace=ws, timer=t)
            ml, oo = _C.mla_decode_partial(kv, q_r, W_UV, cos, sin, *dims, q_nope=q_n, W_UK=W_UK,
                                           kv_pos_offset=pos_offset, workspace=ws, timer=t)
            return _C.mla_combine_partials(ml.unsqueeze(0), oo.unsqueeze(0), W_UV, *dims, out=o)
    else:
        def step(q_n=q_nope, q_r=q_rope, o=out, t=None):
            return mla_decode(kv, q_r, W_UV, cos, sin, cfg, q_nope=q_n, W_UK=W_UK, seq_lens=seq, kv_offsets=offs,
                              max_seq_len=Lmax, seq_lens_host=my_lens if seq is not None else None, out=o,
                              workspace=ws, timer=t)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    # ---- warmup
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()

    gpu_uuid = str(local_rank)
    try:
        gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
        if not gpu_uuid.startswith("GPU-"):
            gpu_uuid = "GPU-" + gpu_uuid
    except Exception:
        pass
    clocks = ClockSampler(gpu_uuid)
    clocks.start()
    time.sleep(0.15)

    # ---- device-timed region: K steps, each bracketed by CUDA events on the launching stream.
    # The steps run as a user's call runs (no timer, so the decode kernel overlaps the absorption
    # through programmatic dependent launch). A second loop of K steps, each with a decode-kernel
    # timer (which keeps the decode kernel from overlapping its neighbours, so the events bracket it
    # exactly), gives the kernel time for the roofline. Nothing in either loop waits for the device:
    # timers and the decode status word are read afterwards (the status is summed on the device).
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    timers = [_lib.DecodeTimer() for _ in range(args.steps)]
    status_word = ws[:4].view(torch.int32)
    status_sum = torch.zeros(1, dtype=torch.int32, device=dev)
    host_s = 0.0
    use_graphs = not args.eager
    graphs = []        # every graph, so all can be released before process-group teardown
    timed = []
    if use_graphs:
        launches0 = _lib.kernel_launch_count()
        side = torch.cuda.Stream(dev)
        graphs.append(torch.cuda.CUDAGraph())   # the step without a timer
        with torch.cuda.graph(graphs[0], stream=side):
            step()
        per_step = _lib.kernel_launch_count() - launches0
        for k in range(args.steps):             # one graph per timed step of the roofline loop
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], stream=side):
                step(t=timers[k])
            timed.append(graphs[-1])
        for g in graphs[:4]:
            g.replay()
        torch.cuda.synchronize(dev)
    launches0 = _lib.kernel_launch_count()
    barrier()
    clocks.mark(True)
    for k in range(args.steps):
        flush.zero_()
        ev0[k].record(stream)
        h0 = time.perf_counter()
        if use_graphs:
            graphs[0].replay()
        else:
            step()
        host_s += time.perf_counter() - h0
        ev1[k].record(stream)
        status_sum.add_(status_word[:1].clamp(0, 1))
    barrier()
    clocks.mark(False)
    launches = _lib.kernel_launch_count() - launches0
    if use_graphs:
        launches = int(round(per_step * args.steps))  # the graph's kernels, counted when captured
    # roofline loop: the same steps, each with its decode-kernel timer
    for k in range(args.steps):
        flush.zero_()
        if use_graphs:
            timed[k].replay()
        else:
            step(t=timers[k])
        status_sum.add_(status_word[:1].clamp(0, 1))
    barrier()
    # before any process-group teardown: a graph that holds NCCL calls keeps the teardown waiting
    timed.clear()
    for gr in graphs:
        gr.reset()
    graphs.clear()
    torch.cuda.synchronize(dev)
    step_ms = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]
    dec_ms = [t.decode_ms() for t in timers]
    for t in timers:
        t.close()
    status_errors = int(status_sum.item())
    total_ms = sum(step_ms)

    # ---- end-to-end: host buffers, H2D of the step's queries and D2H of the output inside the timed span
    # the step's queries live in one pinned host buffer (q_nope then q_rope), so one copy uploads them
    nqn, nqr = q_nope.numel(), q_rope.numel()
    q_h = torch.empty(nqn + nqr, dtype=torch.float32).pin_memory()
    q_h[:nqn].copy_(inp.q_nope.float().reshape(-1))
    q_h[nqn:].copy_(inp.q_rope.float().reshape(-1))
    qn_h, qr_h = q_h[:nqn], q_h[nqn:]
    out_h = torch.empty(B, 128, 128, dtype=torch.float32).pin_memory()
    q_d = torch.empty(nqn + nqr, dtype=torch.float32, device=dev)
    qn_d, qr_d = q_d[:nqn].view(q_nope.shape), q_d[nqn:].view(q_rope.shape)
    e2e_ms = []
    barrier()
    for k in range(args.steps):
        flush.zero_()
        ev0[k].record(stream)
        q_d.copy_(q_h, non_blocking=True)
        o = step(q_n=qn_d, q_r=qr_d)
        out_h.copy_(o, non_blocking=True)
        ev1[k].record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms.append(ev0[k].elapsed_time(ev1[k]))
    barrier()
    clock_info = clocks.stop()
    h2d = qn_h.numel() * 4 + qr_h.numel() * 4
    d2h = out_h.numel() * 4
    e2e_total = sum(e2e_ms)

    # ---- max over ranks
    t = torch.tensor([total_ms, e2e_total], dtype=torch.float64, device=dev)
    nbytes = torch.tensor([bytes_per_step], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(nbytes, op=dist.ReduceOp.SUM)
    total_max, e2e_max = float(t[0]), float(t[1])
    job_bytes = float(nbytes[0])
    value = job_bytes * args.steps / total_max / 1e6          # bytes / ms -> GB/s
    e2e_value = job_bytes * args.steps / e2e_max / 1e6

    if rank == 0:
        peak, peak_src = measured_peaks()
        roof = None
        if dec_ms:
            dmean = statistics.mean(dec_ms)
            achieved = bytes_per_step / dmean / 1e6
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4),
                    "traffic": ncu_traffic(args.workload, sum(my_lens) / sum(lens_all)),
                    "kernel": "mla::decode_sm100_kernel", "kernel_us": round(dmean * 1e3, 3),
                    "algorithmic_bytes": bytes_per_step, "peak_source": peak_src + " -- fraction is of measured"}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            gbs, cores, sample = cpu_oracle_rate(lens_all, args.cpu_seconds)
            cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
        B_job = len(lens_all) if spec["sharding"] != "batch-replica" else world
        line = {
            "metric": "MLA decode latent-cache GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_max / args.steps, 5),
            "us_per_step": round(total_max / args.steps * 1e3, 2),
            "tokens_per_s": round(B_job * args.steps / (total_max / 1e3), 1),
            "higher_is_better": True,
            "scaling": "weak" if spec["sharding"] == "batch-replica" else "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) cache rows and queries, N(0,1/sqrt(512)) W_UK/W_UV",
            "config": {"workload": spec["desc"], "batch_per_gpu": B if spec["sharding"] != "kv-range" else 1,
                       "seq_len": max(lens_all), "heads": 128, "kv_lora_rank": 512, "qk_rope_head_dim": 64,
                       "parallelism": {"batch-replica": f"dp{world} (one sequence per GPU, no collective)",
                                       "batch": f"batch-sharded over {world} GPU(s), LPT, no collective",
                                       "kv-range": f"KV-range over {world} GPU(s) + NCCL all-gather"}[spec["sharding"]],
                       "l2": "flushed before every timed step (256 MiB write outside the events)"},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_max / args.steps, 5),
                    "api": "latent_attn.functional.mla_decode (q_nope/q_rope pinned host -> device, output -> host)"},
            "gpu_launches": int(launches),
            "launch": "cuda-graph replay per step" if use_graphs else "direct",
            "host_us_per_step_call": round(host_s / args.steps * 1e6, 1),
            "decode_status_errors": status_errors,
            "output_finite": bool(torch.isfinite(out).all()),
            "clocks": clock_info,
        }
        print(json.dumps(line), file=json_out, flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
