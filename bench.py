#!/usr/bin/env python
"""MLA decode benchmark -- prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload cfg1|cfg2|cfg3|cfg4]
                    [--rope otf|tables] [--no-extra]

Multi-GPU runs are launched by torchrun (one process per GPU, NCCL); RANK /
LOCAL_RANK / WORLD_SIZE come from the environment.

Workloads (seeded synthetic inputs with the BASELINE shapes; no dataset exists):
  cfg1 (default)  DeepSeek-V2 decode step, B=1 per GPU, H=128, L=8192, bf16.
                  N GPUs run N independent sequences (batch-sharded, weak scaling).
  cfg2            B=64 sequences, L_b ~ U[1024, 16384], sharded by batch (LPT) over GPUs.
  cfg3            B=1, L=131072, KV-range sharded over GPUs; per-head partials
                  (m, l, o_latent) go to the rank owning the head (put kernels storing
                  into the peers' memory over NVLink), which merges and projects them,
                  and the outputs go back to every rank the same way.
  cfg4            B=256, L=4096 (DeepSeek-V3 shape), sharded by batch.

A step = Q absorption (q_nope @ W_UK) + split-KV latent attention over the cache
+ log-sum-exp combine + W_UV projection, i.e. one pass of the decode hot path.
The metric is the latent-cache bytes a step reads divided by the step time
(whole job: summed over GPUs, time = max over GPUs); the step time itself is
reported as ms_per_step / us_per_step. L2 is flushed (256 MiB write) before
every timed step because the config-1 inputs fit in the 126 MB L2.

Device-timed leg: each timed step is one replay of a CUDA graph captured from the
public call (latent_attn.functional.mla_decode, or the KV-range decoder with its
peer-memory exchange on several GPUs), so the events bracket the step's kernels rather
than the host's time to enqueue them (--eager launches it directly). The roofline's
decode-kernel time comes from a second loop of the same steps, each carrying the
library's kernel timer. Graphs are released, and the exchange's peer buffers closed,
before the process group is destroyed.
The end-to-end leg calls the public API every step, with the host copies inside.

RoPE: by default the step passes no cos/sin tables, so the kernels compute the
rotation themselves (on-the-fly mode, no table traffic); --rope tables passes the
reference's fp32 tables instead.

Besides the headline workload, the same line carries the other BASELINE
configurations measured in the same run ("workloads": step time, cache GB/s and
the decode kernel's fraction of the HBM peak): on one GPU configs 2, 3 and 4; on
several GPUs config 3 KV-range sharded with its exchange (an all-to-all of per-head
partials, then an all-gather of the outputs, both as the library's own put / wait
kernels storing into the peers' memory over NVLink) and config 4
batch-sharded. Their inputs are drawn on the device with the same distributions.
The CPU leg also times BASELINE config 0 (H=16, L=1024, fp32) on the host.
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


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4"], default="cfg1")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch the device-timed steps directly, not from CUDA graphs")
    ap.add_argument("--rope", choices=["otf", "tables"], default="otf",
                    help="otf: the kernels compute cos/sin (no tables); tables: pass the fp32 tables")
    ap.add_argument("--no-extra", action="store_true", help="skip the other configurations' legs")
    ap.add_argument("--extra-steps", type=int, default=10, help="timed steps of each extra leg")
    return ap.parse_args(argv)


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return HBM_FALLBACK_GBS, "fallback (6.65 TB/s, earlier pool measurement)"


def measured_tensor_peak():
    """Sustained dense bf16 TFLOP/s (MEASURED_PEAKS.json), the denominator for a kernel timed inside a long step."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    return 1400.0, "fallback (1.4 PFLOP/s sustained, earlier pool measurement)"


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
                    desc="config 3: B=1, L=131072, H=128, bf16, KV-range sharded + exchange of per-head partials")
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


# ----------------------------------------------------------------------------- CPU legs

def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info()] or [os.cpu_count() or 1])
    except Exception:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_model():
    """The host CPU's model name (first processor of /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:  # pragma: no cover
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_oracle_rate(lens, seconds, H=128):
    """Time the oracle's restatement of the reference's torch-CPU MLA decode
    (decompress-then-attend, fp32 numpy) on the workload's first sequence; returns
    (GB/s of latent cache, cores, sample description)."""
    from oracle import mla_oracle as O
    from latent_attn import synthetic
    cores = cpu_threads()
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


def cpu_config0(iters=20, warmup=3):
    """BASELINE config 0 on the host: B=1, H=16, L=1024, fp32 inputs, the oracle's numpy
    restatement of the reference's torch_mla_reference; median of `iters` after `warmup`."""
    from oracle import mla_oracle as O
    from latent_attn import synthetic
    import torch
    L, H = 1024, 16
    inp = synthetic.baseline_inputs(num_heads=H, seq_lens=[L], seed=0, dtype=torch.float32)
    kv = inp.kv_cache.numpy()
    WK, WV = inp.W_UK.numpy(), inp.W_UV.numpy()
    qn, qr = inp.q_nope[0].numpy(), inp.q_rope[0].numpy()
    cos, sin = O.rope_tables(L, 64)
    ts = []
    for i in range(warmup + iters):
        t0 = time.perf_counter()
        O.naive_decode(kv, WK, WV, qn, qr, cos, sin, H, 512, 128, 64, 128)
        if i >= warmup:
            ts.append(time.perf_counter() - t0)
    ms = statistics.median(ts) * 1e3
    return {"ms_per_step": round(ms, 3), "GBps": round(L * 576 * 4 / (ms / 1e3) / 1e9, 4),
            "cores": cpu_threads(), "cpu_model": cpu_model(),
            "what": "config 0 (B=1, H=16, L=1024, fp32): the oracle's numpy restatement of the reference's "
                    f"torch_mla_reference, median of {iters} after {warmup} warm-ups"}


# ----------------------------------------------------------------------------- shared line pieces

def config_of(spec, world):
    """The line's `config` object; both arms print the same one."""
    B_per = len(spec["lens"]) if spec["sharding"] == "batch" else 1
    return {"workload": spec["desc"],
            "batch_per_gpu": B_per if spec["sharding"] != "batch" else f"{len(spec['lens'])} over {world} GPU(s)",
            "seq_len": max(spec["lens"]), "heads": 128, "kv_lora_rank": 512, "qk_rope_head_dim": 64,
            "parallelism": {"batch-replica": f"dp{world} (one sequence per GPU, no collective)",
                            "batch": f"batch-sharded over {world} GPU(s), LPT, no collective",
                            "kv-range": f"KV-range over {world} GPU(s) + peer-memory (NVLink stores) all-to-all of "
                                        "head slices and output all-gather"}[spec["sharding"]],
            "l2": "flushed before every timed step (256 MiB write outside the events)"}


# ----------------------------------------------------------------------------- reference arm

def json_stdout():
    """The real stdout, kept for the one JSON line; file descriptor 1 then goes to stderr, so whatever
    else libraries print there (NCCL's version banner on rank 0, for one) cannot add lines to it."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def run_reference(args, rank, world, out):
    if rank != 0:
        return
    spec = workload_spec(args.workload)
    budget = max(10.0, min(150.0, 8.0 * (args.steps + args.warmup)))
    gbs, cores, sample = cpu_oracle_rate(spec["lens"], budget)
    sample += f"; CPU: {cpu_model()}"
    line = {
        "impl": "reference", "metric": "MLA decode latent-cache GB/s", "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak" if spec["sharding"] == "batch-replica" else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": config_of(spec, world),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ms_per_step": round(spec["lens"][0] * CACHE_ROW_BYTES / gbs / 1e6, 4),
    }
    print(json.dumps(line), file=out, flush=True)


# ----------------------------------------------------------------------------- main arm

def device_inputs(lens, dev, seed, H=128):
    """Seeded inputs drawn on the device with the benchmark recipe's distributions (cache rows,
    q_nope, q_rope ~ N(0, 1); W_UK, W_UV ~ N(0, 1/sqrt(512))), for the extra legs."""
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    total = sum(lens)
    kv = torch.empty(total, 576, dtype=torch.bfloat16, device=dev)
    for r0 in range(0, total, 1 << 18):  # in slices: no fp32 copy of the whole cache
        r1 = min(total, r0 + (1 << 18))
        kv[r0:r1] = torch.randn(r1 - r0, 576, generator=g, device=dev)
    B = len(lens)
    q_nope = torch.randn(B, H, 128, generator=g, device=dev)
    q_rope = torch.randn(B, H, 64, generator=g, device=dev)
    W_UK = (torch.randn(H * 128, 512, generator=g, device=dev) / math.sqrt(512)).to(torch.bfloat16)
    W_UV = (torch.randn(H * 128, 512, generator=g, device=dev) / math.sqrt(512)).to(torch.bfloat16)
    offs = [0]
    for L in lens[:-1]:
        offs.append(offs[-1] + L)
    return kv, q_nope, q_rope, W_UK, W_UV, offs


def build_step(spec, world, rank, dev, cfg, rope, ws, host_inputs):
    """This rank's share of a workload and a step function over it.

    Returns (step(q_n, q_r, o, t), inputs dict, cache bytes this rank's step reads, batch)."""
    import torch
    from latent_attn import synthetic, _C
    from latent_attn.functional import mla_decode
    from latent_attn.distributed import KVRangeDecoder, kv_range, lpt_shard
    lens_all = spec["lens"]
    if spec["sharding"] == "batch-replica":
        my_lens, seed, lo = lens_all, 1000 + rank, 0
    elif spec["sharding"] == "batch":
        my_lens, seed, lo = [lens_all[i] for i in lpt_shard(lens_all, world)[rank]], 2000 + rank, 0
    else:
        lo, hi = kv_range(lens_all[0], world, rank)
        my_lens, seed = [hi - lo], 0
    inp = None
    if host_inputs:
        if spec["sharding"] == "kv-range":
            inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens_all, seed=seed)
            kv = inp.kv_cache[lo:lo + my_lens[0]].contiguous().to(dev)
        else:
            inp = synthetic.baseline_inputs(num_heads=128, seq_lens=my_lens, seed=seed)
            kv = inp.kv_cache.to(dev)
        W_UK, W_UV = inp.W_UK.to(dev), inp.W_UV.to(dev)
        q_nope, q_rope = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
        offs_l = inp.kv_offsets
    else:
        kv, q_nope, q_rope, W_UK, W_UV, offs_l = device_inputs(my_lens, dev, seed)
    B = len(my_lens) if spec["sharding"] != "kv-range" else 1
    Lmax = max(lens_all) if spec["sharding"] == "kv-range" else max(my_lens)
    if rope == "tables":
        cos, sin = synthetic.build_rope_tables(max(lens_all), 64, device=dev)
    else:
        cos = sin = None
    seq = offs = None
    if spec["sharding"] == "batch" and len(set(my_lens)) > 1:
        seq = torch.tensor(my_lens, dtype=torch.int32, device=dev)
        offs = torch.tensor(offs_l, dtype=torch.int64, device=dev)
    out = torch.empty(B, 128, 128, dtype=torch.float32, device=dev)
    if spec["sharding"] == "kv-range" and world > 1:
        sharded = KVRangeDecoder(cfg)

        # the output lands in the exchange's own buffer (every rank's rows stored there by the peers)
        def step(q_n=q_nope, q_r=q_rope, o=None, t=None):
            return sharded(kv, q_r, W_UV, cos, sin, pos_offset=lo, q_nope=q_n, W_UK=W_UK, out=o, workspace=ws,
                           timer=t)
    else:
        def step(q_n=q_nope, q_r=q_rope, o=out, t=None):
            return mla_decode(kv, q_r, W_UV, cos, sin, cfg, q_nope=q_n, W_UK=W_UK, seq_lens=seq, kv_offsets=offs,
                              max_seq_len=Lmax, seq_lens_host=my_lens if seq is not None else None, out=o,
                              workspace=ws, timer=t)
    tensors = dict(kv=kv, q_nope=q_nope, q_rope=q_rope, W_UK=W_UK, W_UV=W_UV, out=out, inp=inp,
                   close=sharded.close if spec["sharding"] == "kv-range" and world > 1 else None)
    return step, tensors, sum(my_lens) * CACHE_ROW_BYTES, B, my_lens


class Timed:
    """Device-timed replays of one step: a CUDA graph of the step without a kernel timer (the
    value), then one graph per step carrying the library's decode-kernel timer (the roofline).
    The graphs are released with release(), before any process-group teardown."""

    def __init__(self, step, steps, dev, eager):
        import torch
        from latent_attn import _lib
        self.step, self.steps, self.dev, self.eager = step, steps, dev, eager
        self.timers = [_lib.DecodeTimer() for _ in range(steps)]
        self.graphs, self.timed = [], []
        self.per_step_launches = None
        if not eager:
            side = torch.cuda.Stream(dev)
            n0 = _lib.kernel_launch_count()
            self.graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(self.graphs[0], stream=side):
                step()
            self.per_step_launches = _lib.kernel_launch_count() - n0
            for k in range(steps):
                self.graphs.append(torch.cuda.CUDAGraph())
                with torch.cuda.graph(self.graphs[-1], stream=side):
                    step(t=self.timers[k])
                self.timed.append(self.graphs[-1])
            for g in self.graphs[:4]:
                g.replay()
            torch.cuda.synchronize(dev)

    def run_plain(self, k):
        if self.eager:
            self.step()
        else:
            self.graphs[0].replay()

    def run_timed(self, k):
        if self.eager:
            self.step(t=self.timers[k])
        else:
            self.timed[k].replay()

    def decode_ms(self):
        return [t.decode_ms() for t in self.timers]

    def release(self):
        import torch
        self.timed.clear()
        for g in self.graphs:
            g.reset()
        self.graphs.clear()
        for t in self.timers:
            t.close()
        torch.cuda.synchronize(self.dev)


def run_leg(name, world, rank, dev, cfg, rope, ws, flush, barrier, steps, eager, peak):
    """One extra configuration: device-timed steps and the decode kernel's time, max over ranks."""
    import torch
    import torch.distributed as dist
    spec = workload_spec(name)
    step, tensors, nbytes, B, my_lens = build_step(spec, world, rank, dev, cfg, rope, ws, host_inputs=False)
    for _ in range(3):
        step()
    barrier()
    tm = Timed(step, steps, dev, eager)
    stream = torch.cuda.current_stream(dev)
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    for k in range(steps):
        flush.zero_()
        ev0[k].record(stream)
        tm.run_plain(k)
        ev1[k].record(stream)
    barrier()
    for k in range(steps):
        flush.zero_()
        tm.run_timed(k)
    barrier()
    dec = tm.decode_ms()
    tm.release()
    if tensors["close"] is not None:
        tensors["close"]()
    step_ms = sum(a.elapsed_time(b) for a, b in zip(ev0, ev1)) / steps
    dec_ms = statistics.mean(dec)
    frac_rank = nbytes / (dec_ms / 1e3) / 1e9 / peak
    t = torch.tensor([step_ms, dec_ms, nbytes], dtype=torch.float64, device=dev)
    fr = torch.tensor([frac_rank], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t[:2].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = t[2:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        dist.all_reduce(fr, op=dist.ReduceOp.MIN)
        t = torch.cat([mx, tot])
    step_ms, dec_ms, job_bytes = float(t[0]), float(t[1]), float(t[2])
    del tensors, step
    torch.cuda.empty_cache()
    return {"workload": spec["desc"], "us_per_step": round(step_ms * 1e3, 2),
            "GBps": round(job_bytes / (step_ms / 1e3) / 1e9, 1),
            "tokens_per_s": round(len(spec["lens"]) / (step_ms / 1e3), 1),
            "decode_kernel_us": round(dec_ms * 1e3, 2),
            "decode_frac": round(float(fr[0]), 4),
            "decode_frac_is": "min over ranks of (rank's cache bytes / its decode-kernel time) / measured HBM peak",
            "cache_bytes_per_step": int(job_bytes),
            "parallelism": config_of(spec, world)["parallelism"], "steps": steps}


def main(argv=None):
    json_out = json_stdout()
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world, json_out)
        return

    import torch
    import torch.distributed as dist
    from latent_attn import MLAConfig, _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    cfg = MLAConfig.deepseek_v2()
    spec = workload_spec(args.workload)
    lens_all = spec["lens"]
    ws = torch.empty(1 << 28, dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_src = measured_peaks()
    step, tens, bytes_per_step, B, my_lens = build_step(spec, world, rank, dev, cfg, args.rope, ws, host_inputs=True)
    inp, out = tens["inp"], tens["out"]

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
    status_word = ws[:4].view(torch.int32)
    status_sum = torch.zeros(1, dtype=torch.int32, device=dev)
    host_s = 0.0
    tm = Timed(step, args.steps, dev, args.eager)
    launches0 = _lib.kernel_launch_count()
    barrier()
    clocks.mark(True)
    for k in range(args.steps):
        flush.zero_()
        ev0[k].record(stream)
        h0 = time.perf_counter()
        tm.run_plain(k)
        host_s += time.perf_counter() - h0
        ev1[k].record(stream)
        status_sum.add_(status_word[:1].clamp(0, 1))
    barrier()
    clocks.mark(False)
    launches = _lib.kernel_launch_count() - launches0
    if tm.per_step_launches is not None:
        launches = int(round(tm.per_step_launches * args.steps))  # the graph's kernels, counted when captured
    for k in range(args.steps):
        flush.zero_()
        tm.run_timed(k)
        status_sum.add_(status_word[:1].clamp(0, 1))
    barrier()
    dec_ms = tm.decode_ms()
    tm.release()
    step_ms = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]
    status_errors = int(status_sum.item())
    total_ms = sum(step_ms)

    # ---- end-to-end: host buffers, the step's queries from pinned host memory and its output back to pinned
    # host memory inside the timed span. Two ways through the same public call, both timed:
    #   zero-copy (the value): the call is given the pinned host tensors, and the kernels read the queries and
    #     store the output over the host link themselves;
    #   memcpy: one cudaMemcpyAsync of the queries to device buffers, the call, one copy of the output back.
    # The step's queries live in one pinned host buffer (q_nope then q_rope).
    q_nope, q_rope = tens["q_nope"], tens["q_rope"]
    nqn, nqr = q_nope.numel(), q_rope.numel()
    q_h = torch.empty(nqn + nqr, dtype=torch.float32).pin_memory()
    q_h[:nqn].copy_(inp.q_nope.float().reshape(-1))
    q_h[nqn:].copy_(inp.q_rope.float().reshape(-1))
    qn_h, qr_h = q_h[:nqn].view(q_nope.shape), q_h[nqn:].view(q_rope.shape)
    out_h = torch.empty(B, 128, 128, dtype=torch.float32).pin_memory()
    q_d = torch.empty(nqn + nqr, dtype=torch.float32, device=dev)
    qn_d, qr_d = q_d[:nqn].view(q_nope.shape), q_d[nqn:].view(q_rope.shape)
    zero_copy = spec["sharding"] != "kv-range" or world == 1   # the KV-range decoder takes device queries
    e2e_ms, e2e_copy_ms = [], []
    barrier()
    for k in range(args.steps):
        flush.zero_()
        ev0[k].record(stream)
        if zero_copy:
            o = step(q_n=qn_h, q_r=qr_h, o=out_h)
        else:
            q_d.copy_(q_h, non_blocking=True)
            o = step(q_n=qn_d, q_r=qr_d)
            out_h.copy_(o, non_blocking=True)
        ev1[k].record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms.append(ev0[k].elapsed_time(ev1[k]))
    out_zero_copy = out_h.clone()
    barrier()
    for k in range(args.steps):
        flush.zero_()
        ev0[k].record(stream)
        q_d.copy_(q_h, non_blocking=True)
        o = step(q_n=qn_d, q_r=qr_d)
        out_h.copy_(o, non_blocking=True)
        ev1[k].record(stream)
        torch.cuda.synchronize(dev)
        e2e_copy_ms.append(ev0[k].elapsed_time(ev1[k]))
    barrier()
    clock_info = clocks.stop()
    h2d = nqn * 4 + nqr * 4
    d2h = out_h.numel() * 4
    e2e_total = sum(e2e_ms)
    e2e_copy_total = sum(e2e_copy_ms)
    e2e_outputs_match = bool(torch.equal(out_zero_copy, out_h))   # same kernels, same inputs: bit-identical

    # ---- max over ranks
    t = torch.tensor([total_ms, e2e_total, e2e_copy_total], dtype=torch.float64, device=dev)
    nbytes = torch.tensor([bytes_per_step], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(nbytes, op=dist.ReduceOp.SUM)
    total_max, e2e_max, e2e_copy_max = float(t[0]), float(t[1]), float(t[2])
    job_bytes = float(nbytes[0])
    value = job_bytes * args.steps / total_max / 1e6          # bytes / ms -> GB/s
    e2e_value = job_bytes * args.steps / e2e_max / 1e6
    e2e_copy_value = job_bytes * args.steps / e2e_copy_max / 1e6
    output_finite = bool(torch.isfinite(o).all())
    if tens["close"] is not None:
        tens["close"]()
    del step, tens, inp, out, o
    torch.cuda.empty_cache()

    # ---- the other configurations, same run
    legs = {}
    if not args.no_extra:
        names = ["cfg2", "cfg3", "cfg4"] if world == 1 else ["cfg3", "cfg4"]
        for name in names:
            if name == args.workload:
                continue
            legs[name] = run_leg(name, world, rank, dev, cfg, args.rope, ws, flush, barrier, args.extra_steps,
                                 args.eager, peak)

    if rank == 0:
        roof = None
        if dec_ms:
            dmean = statistics.mean(dec_ms)
            achieved = bytes_per_step / dmean / 1e6
            traffic = ncu_traffic(args.workload + ("" if args.rope == "otf" else "_tables"),
                                  sum(my_lens) / sum(lens_all))
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": traffic,
                    "kernel": "mla::decode_sm100_kernel", "kernel_us": round(dmean * 1e3, 3),
                    "algorithmic_bytes": bytes_per_step, "peak_source": peak_src + " -- fraction is of measured"}
            # the same kernel against the tensor pipe: per cache row 128 heads x 2 x (576 + 512) flop
            # (score over [c_t | k_rope], then P . c_t), 242 flop per byte
            tpeak, tsrc = measured_tensor_peak()
            flops = bytes_per_step // CACHE_ROW_BYTES * 128 * 2 * (576 + 512)
            tflops = flops / dmean / 1e9
            roof["tensor"] = {"achieved": round(tflops, 1), "peak": tpeak, "unit": "TFLOP/s",
                              "frac": round(tflops / tpeak, 4), "flops": flops,
                              "peak_source": tsrc + " -- fraction is of measured"}
        cpu = cfg0 = None
        if world == 1 and not args.no_cpu_baseline:
            gbs, cores, sample = cpu_oracle_rate(lens_all, args.cpu_seconds)
            cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                   "sample": sample + f"; CPU: {cpu_model()}", "cpu_model": cpu_model()}
            cfg0 = cpu_config0()
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
            "config": config_of(spec, world),
            "roofline": roof,
            "cpu_baseline": cpu,
            "cpu_config0": cfg0,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_max / args.steps, 5),
                    "api": ("latent_attn.functional.mla_decode given pinned host q_nope/q_rope and a pinned host "
                            "output: the kernels read the queries and store the output over the host link "
                            "(zero-copy), no copy launches" if zero_copy else
                            "KVRangeDecoder with q_nope/q_rope copied from pinned host memory and the output "
                            "copied back (cudaMemcpyAsync)"),
                    "memcpy": {"value": round(e2e_copy_value, 2), "ms_per_step": round(e2e_copy_max / args.steps, 5),
                               "api": "the same call on device tensors, one cudaMemcpyAsync of the queries in "
                                      "and one of the output out per step"},
                    "outputs_match": e2e_outputs_match},
            "gpu_launches": int(launches),
            "launch": "cuda-graph replay per step" if not args.eager else "direct",
            "host_us_per_step_call": round(host_s / args.steps * 1e6, 1),
            "decode_status_errors": status_errors,
            "output_finite": output_finite,
            "rope": ("on the fly: the kernels compute cos/sin, no table is read" if args.rope == "otf"
                     else "the reference's fp32 cos/sin tables"),
            "workloads": legs,
            "clocks": clock_info,
        }
        print(json.dumps(line), file=json_out, flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
