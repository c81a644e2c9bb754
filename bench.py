#!/usr/bin/env python3
"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload auto|c2|c2q4|c5]

Workloads (seeded synthetic tensors, random data of the
stated distributions -- no datasets are involved):
  c2   config 2: one decode step, 16 Q / 2 KV heads, D=256, kv 32768, Q8_0 KV
       (the N=1 headline).  Eight rotated input sets (286 MB > 2 x L2) so every
       step streams its KV from HBM.
  c2q4 the same with Q4_0 KV.
  c5   config 5: 8 sequences x 262144 KV rows, 24 Q / 4 KV heads, D=256, Q8_0;
       the KV rows are cut into 256 fixed global splits, each GPU holds and
       reads its contiguous block of splits, the (m, l, O) partials are
       all-gathered over NCCL and merged in split order (bit-identical for any
       GPU count).  Default for N > 1 ("strong" scaling: total work fixed).
A step = the attention kernels of one decode step over that workload.
`value` is KV GB/s (algorithmic bytes: K + V + q + out per step) with inputs
resident; `e2e` is the same metric through the public call xq.flash_attn_ext
with q copied host->device (pinned) and the output read back every step.
--impl reference times the reference's CPU algorithm (the ggml-cpu
restatement in oracle/, all host threads) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "xllama-qwen35-xbox_b200"))
sys.path.insert(0, REPO)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return FALLBACK_HBM_GBS, 1590.0, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md
    (line 'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(REPO, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.samples, self.proc = index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if not self.samples:
            return None
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if s[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workloads

C2 = dict(n_head=16, n_hkv=2, D=256, n_kv=32768, n_seq=1)
C5 = dict(n_head=24, n_hkv=4, D=256, n_kv=262144, n_seq=8)


def algo_bytes(w, ty):
    import xq
    kv = 2 * w["n_seq"] * w["n_kv"] * w["n_hkv"] * xq.row_bytes(ty, w["D"])
    qo = 2 * w["n_seq"] * w["n_head"] * w["D"] * 4
    return kv, kv + qo


def make_kv(torch, xq, w, ty, n_rows, seed, dev):
    """Quantized KV rows (n_seq, n_rows, n_hkv, row_bytes) from N(0,1), built
    on the device in chunks with the ggml reference quantizer."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rb = xq.row_bytes(ty, w["D"])
    out = torch.empty((w["n_seq"], n_rows, w["n_hkv"], rb), dtype=torch.uint8, device=dev)
    chunk = 1 << 22  # float32 elements per chunk
    rows_per = max(1, chunk // (w["n_hkv"] * w["D"]))
    for s in range(w["n_seq"]):
        for r0 in range(0, n_rows, rows_per):
            r1 = min(n_rows, r0 + rows_per)
            x = torch.randn((r1 - r0, w["n_hkv"], w["D"]), generator=g, device=dev)
            out[s, r0:r1] = xq.quantize_rows(ty, x)
    return out


def run_ours(args, rank, world, torch, dist):
    import xq
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    workload = args.workload
    if workload == "auto":
        workload = "c2" if world == 1 else "c5"
    ty = xq.Q4_0 if workload == "c2q4" else xq.Q8_0
    w = C5 if workload == "c5" else C2
    hbm, _, peak_kind = peaks()
    st = torch.cuda.current_stream()
    D, H, Hkv, n_seq = w["D"], w["n_head"], w["n_hkv"], w["n_seq"]
    kv_bytes, step_bytes = algo_bytes(w, ty)
    n_rows_out = n_seq * H

    if workload == "c5":
        rows_per_split, n_splits = 1024, w["n_kv"] // 1024
        per = n_splits // world
        sb, se = rank * per, (rank + 1) * per
        local_rows = (se - sb) * rows_per_split
        # each GPU holds only its block of KV rows; global row r = sb*1024 + local r
        k = make_kv(torch, xq, w, ty, local_rows, 1000 + rank, dev)
        v = make_kv(torch, xq, w, ty, local_rows, 2000 + rank, dev)
        sets = [(k, v)]
        local_split_rows = rows_per_split
    else:
        n_sets = max(4, math.ceil(2 * L2_BYTES / kv_bytes) + 1)
        sets = [(make_kv(torch, xq, w, ty, w["n_kv"], 10 + 2 * i, dev),
                 make_kv(torch, xq, w, ty, w["n_kv"], 11 + 2 * i, dev)) for i in range(n_sets)]
        rows_per_split = None
    gq = torch.Generator(device=dev)
    gq.manual_seed(7)
    qs = [torch.randn((n_seq, H, 1, D), generator=gq, device=dev) for _ in sets]
    scale = 1.0 / math.sqrt(D)

    # plan: automatic split count for the single-GPU decode
    if workload != "c5":
        sm = torch.cuda.get_device_properties(dev).multi_processor_count
        n_splits = max(1, min(math.ceil(2 * sm / (Hkv * n_seq)), math.ceil(w["n_kv"] / 64)))
        rows_per_split = math.ceil(w["n_kv"] / n_splits)
        n_splits = math.ceil(w["n_kv"] / rows_per_split)
        sb, se = 0, n_splits
    part_local = torch.empty((se - sb, n_rows_out, D + 2), dtype=torch.float32, device=dev)
    part_all = torch.empty((n_splits, n_rows_out, D + 2), dtype=torch.float32, device=dev)
    out = torch.empty((n_rows_out, D), dtype=torch.float32, device=dev)

    def step(i, parts=("dec", "gather", "merge")):
        k, v = sets[i % len(sets)]
        q = qs[i % len(sets)]
        if "dec" in parts:
            xq.fa_partials(q, k, v, ty, rows_per_split, 0 if workload == "c5" else sb,
                           (se - sb) if workload == "c5" else se, scale=scale, out=part_local)
        src = part_local
        if world > 1:
            if "gather" in parts:
                dist.all_gather_into_tensor(part_all, part_local)
            src = part_all
        if "merge" in parts:
            xq.lse_merge(src, out=out, want_lse=False)

    use_graph = os.environ.get("XQ_BENCH_NO_GRAPH", "0") != "1"

    def timed(fn, n):
        """Device time (ms) of n calls of fn, replayed from one CUDA graph so
        host launch overhead stays out of the timed region; max over ranks."""
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        g = None
        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(n):
                    fn(i)
            g.replay()  # warm replay
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        if g is not None:
            g.replay()
        else:
            for i in range(n):
                fn(i)
        e1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t = e0.elapsed_time(e1)
        del g
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    clk = ClockSampler(dev.index)
    clk.start()
    ms = timed(step, args.steps) / args.steps
    clocks = clk.stop()
    dec_ms = timed(lambda i: step(i, ("dec",)), args.steps) / args.steps
    mrg_ms = timed(lambda i: step(i, ("merge",)), args.steps) / args.steps
    col_ms = (timed(lambda i: step(i, ("gather",)), args.steps) / args.steps) if world > 1 else 0.0

    # end to end through the public call with host buffers (pinned)
    q_host = torch.empty((n_seq, H, 1, D), dtype=torch.float32, pin_memory=True)
    q_host.copy_(qs[0].cpu())
    o_host = torch.empty((n_seq, 1, H, D), dtype=torch.float32, pin_memory=True)
    q_dev = torch.empty_like(qs[0])
    if workload != "c5":
        o_dev = torch.empty((n_seq, 1, H, D), dtype=torch.float32, device=dev)

        def e2e_step(i):
            k, v = sets[i % len(sets)]
            q_dev.copy_(q_host, non_blocking=True)
            xq.flash_attn_ext(q_dev, k, v, ty, scale=scale, n_splits=n_splits, out=o_dev)
            o_host.copy_(o_dev, non_blocking=True)
    else:
        def e2e_step(i):
            q_dev.copy_(q_host, non_blocking=True)
            qs[0].copy_(q_dev)
            step(0)
            o_host.view(-1).copy_(out.view(-1), non_blocking=True)
    e2e_ms = timed(e2e_step, args.steps) / args.steps

    if rank != 0:
        return None
    value = step_bytes / (ms * 1e-3) / 1e9
    local_kv = kv_bytes / world
    achieved = (local_kv + (step_bytes - kv_bytes) / 2) / (dec_ms * 1e-3) / 1e9
    kname = f"fa_decode_{workload}"
    traffic = profile_traffic(kname)
    line = {
        "metric": "flash-decode KV GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if workload == "c5" else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), ggml reference quantizer)",
        "config": {"workload": {"c2": "BASELINE config 2 (Q8_0 decode, kv 32768)",
                                "c2q4": "BASELINE config 2, Q4_0 variant",
                                "c5": "BASELINE config 5 (8 x 262144 Q8_0, KV-sharded)"}[workload],
                   "kv_type": "q8_0" if ty == xq.Q8_0 else "q4_0",
                   "n_seq": n_seq, "n_head": H, "n_head_kv": Hkv, "head_dim": D,
                   "kv_len": w["n_kv"], "kv_splits": n_splits, "rows_per_split": rows_per_split,
                   "parallelism": f"kv-shard{world}" if world > 1 else "single",
                   "l2": ("rotating %d input sets (%.0f MB > 2x L2)" % (len(sets),
                          len(sets) * kv_bytes / 1e6)) if workload != "c5" else
                         "inputs %.0f MB per GPU > L2" % (local_kv / 1e6)},
        "breakdown_ms": {"decode_kernel": round(dec_ms, 5), "nccl_gather": round(col_ms, 5),
                         "merge_kernel": round(mrg_ms, 5)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_kind": peak_kind,
                     "kernel": ("fa_decode_kernel" if os.environ.get("XQ_DECODE_MMA") == "0"
                                else "fa_decode_mma_kernel"),
                     "traffic": traffic},
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": int(q_host.numel() * 4),
                "d2h_bytes_per_step": int(o_host.numel() * 4)},
        "gpu_launches": args.steps * 2,
        "timing": "CUDA-graph replay of %d steps, CUDA events" % args.steps if use_graph
                  else "eager launches, CUDA events",
        "clocks": clocks,
    }
    return line


def cpu_oracle_sample(workload, seconds_cap=20.0, sample_kv=None):
    """Time the CPU restatement of ggml-cpu FLASH_ATTN_EXT on a bounded sample
    of the workload (all host threads); returns (GB/s, info)."""
    import oracle
    w = C5 if workload == "c5" else C2
    ty = oracle.Q4_0 if workload == "c2q4" else oracle.Q8_0
    n_kv = sample_kv or w["n_kv"]
    n_seq = 1
    rng = np.random.default_rng(0)
    q = rng.normal(0, 1, (n_seq, w["n_head"], 1, w["D"])).astype(np.float32)
    kf = rng.normal(0, 1, (n_seq, n_kv, w["n_hkv"], w["D"])).astype(np.float32)
    k = oracle.quantize(ty, kf)
    v = oracle.quantize(ty, rng.normal(0, 1, kf.shape).astype(np.float32))
    del kf
    cores = os.cpu_count() or 1
    oracle.flash_attn_ext(q, k, v, ty, ty, scale=1 / 16, nth=cores, n_workers=cores)  # warm
    t = time.perf_counter()
    reps = 0
    while True:
        oracle.flash_attn_ext(q, k, v, ty, ty, scale=1 / 16, nth=cores, n_workers=cores)
        reps += 1
        if time.perf_counter() - t > min(seconds_cap, 3.0) or reps >= 5:
            break
    dt = (time.perf_counter() - t) / reps
    b = k.nbytes + v.nbytes + 2 * q.nbytes
    return b / dt / 1e9, {"cores": cores, "sample": f"1 sequence x {n_kv} rows, {reps} reps, "
                          f"{dt * 1e3:.1f} ms each, {cores} threads"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="auto", choices=["auto", "c2", "c2q4", "c5"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    workload = args.workload if args.workload != "auto" else ("c2" if world == 1 else "c5")

    if args.impl == "reference":
        if rank != 0:
            return 0
        val, info = cpu_oracle_sample(workload)
        line = {"metric": "flash-decode KV GB/s", "value": round(val, 3), "unit": "GB/s",
                "impl": "reference", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
                "config": {"workload": workload}, "data": "synthetic",
                "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": info["cores"],
                                 "kind": "port", "sample": info["sample"]},
                "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    line = run_ours(args, rank, world, torch, dist)
    if rank == 0 and line is not None:
        if world == 1 and not args.no_cpu_baseline:
            val, info = cpu_oracle_sample(workload)
            line["cpu_baseline"] = {"value": round(val, 3), "unit": "GB/s",
                                    "cores": info["cores"], "kind": "port",
                                    "sample": info["sample"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
