#!/usr/bin/env python3
"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload auto|c1|c2|c2q4|c2mtp|c3a|c3b|c4|c4q8|c4q4|c5|kvw|kv4]

Workloads (seeded synthetic tensors, random data of the
stated distributions -- no datasets are involved):
  c2   config 2: one decode step, 16 Q / 2 KV heads, D=256, kv 32768, Q8_0 KV
       (the N=1 headline).  Eight rotated input sets (286 MB > 2 x L2) so every
       step streams its KV from HBM.
  c2q4 the same with Q4_0 KV.
  c2mtp multi-token-prediction verify over the config-2 cache: 4 query tokens
       (3 draft tokens + 1) per step, causal among themselves through an F16
       mask over their last 4 cache rows (the reference's nq 2..9 multi-query
       tiles), the same rotated input sets.
  c1   config 1: one decode step, F16 KV, 16 Q / 4 KV heads, D=128, kv 4096
       (31 rotated input sets > 2 x L2).
  c3a  config 3 decode: GATED_DELTA_NET, 8 sequences x 1 token, 32 v-heads /
       16 k-heads, d 128 (fp32 state read + written; 9 rotated sets).
  c3b  config 3 prefill: GATED_DELTA_NET, 1 sequence x 4096 tokens.
       With N > 1 both shard the op by value head (each GPU its block of the
       32 heads, whole q/k, no exchange step; strong scaling) and the line
       carries `scaling_reference`, the unsharded op on rank 0's GPU.
  c4   config 4: causal prefill, 8192 tokens, 24 Q / 4 KV heads, D=256, F16
       K/V, explicit causal F16 mask (tensor-core kernel); metric TFLOP/s.
  c4q8 / c4q4  the config-4 shape over a Q8_0 / Q4_0 cache (the reference's
       product configuration): K/V widened to f16 by the library's pre-pass
       inside every step, q quantized to Q8_0 as ggml-cpu does.
       With N > 1 the prefill rows shard by KV-head group (up to 4 GPUs take
       one KV head group each; at 8, each KV head's query rows are cut in two
       blocks of equal causal work), strong scaling, with `scaling_reference`.
  kvw  KV-cache write (GGML_OP_SET_ROWS, the row after the hot path): a
       prefill batch of 8192 tokens x 4 KV heads x D=256, K and V, quantized
       to Q8_0 into 32768-row caches (4 rotated input sets > 2 x L2).
  kv4  native KVarN4 range attention (the RKVA server's resident image):
       24 Q / 4 KV heads, D=256, 32768 rows past origin 102400 in 4-bit
       records plus the 128-row F16 precision tail, one query (9 rotated
       plane sets > 2 x L2).
  c5   config 5: 8 sequences x 262144 KV rows, 24 Q / 4 KV heads, D=256, Q8_0;
       the KV rows are cut into 256 fixed global splits in 8 fixed groups; each
       GPU holds and reads its contiguous block of groups, merges each group
       into one (O, lse) record, the group records are all-gathered over NCCL
       and merged in group order (bit-identical for any GPU count dividing 8).
       Default for N > 1 ("strong" scaling: total work fixed); those lines
       also carry `scaling_reference`, config 5 timed on one GPU in the same
       run (the N = 1 point of the series), with `bit_identical_to_n_gpus`:
       the KV rows are generated per global group, so the one-GPU output and
       the N-GPU output are compared bit for bit.
A step = the attention kernels of one decode step over that workload.
`value` is KV GB/s (algorithmic bytes: K + V + q + out per step) with inputs
resident; `e2e` is the same metric through the public call xq.flash_attn_ext
with q and the output in pinned host memory (q copied to the GPU by the
library's staging kernel, the result written back over PCIe) every step,
replayed from a CUDA graph; `e2e_eager` makes the same calls eagerly, one
prebuilt C-ABI call per step, so the library's per-call host work (as the
ggml backend's graph_compute pays it) is inside the timed region.
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

C1 = dict(n_head=16, n_hkv=4, D=128, n_kv=4096, n_seq=1)
C2 = dict(n_head=16, n_hkv=2, D=256, n_kv=32768, n_seq=1)
C2MTP = dict(C2, n_q=4)
C3 = dict(S=128, H=32, H_k=16, slots=1)
C4 = dict(n_head=24, n_hkv=4, D=256, n_q=8192)
TYPE_NAMES = {0: "f32", 1: "f16", 2: "q4_0", 8: "q8_0"}
C5 = dict(n_head=24, n_hkv=4, D=256, n_kv=262144, n_seq=8)
WORKLOAD_NAMES = {
    "c1": "BASELINE config 1 (F16 decode, kv 4096)",
    "c2": "BASELINE config 2 (Q8_0 decode, kv 32768)",
    "c2q4": "BASELINE config 2, Q4_0 variant",
    "c2mtp": "BASELINE config 2 cache, 4-token MTP verify (causal mask over the new rows)",
    "c5": "BASELINE config 5 (8 x 262144 Q8_0, KV-sharded)",
    "c3a": "BASELINE config 3 decode (GDN, 8 seqs x 1 token)",
    "c3b": "BASELINE config 3 prefill (GDN, 1 seq x 4096 tokens)",
    "c4": "BASELINE config 4 (causal prefill, 8192 tokens, F16 KV)",
    "c4q8": "BASELINE config 4 shape over a Q8_0 KV cache (causal prefill, 8192 tokens)",
    "c4q4": "BASELINE config 4 shape over a Q4_0 KV cache (causal prefill, 8192 tokens)",
    "kvw": "KV-cache write (SET_ROWS), 8192 tokens x 4 KV heads x D=256, K and V to Q8_0",
    "kv4": "native KVarN4 range attention, 24 Q / 4 KV heads, D=256, 32768 rows past origin "
           "102400, precision tail 128, 1 query",
}


def algo_bytes(w, ty):
    """(K + V bytes, all bytes of a step: K, V, q, out and the F16 mask of a
    multi-query step)."""
    import xq
    n_q = w.get("n_q", 1)
    kv = 2 * w["n_seq"] * w["n_kv"] * w["n_hkv"] * xq.row_bytes(ty, w["D"])
    qo = 2 * w["n_seq"] * n_q * w["n_head"] * w["D"] * 4
    mask = w["n_kv"] * n_q * 2 if n_q > 1 else 0
    return kv, kv + qo + mask


def mtp_mask(torch, w, dev):
    """F16 mask [1, 1, n_q, n_kv] of an MTP verify step: query i sees the cache
    and the new rows up to its own (the last n_q rows are the new tokens)."""
    n_q, n_kv = w["n_q"], w["n_kv"]
    m = torch.zeros((1, 1, n_q, n_kv), dtype=torch.float16, device=dev)
    for i in range(n_q):
        m[0, 0, i, n_kv - n_q + i + 1:] = float("-inf")
    return m


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


def graph_timed(torch, fn, n, warmup, world=1, dist=None, dev=None, use_graph=True):
    """Device time (ms) of n calls of fn, replayed from one CUDA graph so host
    launch overhead stays out of the timed region; max over ranks."""
    for i in range(warmup):
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


def workload_config(workload, world=1):
    """The `config` object of a JSON line: static facts of the workload (no
    device query), the same in the repo arm and the reference arm."""
    def l2_sets(step_bytes):
        return max(4, math.ceil(2 * L2_BYTES / step_bytes) + 1)
    if workload in ("c1", "c2", "c2q4", "c2mtp", "c5"):
        w = {"c5": C5, "c1": C1, "c2mtp": C2MTP}.get(workload, C2)
        ty = {"c2q4": 2, "c1": 1}.get(workload, 8)
        kv, _ = algo_bytes(w, ty)
        cfg = {"workload": WORKLOAD_NAMES[workload], "kv_type": TYPE_NAMES[ty],
               "n_seq": w["n_seq"], "n_head": w["n_head"], "n_head_kv": w["n_hkv"],
               "head_dim": w["D"], "kv_len": w["n_kv"],
               **({"n_q": w["n_q"], "mask": "F16 causal over the new rows"}
                  if w.get("n_q", 1) > 1 else {}),
               "parallelism": f"kv-shard{world}" if world > 1 else "single"}
        if workload == "c5":
            cfg["l2"] = "inputs %.0f MB per GPU > L2" % (kv / world / 1e6)
        else:
            n = l2_sets(kv)
            cfg["l2"] = "rotating %d input sets (%.0f MB > 2x L2)" % (n, n * kv / 1e6)
        return cfg
    if workload in ("c3a", "c3b"):
        n_seq, T = (8, 1) if workload == "c3a" else (1, 4096)
        b = gdn_bytes(n_seq, T)[0]
        n = 1 if b > 2 * L2_BYTES else math.ceil(2 * L2_BYTES / b) + 1
        return {"workload": WORKLOAD_NAMES[workload], "n_seq": n_seq, "tokens": T,
                "v_heads": C3["H"], "k_heads": C3["H_k"], "head_dim": C3["S"],
                "slots": C3["slots"],
                "parallelism": f"value-head-shard{world}" if world > 1 else "single",
                "l2": ("rotating %d input sets (%.0f MB > 2x L2)" % (n, n * b / 1e6)) if n > 1
                      else "inputs %.0f MB > L2" % (b / 1e6)}
    if workload in ("c4", "c4q8", "c4q4"):
        w = C4
        ty = {"c4q8": 8, "c4q4": 2}.get(workload, 1)
        N, H, Hkv, D = w["n_q"], w["n_head"], w["n_hkv"], w["D"]
        kv = 2 * N * Hkv * {1: 2 * D, 8: D // 32 * 34, 2: D // 32 * 18}[ty]
        return {"workload": WORKLOAD_NAMES[workload], "kv_type": TYPE_NAMES[ty], "n_q": N,
                "n_kv": N, "n_head": H, "n_head_kv": Hkv, "head_dim": D, "mask": "causal F16",
                "flops_per_step": prefill_flops(N, H, D),
                "parallelism": f"kv-head-group-shard{world}" if world > 1 else "single",
                "l2": "inputs %.0f MB > L2" % ((N * H * D * 4 + kv + N * N * 2) / 1e6)}
    if workload == "kvw":
        n = 4
        return {"workload": WORKLOAD_NAMES[workload], "cache_rows": KVW["rows"],
                "l2": "rotating %d input sets (%.0f MB > 2x L2)" % (
                    n, n * 2 * KVW["n_tok"] * KVW["n_hkv"] * KVW["D"] * 4 / 1e6)}
    b = kvarn4_bytes()
    n = max(4, math.ceil(2 * L2_BYTES / b) + 1)
    return {"workload": WORKLOAD_NAMES[workload], "bytes_per_step": b,
            "l2": "rotating %d plane sets (%.0f MB > 2x L2)" % (n, n * b / 1e6)}


def eager_timed(torch, fn, n, warmup):
    """Device time (ms) of n eager calls of fn (no graph: every call's host
    work -- argument checks, planning, tensor-map encoding, launches -- sits
    between the kernels, as it does for the ggml backend's graph_compute)."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(n):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def fa_eager_call(torch, q, k, v, ty, scale, n_splits, out, mask=None):
    """One prebuilt C-ABI call of xq_flash_attn_ext (the argument struct and
    the workspace are built once, as a C caller keeps them), returned as a
    zero-argument function: the eager e2e then times the library's own host
    work plus one ctypes transition per step."""
    import ctypes as C

    import xq
    from xq import _lib
    from xq.ops import _fa_params, _stream, _workspace
    p = _fa_params(q, k, v, ty, ty, mask, None, out, scale, 0.0, 0.0, n_splits)
    L = _lib.lib()
    nbytes = L.xq_flash_attn_ext_workspace(C.byref(p))
    ws = _workspace(nbytes, torch.device("cuda", torch.cuda.current_device()))
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    fn, ref, st = L.xq_flash_attn_ext, C.byref(p), _stream(None)
    keep = (p, ws, q, out, mask)

    def call():
        rc = fn(ref, wsp, wsn, st)
        if rc:
            xq._lib.check(rc)
        return keep
    return call


def make_kv_groups(torch, xq, w, ty, g0, g1, rows_per_group, seed_base, dev):
    """KV rows of global groups [g0, g1), each group generated from its own
    seed (seed_base + g): the same rows whichever GPU holds them."""
    rb = xq.row_bytes(ty, w["D"])
    out = torch.empty((w["n_seq"], (g1 - g0) * rows_per_group, w["n_hkv"], rb),
                      dtype=torch.uint8, device=dev)
    for g in range(g0, g1):
        lo = (g - g0) * rows_per_group
        out[:, lo:lo + rows_per_group] = make_kv(torch, xq, w, ty, rows_per_group,
                                                 seed_base + g, dev)
    return out


def run_decode(args, rank, world, torch, dist, workload):
    import xq
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    ty = {"c2q4": xq.Q4_0, "c1": xq.F16}.get(workload, xq.Q8_0)
    w = {"c5": C5, "c1": C1, "c2mtp": C2MTP}.get(workload, C2)
    hbm, _, peak_kind = peaks()
    D, H, Hkv, n_seq = w["D"], w["n_head"], w["n_hkv"], w["n_seq"]
    n_q = w.get("n_q", 1)
    kv_bytes, step_bytes = algo_bytes(w, ty)
    n_rows_out = n_seq * n_q * H
    mask = mtp_mask(torch, w, dev) if n_q > 1 else None

    if workload == "c5":
        from xq import shard
        rows_per_split, n_splits, n_groups = 1024, w["n_kv"] // 1024, 8
        per_group = n_splits // n_groups
        gb, ge = shard.split_block(n_groups, world, rank)
        sb, se = gb * per_group, ge * per_group
        # each GPU holds only its groups' rows, generated per group (seeded by
        # global group), so any GPU count sees the same KV cache
        rpg = per_group * rows_per_split
        k = make_kv_groups(torch, xq, w, ty, gb, ge, rpg, 1000, dev)
        v = make_kv_groups(torch, xq, w, ty, gb, ge, rpg, 2000, dev)
        sets = [(k, v)]
    else:
        n_sets = max(4, math.ceil(2 * L2_BYTES / kv_bytes) + 1)
        sets = [(make_kv(torch, xq, w, ty, w["n_kv"], 10 + 2 * i, dev),
                 make_kv(torch, xq, w, ty, w["n_kv"], 11 + 2 * i, dev)) for i in range(n_sets)]
    gq = torch.Generator(device=dev)
    gq.manual_seed(7)
    qs = [torch.randn((n_seq, H, n_q, D), generator=gq, device=dev) for _ in sets]
    scale = 1.0 / math.sqrt(D)

    if workload != "c5":
        # the library's automatic plan (every CTA slot of the decode variant
        # filled in one wave, whole 64-row rounds per split)
        _, n_splits, rows_per_split = xq.flash_attn_ext_plan(qs[0], sets[0][0], sets[0][1], ty,
                                                             mask=mask)
        sb, se = 0, n_splits
    part_local = torch.empty((se - sb, n_rows_out, D + 2), dtype=torch.float32, device=dev)
    if workload == "c5":
        rec_local = torch.empty((ge - gb, n_rows_out, D + 2), dtype=torch.float32, device=dev)
        rec_all = torch.empty((n_groups, n_rows_out, D + 2), dtype=torch.float32, device=dev)
    out = torch.empty((n_rows_out, D), dtype=torch.float32, device=dev)

    out4 = out.view(n_seq, n_q, H, D)

    def step(i, parts=("dec", "gather", "merge")):
        k, v = sets[i % len(sets)]
        q = qs[i % len(sets)]
        if workload != "c5" and parts == ("dec", "gather", "merge"):
            # the public call (device buffers): the split-KV decode kernel and
            # the merge kernel, as xq_flash_attn_ext launches them
            xq.flash_attn_ext(q, k, v, ty, mask=mask, scale=scale, n_splits=n_splits, out=out4)
            return
        if "dec" in parts:
            xq.fa_partials(q, k, v, ty, rows_per_split, 0 if workload == "c5" else sb,
                           (se - sb) if workload == "c5" else se, mask=mask, scale=scale,
                           out=part_local)
        src = part_local
        if workload == "c5":
            if "merge" in parts:
                xq.lse_merge_records(part_local, per_group, out=rec_local)
            src = rec_local
            if world > 1:
                if "gather" in parts:
                    shard.gather_partials(rec_local, n_groups, out=rec_all)
                src = rec_all
        if "merge" in parts:
            xq.lse_merge(src, out=out, want_lse=False)

    def timed(fn, n):
        return graph_timed(torch, fn, n, args.warmup, world, dist, dev)

    ex, nccl_ms = None, None
    if workload == "c5" and world > 1:
        # the sharded step through the C ABI: group records stored into every
        # rank's exchange buffer over NVLink (xq_fa_shard_push / _finish);
        # step numbers rise by one per call on every rank, and the captured
        # sequences hold an even number of steps (the exchange halves alternate)
        ex = shard.ShardExchange(n_groups, n_rows_out, D)
        p2p_ws = torch.empty(max(1 << 20, 2 * part_local.numel() * 4), dtype=torch.uint8,
                             device=dev)
        step_no = [0]
        dist.barrier()
        torch.cuda.synchronize()
        nccl_step = step

        def step(i, parts=None):
            k, v = sets[0]
            shard.shard_decode_step(qs[0], k, v, ty, ex, rank, world, rows_per_split, per_group,
                                    step_no[0], scale=scale, out=out, ws=p2p_ws)
            step_no[0] += 1
        args.steps += args.steps % 2
        nccl_ms = timed(nccl_step, args.steps) / args.steps

    clk = ClockSampler(dev.index)
    clk.start()
    ms = timed(step, args.steps) / args.steps
    clocks = clk.stop()
    # breakdown: each kernel of the step graph-timed alone
    parts_step = nccl_step if ex is not None else step
    dec_ms = timed(lambda i: parts_step(i, ("dec",)), args.steps) / args.steps
    mrg_ms = timed(lambda i: parts_step(i, ("merge",)), args.steps) / args.steps
    col_ms = (timed(lambda i: parts_step(i, ("gather",)), args.steps) / args.steps
              if world > 1 else 0.0)

    # end to end through the public call with host buffers (pinned)
    q_host = torch.empty((n_seq, H, n_q, D), dtype=torch.float32, pin_memory=True)
    q_host.copy_(qs[0].cpu())
    o_host = torch.empty((n_seq, n_q, H, D), dtype=torch.float32, pin_memory=True)
    q_dev = torch.empty_like(qs[0])
    eager_ms = None
    if workload != "c5":

        def e2e_step(i):
            # q and the output stay in pinned host memory: the library copies q
            # to the GPU with its staging kernel and writes the result back over
            # PCIe every step
            k, v = sets[i % len(sets)]
            xq.flash_attn_ext(q_host, k, v, ty, mask=mask, scale=scale, n_splits=n_splits,
                              out=o_host)
        calls = [fa_eager_call(torch, q_host, k_, v_, ty, scale, n_splits, o_host, mask)
                 for k_, v_ in sets]
        eager_ms = eager_timed(torch, lambda i: calls[i % len(calls)](), args.steps,
                               args.warmup) / args.steps
    else:
        def e2e_step(i):
            q_dev.copy_(q_host, non_blocking=True)
            qs[0].copy_(q_dev)
            step(0)
            o_host.view(-1).copy_(out.view(-1), non_blocking=True)
    e2e_ms = timed(e2e_step, args.steps) / args.steps

    # the N = 1 point of the config-5 series, measured in the same run (the
    # default N = 1 line is config 2), and the bit-identity of the N-GPU output
    ref1 = None
    if workload == "c5" and world > 1:
        step(0)
        step(0)
        torch.cuda.synchronize()
        dist.barrier()
        ex.close()
        if rank == 0:
            ref1, out1 = c5_single_gpu(torch, xq, dev, ty, args.steps, args.warmup, step_bytes)
            ref1["bit_identical_to_n_gpus"] = bool(torch.equal(out1, out))
            del out1
        dist.barrier()
    if rank != 0:
        return None
    value = step_bytes / (ms * 1e-3) / 1e9
    local_kv = kv_bytes / world
    # dominant kernel: the split-KV decode (this GPU's splits under sharding)
    achieved = (local_kv + (step_bytes - kv_bytes) / 2) / (dec_ms * 1e-3) / 1e9
    traffic = profile_traffic(f"fa_decode_{workload}")
    line = {
        "metric": "flash-decode KV GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if workload == "c5" else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), ggml reference quantizer)",
        "config": workload_config(workload, world),
        "plan": {"kv_splits": n_splits, "rows_per_split": rows_per_split,
                 **({"split_groups": n_groups, "groups_per_gpu": ge - gb}
                    if workload == "c5" else {})},
        "breakdown_ms": {"decode_kernel": round(dec_ms, 5), "nccl_gather": round(col_ms, 5),
                         "merge_kernel" + ("s" if workload == "c5" else ""): round(mrg_ms, 5)},
        **({"exchange": "group records stored into every rank's exchange buffer with NVLink "
                        "peer stores (xq_fa_shard_push / xq_fa_shard_finish)",
            "nccl_exchange_step_ms": round(nccl_ms, 5)} if ex is not None else {}),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_kind": peak_kind,
                     "kernel": ("fa_decode_kernel" if os.environ.get("XQ_DECODE_MMA") == "0"
                                else "fa_decode_mma_kernel"),
                     "traffic": traffic},
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": int(q_host.numel() * 4),
                "d2h_bytes_per_step": int(o_host.numel() * 4),
                "timing": "CUDA-graph replay (host launch work outside the timed region)"},
        **({"e2e_eager": {"value": round(step_bytes / (eager_ms * 1e-3) / 1e9, 2),
                          "unit": "GB/s", "ms_per_step": round(eager_ms, 5),
                          "timing": "eager: one prebuilt xq_flash_attn_ext call per step "
                                    "from a Python loop (the library's host work and one "
                                    "ctypes transition per step inside the timed region)"}}
           if eager_ms is not None else {}),
        # decode + merge per step; c5 over N GPUs: decode, group records, push,
        # wait, final merge; e2e adds the q staging kernel
        "gpu_launches": args.steps * ((5 if world > 1 else 3) if workload == "c5" else 2),
        **({"scaling_reference": ref1} if ref1 else {}),
        "timing": "CUDA-graph replay of %d steps, CUDA events" % args.steps,
        "clocks": clocks,
    }
    return line


def c5_single_gpu(torch, xq, dev, ty, steps, warmup, step_bytes):
    """Config 5 on one GPU (all 256 splits, the 8 group merges, the final
    merge; no collective): the N = 1 point of the KV-sharded series.  Returns
    (line fragment, merged output of the last step)."""
    w = C5
    n_splits, rows_per_split, per_group = w["n_kv"] // 1024, 1024, 32
    n_groups = n_splits // per_group
    k = make_kv_groups(torch, xq, w, ty, 0, n_groups, per_group * rows_per_split, 1000, dev)
    v = make_kv_groups(torch, xq, w, ty, 0, n_groups, per_group * rows_per_split, 2000, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    q = torch.randn((w["n_seq"], w["n_head"], 1, w["D"]), generator=g, device=dev)
    rows = w["n_seq"] * w["n_head"]
    part = torch.empty((n_splits, rows, w["D"] + 2), dtype=torch.float32, device=dev)
    rec = torch.empty((n_groups, rows, w["D"] + 2), dtype=torch.float32, device=dev)
    out = torch.empty((rows, w["D"]), dtype=torch.float32, device=dev)
    scale = 1.0 / math.sqrt(w["D"])

    def step(i):
        xq.fa_partials(q, k, v, ty, rows_per_split, 0, n_splits, scale=scale, out=part)
        xq.lse_merge_records(part, per_group, out=rec)
        xq.lse_merge(rec, out=out, want_lse=False)

    ms = graph_timed(torch, step, steps, warmup) / steps
    step(0)
    torch.cuda.synchronize()
    del k, v
    return {"n_gpus": 1, "workload": "BASELINE config 5 on one GPU (no collective)",
            "value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms, 5),
            "note": "the N = 1 point of this strong-scaling series (the default N = 1 line "
                    "is BASELINE config 2)"}, out


def cpu_oracle_sample(workload, seconds_cap=20.0, sample_kv=None):
    """Time the CPU restatement of ggml-cpu FLASH_ATTN_EXT on a bounded sample
    of the workload (all host threads); returns (GB/s, info)."""
    import oracle
    w = {"c5": C5, "c1": C1, "c2mtp": C2MTP}.get(workload, C2)
    ty = {"c2q4": oracle.Q4_0, "c1": oracle.F16}.get(workload, oracle.Q8_0)
    n_kv = sample_kv or w["n_kv"]
    n_seq, n_q = 1, w.get("n_q", 1)
    rng = np.random.default_rng(0)
    q = rng.normal(0, 1, (n_seq, w["n_head"], n_q, w["D"])).astype(np.float32)
    kf = rng.normal(0, 1, (n_seq, n_kv, w["n_hkv"], w["D"])).astype(np.float32)
    k = oracle.quantize(ty, kf)
    v = oracle.quantize(ty, rng.normal(0, 1, kf.shape).astype(np.float32))
    del kf
    m = None
    if n_q > 1:
        m = np.zeros((1, 1, n_q, n_kv), np.float16)
        for i in range(n_q):
            m[0, 0, i, n_kv - n_q + i + 1:] = -np.inf
    cores = os.cpu_count() or 1
    sc = 1.0 / math.sqrt(w["D"])
    oracle.flash_attn_ext(q, k, v, ty, ty, mask=m, scale=sc, nth=cores, n_workers=cores)  # warm
    t = time.perf_counter()
    reps = 0
    while True:
        oracle.flash_attn_ext(q, k, v, ty, ty, mask=m, scale=sc, nth=cores, n_workers=cores)
        reps += 1
        if time.perf_counter() - t > min(seconds_cap, 3.0) or reps >= 5:
            break
    dt = (time.perf_counter() - t) / reps
    b = k.nbytes + v.nbytes + 2 * q.nbytes + (m.nbytes if m is not None else 0)
    return b / dt / 1e9, {"cores": cores, "sample": f"1 sequence x {n_kv} rows x {n_q} "
                          f"quer{'ies' if n_q > 1 else 'y'}, {reps} reps, "
                          f"{dt * 1e3:.1f} ms each, {cores} threads"}


# ---------------------------------------------------------------------------
# GATED_DELTA_NET (config 3) and causal prefill (config 4)

def gdn_bytes(n_seq, T, w=C3):
    S, H, Hk, K = w["S"], w["H"], w["H_k"], w["slots"]
    state = n_seq * H * S * S * 4
    ins = 2 * n_seq * T * Hk * S * 4 + n_seq * T * H * S * 4 + 2 * n_seq * T * H * 4
    y = n_seq * T * H * S * 4
    return state * (1 + K) + ins + y, ins, y


def gdn_inputs(torch, dev, n_seq, T, seed, w=C3):
    """q, k L2-normalised N(0,1); v N(0,1); g = -softplus(N(0,1)); beta =
    sigmoid(N(0,1)); state 0.1 N(0,1) -- the config-3 distributions."""
    F = torch.nn.functional
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    S, H, Hk = w["S"], w["H"], w["H_k"]
    rn = lambda *shape: torch.randn(shape, generator=g, device=dev)
    q = F.normalize(rn(n_seq, T, Hk, S), dim=-1)
    k = F.normalize(rn(n_seq, T, Hk, S), dim=-1)
    v = rn(n_seq, T, H, S)
    gate = -F.softplus(rn(n_seq, T, H, 1))
    beta = torch.sigmoid(rn(n_seq, T, H, 1))
    state = 0.1 * rn(n_seq, H, S, S)
    return [q, k, v, gate, beta, state]


def run_gdn(args, rank, world, torch, dist, workload):
    """GATED_DELTA_NET, config 3.  N > 1: sharded by value head, rank r runs
    heads shard.head_block(32, N, r) (strong scaling: the op is fixed)."""
    import xq
    from xq import shard
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    n_seq, T = (8, 1) if workload == "c3a" else (1, 4096)
    w = C3
    hbm, _, peak_kind = peaks()
    step_bytes, in_bytes, y_bytes = gdn_bytes(n_seq, T)
    n_sets = 1 if step_bytes > 2 * L2_BYTES else math.ceil(2 * L2_BYTES / step_bytes) + 1
    sets = [gdn_inputs(torch, dev, n_seq, T, 100 + i) for i in range(n_sets)]
    h0, h1 = shard.head_block(w["H"], world, rank)
    Hl = h1 - h0
    n_dst = w["S"] * Hl * T * n_seq + w["slots"] * w["S"] ** 2 * Hl * n_seq
    dsts = [torch.empty(n_dst, dtype=torch.float32, device=dev) for _ in range(n_sets)]

    def run(x, dst):
        if world == 1:
            xq.gated_delta_net(*x, slots=w["slots"], out=dst)
        else:
            shard.gdn_heads(*x, slots=w["slots"], world=world, rank=rank, out=dst)

    def step(i):
        run(sets[i % n_sets], dsts[i % n_sets])

    clk = ClockSampler(dev.index)
    clk.start()
    ms = graph_timed(torch, step, args.steps, args.warmup, world, dist, dev) / args.steps
    clocks = clk.stop()
    # end to end: this rank's q, k (whole) and v, g, beta (its heads) from
    # pinned host memory, its y block back; the recurrent state stays resident
    x0 = sets[0]
    blocks = [x0[0], x0[1]] + [t[:, :, h0:h1] for t in x0[2:5]]
    hosts = [t.cpu().pin_memory() for t in blocks]
    n_y = n_seq * T * Hl * w["S"]
    y_host = torch.empty(n_y, dtype=torch.float32, pin_memory=True)

    def e2e_step(i):
        for h, d in zip(hosts, blocks):
            d.copy_(h, non_blocking=True)
        run(x0, dsts[0])
        y_host.copy_(dsts[0][:n_y], non_blocking=True)
    e2e_ms = graph_timed(torch, e2e_step, args.steps, args.warmup, world, dist, dev) / args.steps
    h2d = sum(t.numel() for t in hosts) * 4 * world
    ref1 = None
    if world > 1:
        if rank == 0:
            d1 = torch.empty(w["S"] * w["H"] * T * n_seq + w["slots"] * w["S"] ** 2 * w["H"] *
                             n_seq, dtype=torch.float32, device=dev)
            ms1 = graph_timed(torch, lambda i: xq.gated_delta_net(
                *sets[i % n_sets], slots=w["slots"], out=d1), args.steps, args.warmup) / args.steps
            ref1 = {"n_gpus": 1, "workload": "the same op unsharded on one GPU",
                    "value": round(step_bytes / (ms1 * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(ms1, 5)}
        dist.barrier()
    if rank != 0:
        return None
    value = step_bytes / (ms * 1e-3) / 1e9
    return {
        "metric": "gated-delta-net GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; q, k L2-normalised N(0,1), v N(0,1), g = -softplus, "
                "beta = sigmoid, state 0.1 N(0,1))",
        "config": workload_config(workload, world),
        "plan": {"value_heads_per_gpu": Hl},
        "roofline": {"bound": "hbm", "achieved": round(value, 2), "peak": hbm, "unit": "GB/s",
                     "frac": round(value / hbm, 4), "peak_kind": peak_kind,
                     "kernel": ("gdn_recurrent_kernel" if workload == "c3a" else
                                "gdn_chunk_prep_kernel + gdn_chunk_scan_kernel"),
                     "traffic": profile_traffic("gdn_" + workload)},
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": y_bytes},
        # decode: one recurrent kernel; prefill: the chunked prep and scan kernels
        "gpu_launches": args.steps * (1 if workload == "c3a" else 2),
        **({"scaling_reference": ref1} if ref1 else {}),
        "timing": "CUDA-graph replay of %d steps, CUDA events" % args.steps,
        "clocks": clocks,
    }


def prefill_flops(n_q, H, D):
    return 4.0 * D * H * n_q * (n_q + 1) / 2


def run_prefill(args, rank, world, torch, dist, workload):
    """Causal prefill, config 4 (F16 cache) or its shape over a Q8_0 / Q4_0
    cache.  N > 1: sharded by KV-head group (shard.prefill_part; strong
    scaling: the op is fixed)."""
    import xq
    from xq import shard
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    ty = {"c4q8": xq.Q8_0, "c4q4": xq.Q4_0}.get(workload, xq.F16)
    w = C4
    H, Hkv, D, N = w["n_head"], w["n_hkv"], w["D"], w["n_q"]
    _, tflops, peak_kind = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((1, H, N, D), generator=g, device=dev)
    k = xq.quantize_rows(ty, torch.randn((1, N, Hkv, D), generator=g, device=dev))
    v = xq.quantize_rows(ty, torch.randn((1, N, Hkv, D), generator=g, device=dev))
    mask = torch.full((1, 1, N, N), float("-inf"), dtype=torch.float16, device=dev).triu_(1)
    scale = 1.0 / math.sqrt(D)
    (h0, h1), (c0, c1), (r0, r1) = shard.prefill_block(H, Hkv, N, N, world, rank)
    out = torch.empty((1, r1 - r0, h1 - h0, D), dtype=torch.float32, device=dev)

    def step(i):
        shard.prefill_part(q, k, v, ty, mask, world, rank, scale=scale, out=out)

    clk = ClockSampler(dev.index)
    clk.start()
    ms = graph_timed(torch, step, args.steps, args.warmup, world, dist, dev) / args.steps
    clocks = clk.stop()
    q_blk = q[:, h0:h1, r0:r1]
    q_host = q_blk.cpu().pin_memory()
    o_host = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)

    def e2e_step(i):
        q_blk.copy_(q_host, non_blocking=True)
        step(i)
        o_host.copy_(out, non_blocking=True)
    n_e2e = max(3, args.steps // 4)
    e2e_ms = graph_timed(torch, e2e_step, n_e2e, args.warmup, world, dist, dev) / n_e2e
    fl = prefill_flops(N, H, D)
    ref1 = None
    if world > 1:
        if rank == 0:
            o1 = torch.empty((1, N, H, D), dtype=torch.float32, device=dev)
            ms1 = graph_timed(torch, lambda i: xq.flash_attn_ext(q, k, v, ty, mask=mask,
                                                                 scale=scale, out=o1),
                              args.steps, args.warmup) / args.steps
            ref1 = {"n_gpus": 1, "workload": "the same op unsharded on one GPU",
                    "value": round(fl / (ms1 * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "ms_per_step": round(ms1, 5),
                    "rank0_block_bit_identical": bool(torch.equal(o1[:, r0:r1, h0:h1], out))}
        dist.barrier()
    if rank != 0:
        return None
    value = fl / (ms * 1e-3) / 1e12
    quant = ty != xq.F16
    return {
        "metric": "causal prefill TFLOP/s", "value": round(value, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": ("synthetic (seeded N(0,1); K/V " + ("rounded to F16" if not quant else
                 "quantized by the ggml reference quantizer, widened to f16 by the library's "
                 "pre-pass inside every step") + "; explicit causal F16 mask)"),
        "config": workload_config(workload, world),
        "plan": {"q_heads": [h0, h1], "kv_heads": [c0, c1], "q_rows": [r0, r1]},
        "roofline": {"bound": "tensor", "achieved": round(value, 2), "peak": tflops,
                     "unit": "TFLOP/s", "frac": round(value / tflops, 4),
                     "peak_kind": peak_kind + " (bf16 burst)",
                     "kernel": "fa_prefill_kernel" + ("<QQ>" if quant else ""),
                     "traffic": profile_traffic("fa_prefill_" + workload)},
        "e2e": {"value": round(fl / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": q_host.numel() * 4 * world,
                "d2h_bytes_per_step": o_host.numel() * 4 * world},
        # mask block map + prefill (+ the two K/V widening kernels)
        "gpu_launches": args.steps * (4 if quant else 2),
        **({"scaling_reference": ref1} if ref1 else {}),
        "timing": "CUDA-graph replay of %d steps, CUDA events" % args.steps,
        "clocks": clocks,
    }


KVW = dict(n_tok=8192, n_hkv=4, D=256, rows=32768)


def kvw_bytes(w=KVW):
    import xq
    n = w["n_tok"] * w["n_hkv"]
    return 2 * (n * w["D"] * 4 + n * xq.row_bytes(xq.Q8_0, w["D"]) + w["n_tok"] * 8)


def run_kvw(args, torch):
    import xq
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = KVW
    hbm, _, peak_kind = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    n_sets = 4
    srcs = [(torch.randn((1, w["n_tok"], w["n_hkv"], w["D"]), generator=g, device=dev),
             torch.randn((1, w["n_tok"], w["n_hkv"], w["D"]), generator=g, device=dev))
            for _ in range(n_sets)]
    rb = xq.row_bytes(xq.Q8_0, w["D"])
    kc = torch.zeros((1, w["rows"], w["n_hkv"], rb), dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    bases = [i * w["n_tok"] % w["rows"] for i in range(n_sets)]
    idxs = [torch.arange(b, b + w["n_tok"], dtype=torch.int64, device=dev) for b in bases]

    def step(i):
        k, v = srcs[i % n_sets]
        xq.set_rows(kc, k, idxs[i % n_sets], xq.Q8_0)
        xq.set_rows(vc, v, idxs[i % n_sets], xq.Q8_0)

    clk = ClockSampler(dev.index)
    clk.start()
    ms = graph_timed(torch, step, args.steps, args.warmup) / args.steps
    clocks = clk.stop()
    one_ms = graph_timed(torch, lambda i: xq.set_rows(kc, srcs[i % n_sets][0], idxs[i % n_sets],
                                                      xq.Q8_0), args.steps, args.warmup) / args.steps
    # end to end: the new rows from pinned host memory, the written rows read back
    kh = srcs[0][0].cpu().pin_memory()
    vh = srcs[0][1].cpu().pin_memory()
    kback = torch.empty((1, w["n_tok"], w["n_hkv"], rb), dtype=torch.uint8, pin_memory=True)
    vback = torch.empty(kback.shape, dtype=torch.uint8, pin_memory=True)
    b0 = bases[0]

    def e2e_step(i):
        srcs[0][0].copy_(kh, non_blocking=True)
        srcs[0][1].copy_(vh, non_blocking=True)
        step(0)
        kback.copy_(kc[:, b0:b0 + w["n_tok"]], non_blocking=True)
        vback.copy_(vc[:, b0:b0 + w["n_tok"]], non_blocking=True)
    e2e_ms = graph_timed(torch, e2e_step, max(3, args.steps // 4), args.warmup) / max(
        3, args.steps // 4)
    step_bytes = kvw_bytes()
    value = step_bytes / (ms * 1e-3) / 1e9
    achieved = (step_bytes / 2) / (one_ms * 1e-3) / 1e9
    return {
        "metric": "KV-cache write GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32->q8_0",
        "data": "synthetic (seeded N(0,1) rows, contiguous append positions)",
        "config": workload_config("kvw"),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                     "kernel": "set_rows_block_kernel", "traffic": profile_traffic("set_rows_kvw")},
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": int(kh.numel() * 8),
                "d2h_bytes_per_step": int(kback.numel() * 2)},
        "gpu_launches": args.steps * 2,
        "timing": "CUDA-graph replay of %d steps, CUDA events" % args.steps,
        "clocks": clocks,
    }


# native KVarN4 range attention: the reference's overflow layout (records past
# origin 102400, precision tail 128), 24 Q / 4 KV heads, D=256, one query
KV4 = dict(n_head=24, n_hkv=4, origin=102400, active=32768, tail=128)


def kvarn4_bytes(w=KV4, active=None):
    """Bytes the call must read and write: the records of every group that has
    rows below the tail (each KV head's two slices, K and V), the stage and
    tail rows used, q, out and lse."""
    from oracle import kvarn4 as ok
    active = w["active"] if active is None else active
    desc = ok.Desc(w["origin"], active, w["tail"], w["n_hkv"])
    tail_begin = active - min(active, w["tail"])
    rec_groups = stage_rows = 0
    for g in range((active + 127) // 128):
        lo, hi = 128 * g, min(128 * (g + 1), tail_begin)
        if lo >= hi:
            continue
        if ok.staged(desc, g, active):
            stage_rows += hi - lo
        else:
            rec_groups += 1
    n = (rec_groups * desc.phys * ok.RECORD + (stage_rows + active - tail_begin) * desc.row_bytes)
    return 2 * n + w["n_head"] * 256 * 4 * 2 + w["n_head"] * 4


def run_kvarn4(args, torch):
    import xq
    from oracle import kvarn4 as ok
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = KV4
    hbm, _, peak_kind = peaks()
    desc = ok.Desc(w["origin"], w["active"], w["tail"], w["n_hkv"])
    kp = torch.from_numpy(ok.make_plane(desc, w["active"], 1)).to(dev)
    vp = torch.from_numpy(ok.make_plane(desc, w["active"], 2)).to(dev)
    step_bytes = kvarn4_bytes()
    n_sets = max(4, math.ceil(2 * L2_BYTES / step_bytes) + 1)
    planes = [(kp.clone(), vp.clone()) for _ in range(n_sets)]
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((1, w["n_head"], 256), generator=g, device=dev)
    pos = torch.tensor([w["origin"] + w["active"] - 1], dtype=torch.int32, device=dev)

    def step(i):
        k, v = planes[i % n_sets]
        xq.attend_range_kvarn4(k, v, q, pos, w["n_hkv"], w["origin"], w["active"], w["tail"],
                               w["active"], 1 / 16.0)

    clk = ClockSampler(dev.index)
    clk.start()
    ms = graph_timed(torch, step, args.steps, args.warmup) / args.steps
    clocks = clk.stop()
    # end to end: q, out and lse in pinned host memory through the public call
    # (the library stages q with a kernel and the merge writes out / lse over
    # PCIe); the planes stay resident (the server's KV image)
    q_host = q.cpu().pin_memory()
    o_host = torch.empty((1, w["n_head"], 256), dtype=torch.float32, pin_memory=True)
    l_host = torch.empty((1, w["n_head"]), dtype=torch.float32, pin_memory=True)

    def e2e_step(i):
        k, v = planes[i % n_sets]
        xq.attend_range_kvarn4(k, v, q_host, pos, w["n_hkv"], w["origin"], w["active"],
                               w["tail"], w["active"], 1 / 16.0, out=o_host, lse=l_host)
    e2e_ms = graph_timed(torch, e2e_step, max(3, args.steps // 4), args.warmup) / max(
        3, args.steps // 4)
    value = step_bytes / (ms * 1e-3) / 1e9
    return {
        "metric": "KVarN4 range attention GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4 records / f16 rows -> f32",
        "data": "synthetic (seeded native records, stage and tail rows; q N(0,1))",
        "config": workload_config("kv4"),
        "roofline": {"bound": "hbm", "achieved": round(value, 2), "peak": hbm, "unit": "GB/s",
                     "frac": round(value / hbm, 4), "peak_kind": peak_kind,
                     "kernel": "kvarn4_partials_kernel + lse_merge",
                     "traffic": profile_traffic("kvarn4_kv4")},
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": int(q.numel() * 4),
                "d2h_bytes_per_step": int((o_host.numel() + l_host.numel()) * 4)},
        "gpu_launches": args.steps * 2,
        "timing": "CUDA-graph replay of %d steps, CUDA events" % args.steps,
        "clocks": clocks,
    }


def cpu_kvarn4_sample(active=4096):
    """The oracle restatement (float64 numpy, record decode per group) on the
    first `active` rows of the same layout."""
    from oracle import kvarn4 as ok
    w = KV4
    desc = ok.Desc(w["origin"], active, w["tail"], w["n_hkv"])
    kp = ok.make_plane(desc, active, 1)
    vp = ok.make_plane(desc, active, 2)
    q = np.random.default_rng(0).normal(0, 1, (1, w["n_head"], 256)).astype(np.float32)
    t = time.perf_counter()
    reps = 0
    while True:
        ok.attend(desc, kp, vp, active, q, [w["origin"] + active - 1], 1 / 16.0, w["n_head"])
        reps += 1
        if time.perf_counter() - t > 3.0 or reps >= 10:
            break
    dt = (time.perf_counter() - t) / reps
    return kvarn4_bytes(active=active) / dt / 1e9, {
        "cores": 1, "unit": "GB/s",
        "sample": f"{active} rows (of {w['active']}), {reps} reps, {dt * 1e3:.0f} ms each, "
                  f"numpy float64, 1 thread"}


def cpu_kvw_sample(n_tok=1024):
    """The oracle's reference quantizer (all rows of n_tok tokens, K and V)
    plus the scatter, on the host."""
    import oracle
    w = KVW
    rng = np.random.default_rng(0)
    k = rng.normal(0, 1, (1, n_tok, w["n_hkv"], w["D"])).astype(np.float32)
    v = rng.normal(0, 1, k.shape).astype(np.float32)
    rb = oracle.row_size(oracle.Q8_0, w["D"])
    kc = np.zeros((1, w["rows"], w["n_hkv"], rb), np.uint8)
    vc = np.zeros_like(kc)
    pos = np.arange(100, 100 + n_tok)
    t = time.perf_counter()
    reps = 0
    while True:
        kc[0, pos] = oracle.quantize(oracle.Q8_0, k)[0]
        vc[0, pos] = oracle.quantize(oracle.Q8_0, v)[0]
        reps += 1
        if time.perf_counter() - t > 2.0 or reps >= 20:
            break
    dt = (time.perf_counter() - t) / reps
    b = kvw_bytes() * n_tok / w["n_tok"]
    return b / dt / 1e9, {"cores": 1, "unit": "GB/s",
                          "sample": f"{n_tok} tokens x {w['n_hkv']} heads x D={w['D']}, K and V, "
                                    f"{reps} reps, {dt * 1e3:.2f} ms each, 1 thread"}


def cpu_gdn_sample(workload):
    import oracle
    n_seq, T = (8, 1) if workload == "c3a" else (1, 256)
    rng = np.random.default_rng(0)
    S, H, Hk = C3["S"], C3["H"], C3["H_k"]

    def nrm(x):
        return (x / np.linalg.norm(x, axis=-1, keepdims=True)).astype(np.float32)
    q = nrm(rng.normal(0, 1, (n_seq, T, Hk, S)))
    k = nrm(rng.normal(0, 1, (n_seq, T, Hk, S)))
    v = rng.normal(0, 1, (n_seq, T, H, S)).astype(np.float32)
    gg = -np.log1p(np.exp(rng.normal(0, 1, (n_seq, T, H, 1)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, (n_seq, T, H, 1))))).astype(np.float32)
    state = (0.1 * rng.normal(0, 1, (n_seq, H, S, S))).astype(np.float32)
    cores = os.cpu_count() or 1
    oracle.gated_delta_net(q, k, v, gg, beta, state, slots=1, n_workers=cores)
    t = time.perf_counter()
    reps = 0
    while True:
        oracle.gated_delta_net(q, k, v, gg, beta, state, slots=1, n_workers=cores)
        reps += 1
        if time.perf_counter() - t > 3.0 or reps >= 10:
            break
    dt = (time.perf_counter() - t) / reps
    b = gdn_bytes(n_seq, T)[0]
    return b / dt / 1e9, {"cores": cores, "unit": "GB/s",
                          "sample": f"{n_seq} seqs x {T} tokens, {reps} reps, "
                                    f"{dt * 1e3:.2f} ms each, {cores} threads"}


def cpu_prefill_sample(workload="c4", rows=64):
    """The last `rows` queries of config 4 (the longest causal rows), over the
    workload's cache type."""
    import oracle
    H, Hkv, D, N = C4["n_head"], C4["n_hkv"], C4["D"], C4["n_q"]
    ty = {"c4q8": oracle.Q8_0, "c4q4": oracle.Q4_0}.get(workload, oracle.F16)
    rng = np.random.default_rng(0)
    q = rng.normal(0, 1, (1, H, rows, D)).astype(np.float32)
    kf = rng.normal(0, 1, (1, N, Hkv, D)).astype(np.float32)
    k = oracle.quantize(ty, kf)
    v = oracle.quantize(ty, rng.normal(0, 1, kf.shape).astype(np.float32))
    pos = np.arange(N - rows, N)
    mask = np.where(np.arange(N)[None, :] > pos[:, None], -np.inf, 0).astype(np.float16)
    mask = mask.reshape(1, 1, rows, N)
    cores = os.cpu_count() or 1
    t = time.perf_counter()
    oracle.flash_attn_ext(q, k, v, ty, ty, mask=mask, scale=1 / 16, nth=cores, n_workers=cores)
    dt = time.perf_counter() - t
    fl = 4.0 * D * H * float((pos + 1).sum())
    return fl / dt / 1e12, {"cores": cores, "unit": "TFLOP/s",
                            "sample": f"last {rows} of {N} causal queries x {H} heads, "
                                      f"{dt:.2f} s, {cores} threads"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="auto", choices=["auto"] + list(WORKLOAD_NAMES))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    workload = args.workload if args.workload != "auto" else ("c2" if world == 1 else "c5")

    if args.impl == "reference":
        if rank != 0:
            return 0
        metric, unit = "flash-decode KV GB/s", "GB/s"
        if workload in ("c3a", "c3b"):
            (val, info), metric = cpu_gdn_sample(workload), "gated-delta-net GB/s"
        elif workload in ("c4", "c4q8", "c4q4"):
            (val, info), metric, unit = (cpu_prefill_sample(workload), "causal prefill TFLOP/s",
                                         "TFLOP/s")
        elif workload == "kvw":
            (val, info), metric = cpu_kvw_sample(), "KV-cache write GB/s"
        elif workload == "kv4":
            (val, info), metric = cpu_kvarn4_sample(), "KVarN4 range attention GB/s"
        else:
            val, info = cpu_oracle_sample(workload)
        val = float(f"{val:.4g}")
        line = {"metric": metric, "value": val, "unit": unit,
                "impl": "reference", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
                "config": workload_config(workload, world), "data": "synthetic",
                "cpu_baseline": {"value": val, "unit": unit, "cores": info["cores"],
                                 "kind": "port", "sample": info["sample"]},
                "e2e": {"value": val, "unit": unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    if workload in ("kvw", "kv4") and world > 1:
        # the KV-cache write and the KVarN4 range call are measured on one GPU
        print(json.dumps({"error": f"workload {workload} runs on one GPU"}), flush=True)
        return 2
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    if workload in ("c3a", "c3b"):
        line = run_gdn(args, rank, world, torch, dist, workload)
    elif workload in ("c4", "c4q8", "c4q4"):
        line = run_prefill(args, rank, world, torch, dist, workload)
    elif workload == "kvw":
        line = run_kvw(args, torch)
    elif workload == "kv4":
        line = run_kvarn4(args, torch)
    else:
        line = run_decode(args, rank, world, torch, dist, workload)
    if rank == 0 and line is not None:
        if world == 1 and not args.no_cpu_baseline:
            if workload in ("c3a", "c3b"):
                val, info = cpu_gdn_sample(workload)
            elif workload in ("c4", "c4q8", "c4q4"):
                val, info = cpu_prefill_sample(workload)
            elif workload == "kvw":
                val, info = cpu_kvw_sample()
            elif workload == "kv4":
                val, info = cpu_kvarn4_sample()
            else:
                val, info = cpu_oracle_sample(workload)
                info["unit"] = "GB/s"
            line["cpu_baseline"] = {"value": float(f"{val:.4g}"), "unit": info["unit"],
                                    "cores": info["cores"], "kind": "port",
                                    "sample": info["sample"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
