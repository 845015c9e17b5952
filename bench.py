#!/usr/bin/env python
"""Benchmark of the B200 DSA lightning indexer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

A step is one indexer call (score + top-2048 select) over one batch of the
workload.  The default workload is benchmark config 1 (B=64 decode rows,
seq_lens U[4096, 32768], synthetic inputs generated on the device from a
fixed seed).  Under torchrun (N > 1) every rank runs the same batch in its
own GPU's memory (replicated batches, no collective in the timed loop:
"scaling": "weak"), the timing is the max over ranks and value sums the
ranks' bytes.  The same line carries strong_config2 (config 2's B=256 batch
partitioned across the N ranks, each holding only its rows' pages: strong
scaling), split_config3 (config 3's 131072-token row split by page range
with an NCCL all-gather merge) and, at N = 1, configs 2 and 4.

value:     index-K GB/s = algorithmic bytes per call x K / device time of K calls
           (inputs resident in HBM, 3 rotating copies of the inputs so no call
           reuses L2-resident K pages of the previous one).
e2e:       the same metric through the drop-in kernel(...) with pinned host
           inputs: every step copies all input tensors host->device and the
           output device->host inside the timed region.
roofline:  the scoring kernel alone: its algorithmic bytes / its mean
           CUDA-event duration, against the measured HBM copy bandwidth.
cpu_baseline: the torch CPU formulation of the operator (torch's thread
           pool) on a bounded sample of the same batch, with the exact C
           oracle's rate beside it (rank 0, N = 1 only).
parity:    every row of the timed batch (up to 128) against the exact C
           oracle, after the timed region: failures, worst logit error,
           tie-band differences; a failure replaces the line by an error.
reference_kernel: the reference's own CUDA kernel (baseline/Makefile) on the
           same batch, µs per call.
--impl reference: the torch CPU formulation on the host cores, each step a
           bounded sample of the workload.
--op write_k: the index-K cache writer (bf16 keys -> e4m3 pages) on
           --tokens new tokens per call instead of the indexer.
--op prefill: one prefill chunk (--chunk causal rows of a --last-len
           sequence), in groups of 4 rows and row by row.
--op attn: the sparse MLA attention that consumes the indexer's output.
--op graph: small-batch latency (config 0), kernel(...) called eagerly
           against the same call replayed from a CUDA graph (IndexerGraph).
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
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib, kernel, read_status, run  # noqa: E402
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W  # noqa: E402

METRIC = "index-K HBM GB/s per indexer call (score + top-2048), B=64 decode"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) of one scoring launch from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of this bench's workload,
# with the SHA-256 of that kernel's device sources (KERNEL_SOURCES) when it
# was captured.  roofline.traffic
# reports it only while the sources still hash the same; otherwise it is
# null and the old capture is shown as traffic_last_profiled.
SCORE_TRAFFIC = {
    1: {"bytes": 156_345_088 + 4_192_256, "kernel": "score_kernel",
        "src_sha256": "6076b755325c321c8e1e35eca60c837e13ae147d6b8f346240c708937c23a3f7"},
    4: {"bytes": 156_744_448 + 6_459_136, "kernel": "score_mq_kernel<4>",
        "src_sha256": "0dab5fb9f9b421e936b27d330bd289e0645added1da744c932a7cdfad5189a24"},
}
N_SETS = 3


KERNEL_SOURCES = {
    "score_kernel": ["score.cu", "common.cuh", "sm100.cuh", "tiles.cuh"],
    "score_mq_kernel<4>": ["score_mq.cu", "common.cuh", "sm100.cuh", "tiles.cuh"],
}


def kernel_sources_sha256(kernel: str) -> str:
    """SHA-256 over the device sources one kernel is compiled from."""
    import hashlib
    h = hashlib.sha256()
    csrc = REPO / "dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200" / "csrc"
    for name in KERNEL_SOURCES[kernel]:
        h.update(name.encode())
        h.update((csrc / name).read_bytes())
    return h.hexdigest()


def traffic_entry(config: int, rows_per_seq: int, config_rps: int) -> dict:
    cap = SCORE_TRAFFIC.get(config)
    if cap is None or rows_per_seq != config_rps:
        return {"traffic": None, "traffic_source": "no ncu capture for this workload"}
    if cap["src_sha256"] and cap["src_sha256"] == kernel_sources_sha256(cap["kernel"]):
        return {"traffic": cap["bytes"],
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch of this build"}
    return {"traffic": None, "traffic_last_profiled": cap["bytes"],
            "traffic_source": "the last ncu capture ran other kernel sources; not reported as this build's"}


def measured_hbm_peak():
    p = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def score_bytes(inp) -> int:
    """Algorithmic bytes of the scoring kernel: per scored row 132*L (K +
    scale) + 4*ceil(L/64) (block table) + 8192 (q) + 256 (weights) + 4.
    With rows_per_seq = R > 1 the K + scale and block-table bytes count once
    per group of R rows, for its longest row."""
    sl = np.clip(inp.seq_lens.cpu().numpy().astype(np.int64), 0, inp.max_pages * 64)
    R = max(1, inp.rows_per_seq)
    if R == 1:
        sl = sl[sl > 2048]
        return int((132 * sl + 4 * ((sl + 63) // 64) + 8192 + 256 + 4).sum())
    lmax = sl.reshape(-1, R).max(axis=1)
    lmax = lmax[lmax > 2048]
    return int((132 * lmax + 4 * ((lmax + 63) // 64) + R * (8192 + 256 + 4)).sum())


def score_flops(inp) -> int:
    """Algorithmic tensor flops of the scoring kernel: 2 * 64 heads * 128
    dims per scored (row, token) pair, each row over its own length."""
    sl = np.clip(inp.seq_lens.cpu().numpy().astype(np.int64), 0, inp.max_pages * 64)
    R = max(1, inp.rows_per_seq)
    scored = np.repeat(sl.reshape(-1, R).max(axis=1) > 2048, R)
    return int(2 * 64 * 128 * sl[scored].sum())


def measured_fp8_peak():
    """Dense fp8 tensor peak: twice the measured cuBLAS bf16 burst rate (the
    fp8 rate of B200's tensor cores is twice its bf16 rate; no fp8 GEMM is
    measured on this pool)."""
    p = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return 2.0 * float(d["bf16_tflops"]), "2 x measured bf16 burst (MEASURED_PEAKS.json bf16_tflops)"
    except Exception:
        return 2.0 * 1590.0, "2 x fallback bf16 1.59 PFLOP/s"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.lines: list[str] = []
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.sel = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.sel = str(device.index or 0)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.sel], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)  # at least one sample at the end of the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def parity_guard(inp):
    """Refuses to time a wrong kernel: the selected ids of every row must be
    distinct, reachable through the block table and an exact top-2048 of the
    kernel's own logits.  Runs once, outside the timed region, on torch.
    Returns the ids and logits of that call (device tensors)."""
    out = inp.out()
    lg = torch.full((inp.rows, inp.max_pages * 64), float("nan"), device=inp.q.device)
    run(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out, logits_out=lg,
        rows_per_seq=inp.rows_per_seq)
    torch.cuda.synchronize()
    st = read_status(inp.q.device)
    if st != 0:
        raise SystemExit(json.dumps({"error": f"device status {st:#x} on the parity guard call"}))
    sl = inp.seq_lens.tolist()
    for b in range(inp.rows):
        L = sl[b]
        ids = out[b].long()
        if L <= 2048:
            continue
        t = torch.arange(L, device=lg.device)
        phys = inp.block_table[b, t // 64].long() * 64 + t % 64
        inv = torch.full((int(phys.max()) + 1,), -1, dtype=torch.long, device=lg.device)
        inv[phys] = t
        ok = bool((ids >= 0).all()) and bool((ids <= phys.max()).all())
        toks = inv[ids.clamp(0, int(phys.max()))]
        ok = ok and bool((toks >= 0).all()) and int(torch.unique(toks).numel()) == 2048
        if ok:
            sel = torch.zeros(L, dtype=torch.bool, device=lg.device)
            sel[toks] = True
            row = lg[b, :L]
            ok = bool(row[sel].min() >= row[~sel].max())
        if not ok:
            raise SystemExit(json.dumps({"error": f"parity guard failed on row {b}"}))
    return out, lg


def cpu_leg(base, gpu_ids, gpu_logits, budget_s: float, max_parity_rows: int = 128):
    """The CPU baseline and the parity check of the timed batch (rank 0,
    N = 1, after the timed region).

    * The exact C oracle (all host threads) computes every row of the batch
      (at most `max_parity_rows`, sampled evenly beyond that); its logits and
      ids check the GPU's under the north-star rules: logits within rtol
      1e-2, index sets equal outside the tie band, differences inside it
      counted, short rows and -1 padding bit-exact.  Its time is reported
      too.
    * The torch CPU formulation (fp8 -> fp32 dequant per page chunk, GEMM,
      ReLU * weights * scale, torch.topk; torch's thread pool) is timed on as
      many whole rows (groups) as fit in about budget_s: the cpu_baseline.
    Returns (cpu_baseline dict, parity dict); parity["failures"] > 0 means
    the GPU result is wrong."""
    from oracle import oracle, torch_path  # CPU baseline leg only: timed baseline and checker
    R = max(1, base.rows_per_seq)
    threads = os.cpu_count() or 1
    rows = list(range(base.rows))
    if len(rows) > max_parity_rows:
        groups = base.rows // R
        pick = np.linspace(0, groups - 1, max_parity_rows // R).astype(int)
        rows = sorted({int(g) * R + i for g in pick for i in range(R)})
    sub = base.subset(rows) if len(rows) < base.rows or base.k_cache.numel() > (1 << 31) else base.to("cpu")
    d = sub.numpy()
    t0 = time.perf_counter()
    lg, mag = oracle.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                            num_pages=d["num_pages"], nthreads=threads, with_mag=True)
    ora_ids = oracle.topk(lg, d["seq_lens"], d["block_table"])
    t_oracle = time.perf_counter() - t0
    ids_all = gpu_ids.cpu().numpy()
    bt_all = base.block_table.cpu().numpy()
    sl_all = base.seq_lens.cpu().numpy()
    glog = gpu_logits[rows].cpu().numpy()
    failures, diffs, worst, msgs = 0, 0, 0.0, []
    try:
        worst = oracle.check_logits(glog, lg, mag, d["seq_lens"])
    except AssertionError as e:
        failures += 1
        msgs.append(f"logits: {e}")
    for i, b in enumerate(rows):
        L = int(min(max(sl_all[b], 0), base.max_pages * 64))
        ids = ids_all[b]
        if sub.num_pages != base.num_pages or len(rows) < base.rows:
            ids = remap_ids(ids, bt_all[b], d["block_table"][i], L)
        try:
            r = oracle.check_row(ids, lg[i], d["block_table"][i], L, gpu_logits=glog[i])
            diffs += r["diff"]
        except AssertionError as e:
            failures += 1
            msgs.append(f"row {b}: {e}")
    sub_bytes = W.Inputs(sub.q, sub.k_cache, sub.weights, sub.seq_lens, sub.block_table,
                         rows_per_seq=R).algorithmic_bytes()
    parity = {"rows_checked": len(rows), "of_rows": base.rows, "failures": failures,
              "worst_logit_rel_err": float(f"{worst:.3g}"), "tie_band_differences": diffs,
              "checker": "exact C oracle (fp64 head sums, exact top-2048); logits rtol 1e-2, "
                         "index sets equal outside the tie band 1e-2*|s_2048|, short rows bit-exact",
              "oracle_s": round(t_oracle, 3)}
    if msgs:
        parity["messages"] = msgs[:4]
    # torch CPU formulation, timed on whole rows (groups) within the budget
    tth = torch.get_num_threads()

    def torch_rows(n):
        t1 = time.perf_counter()
        torch_path.indexer(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"], rows=range(n))
        return time.perf_counter() - t1

    t_first = torch_rows(R)
    n = int(max(R, min(len(rows), budget_s / max(t_first / R, 1e-4))))
    n = max(R, n - n % R)
    dt = torch_rows(n)
    tsub = W.Inputs(sub.q[:n], sub.k_cache, sub.weights[:n], sub.seq_lens[:n], sub.block_table[:n],
                    rows_per_seq=R)
    gbs = tsub.algorithmic_bytes() / dt / 1e9
    cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": tth, "kind": "port",
           "host_cpus": os.cpu_count(),
           "sample": f"first {n} of {base.rows} rows of the same batch, torch CPU formulation "
                     f"(e4m3->fp32 per page chunk, fp32 GEMM, ReLU*w*scale, torch.topk), "
                     f"torch.get_num_threads()={tth}, {dt:.2f} s",
           "c_oracle": {"value": round(sub_bytes / t_oracle / 1e9, 4), "unit": "GB/s", "cores": threads,
                        "sample": f"{len(rows)} rows (exact fp64 C oracle, {threads} threads), {t_oracle:.2f} s"}}
    return cpu, parity


def remap_ids(ids, bt_orig, bt_sub, L):
    """Physical ids of the full pool rewritten as ids of a compact subset
    pool (Inputs.subset), token by token; ids that are not slots of the
    row's first L tokens map to -2 (the checker then rejects them)."""
    t = np.arange(L)
    tok_of = dict(zip((bt_orig[t // 64].astype(np.int64) * 64 + t % 64).tolist(), t.tolist()))
    out = np.array(ids, dtype=np.int64)
    for j, p in enumerate(out.tolist()):
        if p >= 0:
            tt = tok_of.get(int(p), -1)
            out[j] = int(bt_sub[tt // 64]) * 64 + tt % 64 if tt >= 0 else -2
    return out


def time_reference_kernel(sets, steps: int, warmup: int, active: bool = False) -> dict:
    """The reference's own CUDA kernel (solution/cuda/kernel.cu, built
    unmodified by baseline/Makefile) on the same rotating input sets: K
    back-to-back calls through its entry point, CUDA events on the current
    stream.  Its stage 1 writes fp16 logits into a scratch it allocates per
    call through torch (solution/cuda/kernel.cu:471-476)."""
    from baseline import ref_kernel
    ok, why = ref_kernel.active_available() if active else ref_kernel.available()
    if not ok:
        return {"unavailable": why}
    outs = [s.out() for s in sets]
    fn = ref_kernel.active_kernel if active else ref_kernel.kernel

    def step(i):
        s = sets[i % len(sets)]
        fn(s.q, s.k_cache, s.weights, s.seq_lens, s.block_table, outs[i % len(sets)])

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    alg = sets[0].algorithmic_bytes()
    return {"source": ref_kernel.ACTIVE_SOURCE if active else ref_kernel.SOURCE, "us_per_call": round(ms * 1e3, 2),
            "value": round(alg / (ms / 1e3) / 1e9, 1), "unit": "GB/s", "steps": steps,
            "timing": "CUDA events over back-to-back calls through its own entry point (TVM-FFI export or torch extension)"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
    return world, rank, local


def rotating_sets(base, n=N_SETS):
    """`n` copies of a batch in separate device memory (the copies rotate
    between calls so no call finds the previous call's K pages in L2)."""
    return [base] + [W.Inputs(base.q.clone(), base.k_cache.clone(), base.weights.clone(), base.seq_lens.clone(),
                              base.block_table.clone(), base.name, base.seed, rows_per_seq=base.rows_per_seq)
                     for _ in range(n - 1)]


def time_calls(sets, outs, R, steps, warmup, world, dev):
    """K back-to-back indexer calls over the rotating sets, bracketed by a
    barrier and synchronize on both sides; returns (max over ranks of the
    elapsed ms, clocks sampled during the region)."""
    import torch.distributed as dist

    def step(i):
        s = sets[i % len(sets)]
        run(s.q, s.k_cache, s.weights, s.seq_lens, s.block_table, outs[i % len(sets)], rows_per_seq=R)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), clk


def kernel_times(sets, outs, R, n_ev):
    """Mean CUDA-event durations of the scoring launch and of the selection
    launch (events around each launch on the launching stream; the event
    between the two is recorded inside the library)."""
    ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    ev_m = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    for ev in ev_m:  # torch only times events it has seen recorded
        ev.record()
    torch.cuda.synchronize()
    for i in range(n_ev):
        s = sets[i % len(sets)]
        ev_s[i].record()
        run(s.q, s.k_cache, s.weights, s.seq_lens, s.block_table, outs[i % len(sets)], event_after_score=ev_m[i],
            rows_per_seq=R)
        ev_e[i].record()
    torch.cuda.synchronize()
    score_ms = statistics.mean(ev_s[i].elapsed_time(ev_m[i]) for i in range(n_ev))
    select_ms = statistics.mean(ev_m[i].elapsed_time(ev_e[i]) for i in range(n_ev))
    return score_ms, select_ms


def extra_config(config: int, steps: int, warmup: int, dev, with_reference: bool = True) -> dict:
    """One more benchmark config on this GPU (N = 1): µs per call over K
    back-to-back calls (rotating copies when the pool is smaller than four
    times L2), algorithmic GB/s and fraction of the measured HBM peak, the
    scoring launch alone, and the parity guard (exact top-K of its own
    logits)."""
    base = W.config_inputs(config, seed=100 * config, device=dev)
    R = base.rows_per_seq
    n_sets = 1 if base.k_cache.numel() > 4 * 126e6 else N_SETS
    sets = rotating_sets(base, n_sets)
    outs = [x.out() for x in sets]
    parity_guard(base)
    ms, clk = time_calls(sets, outs, R, steps, warmup, 1, dev)
    score_ms, select_ms = kernel_times(sets, outs, R, max(3, min(steps, 50)))
    alg = base.algorithmic_bytes()
    peak, _ = measured_hbm_peak()
    sb = score_bytes(base)
    gbs = alg / (ms / steps / 1e3) / 1e9
    out = {"workload": f"config{config}: {W.CONFIGS[config]}", "rows": base.rows, "rows_per_seq": R,
           "us_per_call": round(ms / steps * 1e3, 2), "value": round(gbs, 1), "unit": "GB/s",
           "frac_of_hbm_peak": round(gbs / peak, 4), "steps": steps,
           "kernels_ms": {"score": round(score_ms, 5), "select": round(select_ms, 5)},
           "score_frac_of_hbm_peak": round(sb / (score_ms / 1e3) / 1e9 / peak, 4),
           "l2": f"{n_sets} input cop{'y' if n_sets == 1 else 'ies'} of a {base.k_cache.numel() / 1e6:.0f} MB K pool",
           "clocks": clk}
    if R > 1:
        tpeak, _ = measured_fp8_peak()
        out["score_frac_of_fp8_peak"] = round(score_flops(base) / (score_ms / 1e3) / 1e12 / tpeak, 4)
    if with_reference:
        # the reference scores every row on its own (it has no shared-page groups)
        for key, active in (("reference_kernel", False), ("reference_kernel_active", True)):
            ref = time_reference_kernel(sets, max(3, min(steps, 20)), 3, active=active)
            if "us_per_call" in ref:
                ref["value"] = round(alg / (ref["us_per_call"] / 1e6) / 1e9, 1)
                ref["note"] = "value: this config's algorithmic bytes per call over the reference's time"
            out[key] = ref
    del sets, outs, base
    torch.cuda.empty_cache()
    return out


def small_shape_latency(steps: int, warmup: int, dev) -> dict:
    """Latency of small calls (the contest's workload sizes: B <= 31 rows of
    at most 91 pages), where per-call host work and kernel latency dominate:
    the drop-in kernel(...) called back to back (CUDA events over the calls,
    and the host time to issue one call), the same call through the
    library's graph cache (run(..., graph=True): one cached executable graph
    per launch plan, pointers written into its nodes), and the call replayed
    from a CUDA graph of fixed tensors (IndexerGraph; device time only)."""
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import IndexerGraph, run
    shapes = {"config0 (B=2, L {1500, 4096}, 64 pages)": W.config_inputs(0, device=dev),
              "B=14, L 1924..5824, 91 pages": W.make_inputs(list(range(5824 - 13 * 300, 5825, 300)), max_pages=91,
                                                           seed=5, device=dev)}
    res = {}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(call):
        for _ in range(warmup + 20):
            call()
        torch.cuda.synchronize()
        e0.record()
        t0 = time.perf_counter()
        for _ in range(steps):
            call()
        t1 = time.perf_counter()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps * 1e3, (t1 - t0) / steps * 1e6

    for name, g in shapes.items():
        out = g.out()
        eager, host = timed(lambda: kernel(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out))
        cached, chost = timed(lambda: run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, graph=True))
        gr = IndexerGraph(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out)
        replay, _ = timed(gr.replay)
        res[name] = {"eager_us_per_call": round(eager, 2), "host_us_per_call": round(host, 2),
                     "graph_cache_us_per_call": round(cached, 2), "graph_cache_host_us_per_call": round(chost, 2),
                     "graph_replay_us_per_call": round(replay, 2)}
        del gr
    res["timing"] = (f"{steps} back-to-back calls, CUDA events; host = time to issue one call "
                     "(perf_counter, no synchronisation inside)")
    return res


def strong_config2(args, world, rank, local) -> dict:
    """Config 2 as a partitioned batch (strong scaling): the B=256 rows of
    64K-128K tokens are split over the ranks by shard_rows (balanced by
    tokens); each rank holds only its rows' pages (a compact pool of its
    own) and runs the indexer on them with no collective on the data path.
    value = the whole batch's algorithmic bytes / the max over ranks of the
    per-call time; gather_rows (an all-gather of every rank's [rows, 2048]
    ids) is timed separately."""
    import torch.distributed as dist
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import distributed as D
    dev = torch.device("cuda", local)
    full = W.config_inputs(2, seed=200, device=dev)       # the same batch on every rank
    alg_total = full.algorithmic_bytes()
    r0, r1 = D.shard_rows(full.seq_lens.cpu().numpy(), world, rank)
    mine = full.subset(range(r0, r1), device=dev) if world > 1 else full
    del full
    torch.cuda.empty_cache()
    out = mine.out()
    steps = max(3, min(args.steps, args.strong_steps))
    ms, clk = time_calls([mine], [out], 1, steps, max(3, min(args.warmup, 5)), world, dev)
    per_call = ms / steps
    if world > 1:
        cnt = torch.tensor([r1 - r0], device=dev)
        allc = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(allc, cnt)
        counts = [int(c.item()) for c in allc]
        gbuf = torch.empty((world, max(counts), 2048), dtype=torch.int32, device=dev)
        for _ in range(3):
            D.gather_rows(out, counts, buf=gbuf)
        torch.cuda.synchronize()
        # device time of the all-gather: 10 calls captured in a CUDA graph
        ggraph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        dist.barrier()
        with torch.cuda.graph(ggraph, stream=side):
            for _ in range(10):
                D.gather_rows(out, counts, buf=gbuf)
        torch.cuda.current_stream(dev).wait_stream(side)
        ggraph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        ggraph.replay()
        g1.record()
        torch.cuda.synchronize()
        tg = torch.tensor([g0.elapsed_time(g1) / 10], device=dev)
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        gather_us = round(float(tg.item()) * 1e3, 2)
        dist.barrier()
        del ggraph  # holds NCCL work: released before the process group
    else:
        counts, gather_us = [r1 - r0], 0.0
    peak, _ = measured_hbm_peak()
    gbs = alg_total / (per_call / 1e3) / 1e9
    del mine, out
    torch.cuda.empty_cache()
    return {"workload": f"config2: {W.CONFIGS[2]}, rows partitioned across {world} GPU(s)",
            "scaling": "strong", "rows_per_rank": counts, "us_per_call": round(per_call * 1e3, 2),
            "value": round(gbs, 1), "unit": "GB/s (whole batch)", "frac_of_n_x_hbm_peak": round(gbs / (world * peak), 4),
            "steps": steps, "gather_rows_us": gather_us,
            "gather_rows_timing": "10 calls captured in a CUDA graph, replayed once, CUDA events, max over ranks",
            "timing": "CUDA events, max over ranks; each rank holds only its rows' pages; no collective in the timed calls",
            "clocks": clk}


def split_config3(args, world, rank, local, steps: int | None = None) -> dict:
    """Config 3: one 131072-token row split by page range over the ranks
    (strong scaling).  A step = local scoring + local top-2048 pairs
    (dsai_run_pairs), one NCCL all-gather of the 2048 (score, token) pairs of
    every rank (packed in one buffer), merge (dsai_merge_pairs).  Every rank
    builds the same seeded row; a rank reads only the pages of its range.
    The row's pool (9.5 MB) fits in L2, so steps rotate over 16 copies of it
    (152 MB, larger than L2)."""
    import torch.distributed as dist
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import distributed as D
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import merge_pairs, run_pairs
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    steps = steps or args.steps
    seed = 300
    g = W.config_inputs(3, seed=seed, device=dev)
    L = int(g.seq_lens[0])
    p0, p1 = D.page_range(L, world, rank)
    local_len = max(0, min(L, p1 * 64) - p0 * 64)
    bt_local = g.block_table[:, p0:p1].contiguous()
    sl_local = torch.tensor([local_len], dtype=torch.int32, device=dev)
    pairs = torch.empty((2, 2048), dtype=torch.int32, device=dev)   # scores (fp32 bits), tokens
    sc, tk = pairs[0].view(torch.float32).view(1, 2048), pairs[1].view(1, 2048)
    all_pairs = torch.empty((world, 2, 2048), dtype=torch.int32, device=dev)
    pools = [g.k_cache] + [g.k_cache.clone() for _ in range(15)]  # 16 x 9.5 MB > L2
    bt_full = g.block_table[0].contiguous()
    sl_full = g.seq_lens[:1].contiguous()
    out = torch.empty(2048, dtype=torch.int32, device=dev)
    cand_sc = torch.empty(world * 2048, dtype=torch.float32, device=dev)  # every rank's scores, then tokens
    cand_tk = torch.empty(world * 2048, dtype=torch.int32, device=dev)
    ws = _lib.Workspace(dev)  # explicit: the same workspace in eager calls and in the captured graph

    def step(i=0):
        run_pairs(g.q, pools[i % len(pools)], g.weights, sl_local, bt_local, p0 * 64, sc, tk, workspace=ws)
        if world > 1:
            dist.all_gather_into_tensor(all_pairs.view(-1), pairs.view(-1))
            cand_sc.view(world, 2048).copy_(all_pairs[:, 0].view(torch.float32))
            cand_tk.view(world, 2048).copy_(all_pairs[:, 1])
            merge_pairs(cand_sc, cand_tk, bt_full, sl_full, out)
        else:
            merge_pairs(sc.view(-1), tk.view(-1), bt_full, sl_full, out)

    # parity guard: same set as the direct single-call indexer, planted tokens kept
    step()
    direct = g.out()
    kernel(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, direct)
    torch.cuda.synchronize()
    t = torch.tensor(g.planted[0], device=dev)
    planted = (g.block_table[0, t // 64].long() * 64 + t % 64).tolist()
    got = set(out.tolist())
    if not set(planted) <= got or len(got & set(direct[0].tolist())) < 2048 - 16:
        raise SystemExit(json.dumps({"error": "split-row parity guard failed"}))
    for i in range(max(args.warmup, len(pools))):
        step(i)
    torch.cuda.synchronize()
    # The step as a serving loop runs it: one CUDA graph of one step per pool
    # copy (16 steps, the NCCL all-gather included), replayed; the per-call
    # Python and launch work would otherwise dominate this latency-bound step.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    if world > 1:
        dist.barrier()
    with torch.cuda.graph(graph, stream=side):
        for i in range(len(pools)):
            step(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    reps = max(1, steps // len(pools))
    for _ in range(2):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    got_g = set(out.tolist())
    if not set(planted) <= got_g:
        raise SystemExit(json.dumps({"error": "split-row parity guard failed after the graph replays"}))
    steps = reps * len(pools)
    tt = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item()) / steps
    if world > 1:
        dist.barrier()
    del graph  # holds NCCL work: released before the process group
    alg = g.algorithmic_bytes()
    ref = None
    if world == 1 and not args.no_reference_kernel:
        rsets = [W.Inputs(g.q, pool, g.weights, g.seq_lens, g.block_table) for pool in pools]
        ref = {"tvm_ffi_variant": time_reference_kernel(rsets, max(3, min(steps, 200)), 3),
               "active": time_reference_kernel(rsets, max(3, min(steps, 200)), 3, active=True)}
    del pools
    torch.cuda.empty_cache()
    extra = {"reference_kernel": ref} if ref is not None else {}
    return {**extra, "workload": f"config3: {W.CONFIGS[3]}", "scaling": "strong", "seq_len": L,
            "pages_per_rank": p1 - p0, "seed": seed, "us_per_call": round(ms * 1e3, 2),
            "value": round(alg / (ms / 1e3) / 1e9, 1), "unit": "GB/s", "steps": steps,
            "l2": "16 rotating copies of the 9.5 MB page pool (152 MB > 126 MB L2)",
            "parallelism": f"page-range split, NCCL all-gather of 2048 (score, token) pairs per rank x{world}",
            "timing": "CUDA graph of 16 steps (one per pool copy) replayed, CUDA events, max over ranks",
            "launches_per_call": 3, "clocks": clk}


def bench_split(args, world, rank, local):
    """--config 3 as the headline line (see split_config3)."""
    r = split_config3(args, world, rank, local)
    if rank != 0:
        return None
    return {
        "metric": "index-K HBM GB/s, one 131072-token row split by page range", "value": r["value"],
        "unit": "GB/s", "n_gpus": world, "steps": r["steps"], "warmup": args.warmup,
        "ms_per_step": round(r["us_per_call"] / 1e3, 5), "us_per_call": r["us_per_call"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (scores), u32 keys (select)",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": r["workload"], "seq_len": r["seq_len"], "pages_per_rank": r["pages_per_rank"],
                   "seed": r["seed"], "l2": r["l2"], "parallelism": r["parallelism"]},
        "gpu_launches": r["steps"] * 3, "clocks": r["clocks"],
    }


def bench_ours(args, world, rank, local):
    """The headline line.  Every rank runs the same batch of the config
    (identical shapes and contents, in its own GPU's memory): weak scaling of
    replicated batches with no collective in the timed loop; value sums the
    ranks' algorithmic bytes over the max over ranks of the elapsed time.
    With config 1 (the default) the line also carries strong_config2 (config
    2's batch partitioned across the ranks), split_config3 (config 3's row
    split by page range) and, at N = 1, configs 2 and 4 on one GPU."""
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    seed = 100 * args.config
    base = W.config_inputs(args.config, seed=seed, device=dev)
    config_rps = base.rows_per_seq  # the kernel the committed ncu capture of this config measured
    if args.rows_per_seq:
        base.rows_per_seq = args.rows_per_seq
    R = base.rows_per_seq
    sets = rotating_sets(base)
    outs = [x.out() for x in sets]
    g_ids, g_logits = parity_guard(base)
    alg = base.algorithmic_bytes()
    sbytes = score_bytes(base)
    tokens = base.scored_tokens()
    ta = torch.tensor([alg, tokens], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ta, op=dist.ReduceOp.SUM)
    alg_total, tokens_total = float(ta[0].item()), float(ta[1].item())

    # (1) the timed region: K back-to-back calls, no events between them (the
    # two launches of consecutive calls overlap through programmatic
    # dependent launch).
    elapsed_max, clk = time_calls(sets, outs, R, args.steps, args.warmup, world, dev)
    ms_per_step = elapsed_max / args.steps
    value = alg_total * args.steps / (elapsed_max / 1e3) / 1e9
    # (2) per-kernel durations: the same calls with events around each launch
    n_ev = max(1, min(args.steps, 1000))
    score_ms, select_ms = kernel_times(sets, outs, R, n_ev)

    # ---- end to end through the public entry point, host buffers
    host = {k: getattr(base, k).cpu().pin_memory() for k in ("q", "k_cache", "weights", "seq_lens", "block_table")}
    devb = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    out_h = torch.empty((base.rows, 2048), dtype=torch.int32).pin_memory()
    out_d = base.out()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_h.numel() * 4
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def e2e_step():
        for k, v in host.items():
            devb[k].copy_(v, non_blocking=True)
        if R == 1:
            kernel(devb["q"], devb["k_cache"], devb["weights"], devb["seq_lens"], devb["block_table"], out_d)
        else:
            run(devb["q"], devb["k_cache"], devb["weights"], devb["seq_lens"], devb["block_table"], out_d,
                rows_per_seq=R)
        out_h.copy_(out_d, non_blocking=True)

    def timed_host_loop(fn, n):
        for _ in range(min(3, args.warmup)):
            fn()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(n):
            fn()
        f1.record()
        torch.cuda.synchronize()
        te = torch.tensor([f0.elapsed_time(f1)], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return float(te.item()) / n

    e2e_ms = timed_host_loop(e2e_step, e2e_steps)
    e2e_value = alg_total / (e2e_ms / 1e3) / 1e9

    # ---- a decode step with the index-K cache resident on the device: per
    # step the new token of every row (bf16 keys, slot ids), q, weights,
    # seq_lens and the block table cross PCIe, the writer stores the new keys
    # into their pages, the indexer runs, the ids come back
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import write_index_k
    kc_dev = base.k_cache.clone()
    new_k = torch.randn((base.rows, 128), dtype=torch.bfloat16).pin_memory()
    sl_h = base.seq_lens.cpu()
    last = (sl_h - 1).clamp_min(0).long()
    slot_h = (base.block_table.cpu()[torch.arange(base.rows), last // 64].long() * 64 + last % 64).to(torch.int32)
    host_d = {"q": host["q"], "weights": host["weights"], "seq_lens": host["seq_lens"],
              "block_table": host["block_table"], "new_k": new_k, "slots": slot_h.pin_memory()}
    dev_d = {k: torch.empty_like(v, device=dev) for k, v in host_d.items()}
    h2d_step = sum(v.numel() * v.element_size() for v in host_d.values())

    def decode_step():
        for k, v in host_d.items():
            dev_d[k].copy_(v, non_blocking=True)
        write_index_k(dev_d["new_k"], dev_d["slots"], kc_dev)
        if R == 1:
            kernel(dev_d["q"], kc_dev, dev_d["weights"], dev_d["seq_lens"], dev_d["block_table"], out_d)
        else:
            run(dev_d["q"], kc_dev, dev_d["weights"], dev_d["seq_lens"], dev_d["block_table"], out_d,
                rows_per_seq=R)
        out_h.copy_(out_d, non_blocking=True)

    dec_ms = timed_host_loop(decode_step, e2e_steps)
    del kc_dev, dev_d, devb

    # ---- the other shapes, in the same line (every rank takes the same
    # collective steps in the same order)
    strong = None
    split = None
    if args.config == 1 and not args.no_extras:
        strong = strong_config2(args, world, rank, local)
        split = split_config3(args, world, rank, local, steps=max(3, min(args.steps, 500)))
    extras = {}
    small = None
    if world == 1 and args.config == 1 and not args.no_extras:
        small = small_shape_latency(max(10, min(args.steps, 2000)), args.warmup, dev)
        for c in (2, 4):
            extras[f"config{c}"] = extra_config(c, max(3, min(args.steps, args.extra_steps)), args.warmup, dev,
                                                with_reference=not args.no_reference_kernel)

    if rank != 0:
        return None
    peak, peak_src = measured_hbm_peak()
    achieved = sbytes / (score_ms / 1e3) / 1e9
    kname = "score_kernel" if R == 1 else f"score_mq_kernel<{R}>"
    roof = {"kernel": kname, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
            "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "algorithmic_bytes_per_launch": sbytes, **traffic_entry(args.config, R, config_rps)}
    flops = score_flops(base)
    tpeak, tpeak_src = measured_fp8_peak()
    tensor = {"achieved": round(flops / (score_ms / 1e3) / 1e12, 1), "peak": round(tpeak, 1),
              "peak_source": tpeak_src, "unit": "TFLOP/s", "algorithmic_flops_per_launch": flops}
    tensor["frac"] = round(tensor["achieved"] / tpeak, 4)
    if flops / (tpeak * 1e12) > sbytes / (peak * 1e9):
        # the tensor pipe bounds this workload: report it as the roofline
        other = {k: roof[k] for k in ("achieved", "peak", "peak_source", "unit", "frac")}
        roof.update(bound="tensor", **{k: tensor[k] for k in ("achieved", "peak", "peak_source", "unit", "frac")})
        roof["algorithmic_flops_per_launch"] = flops
        roof["hbm"] = other
    else:
        roof["tensor"] = tensor
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "us_per_call": round(ms_per_step * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> f32 (scores), u32 keys (select)", "data": "synthetic (seeded, generated on device)",
        "config": {"workload": f"config{args.config}: {W.CONFIGS[args.config]}", "rows_per_gpu": base.rows,
                   "rows_per_seq": R,
                   "scored_tokens_per_gpu": tokens, "pool_pages": base.num_pages, "max_pages": base.max_pages,
                   "seed": seed, "l2": f"{N_SETS} rotating input copies of {base.k_cache.numel() / 1e6:.0f} MB K pool (> 126 MB L2)",
                   "parallelism": (f"replicated batches, dp{world}: every GPU runs the same batch, no collective "
                                   "in the timed loop; bytes summed over ranks" if world > 1 else "single GPU")},
        "tokens_per_s": round(tokens_total / (ms_per_step / 1e3), 1),
        "frac_of_hbm_peak": round(value / world / peak, 4),
        "frac_of_8tbs": round(value / world / 8000.0, 4),
        "kernels_ms": {"score": round(score_ms, 5), "select": round(select_ms, 5),
                       "timing": f"CUDA events around each launch over {n_ev} further calls"},
        "roofline": roof,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": ("kernel(...) drop-in" if R == 1 else f"run(..., rows_per_seq={R})") + ", pinned host inputs"},
        "e2e_decode_step": {"value": round(alg_total / (dec_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                            "us_per_step": round(dec_ms * 1e3, 2), "h2d_bytes_per_step": h2d_step, "d2h_bytes_per_step": d2h,
                            "path": "index-K cache resident on the device; per step the new token of every row "
                                    "(write_index_k), q, weights, seq_lens, block_table H2D, then the indexer, ids D2H"},
        "gpu_launches": 2 * args.steps,
        "clocks": clk,
    }
    if strong is not None:
        line["strong_config2"] = strong
    if split is not None:
        line["split_config3"] = split
    if extras:
        line["configs"] = extras
    if small is not None:
        line["small_shapes"] = small
    if world == 1 and R == 1 and not args.no_reference_kernel:
        line["reference_kernel"] = time_reference_kernel(sets, max(3, min(args.steps, 200)), args.warmup)
        line["reference_kernel_active"] = time_reference_kernel(sets, max(3, min(args.steps, 200)), args.warmup,
                                                                active=True)
    if world == 1 and not args.no_cpu_baseline:
        cpu, parity = cpu_leg(base, g_ids, g_logits, args.cpu_budget)
        line["cpu_baseline"] = cpu
        line["parity"] = parity
        if parity["failures"]:
            raise SystemExit(json.dumps({"error": "parity against the CPU oracle failed", "parity": parity}))
    else:
        line["parity"] = {"rows_checked": 0, "note": "oracle check runs on rank 0 at N = 1 (cpu_baseline leg)"}
    return line


def bench_reference(args, world, rank):
    """The reference arm: the CPU implementation of the path on the host
    cores.  The reference ships no CPU implementation of its own and its
    CUDA kernel is not a CPU path, so the arm times the torch formulation of
    the reference's operator (oracle/torch_path.py: e4m3 -> fp32 per page
    chunk, fp32 GEMM, ReLU * weights * scale, torch.topk, physical ids) with
    torch's whole thread pool, each step a bounded sample of whole rows of
    the same batch; the exact C oracle's rate is reported beside it."""
    if rank != 0:
        return None
    from oracle import oracle, torch_path
    seed = 100 * args.config
    inp = W.config_inputs(args.config, seed=seed, device="cpu")
    d = inp.numpy()
    tth = torch.get_num_threads()
    threads = os.cpu_count() or 1
    R = max(1, inp.rows_per_seq)

    def one(n):
        t0 = time.perf_counter()
        torch_path.indexer(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"], rows=range(n))
        return time.perf_counter() - t0

    budget = args.ref_step_budget
    t1 = one(R)
    n = int(max(R, min(inp.rows, budget / max(t1 / R, 1e-4))))
    n = max(R, n - n % R)  # whole groups of rows that share a sequence
    sub = W.Inputs(inp.q[:n], inp.k_cache, inp.weights[:n], inp.seq_lens[:n], inp.block_table[:n],
                   rows_per_seq=R)
    alg = sub.algorithmic_bytes()
    for _ in range(args.warmup):
        one(n)
    times = [one(n) for _ in range(args.steps)]
    step_s = statistics.mean(times)
    value = alg / step_s / 1e9
    t0 = time.perf_counter()
    lg = oracle.logits(d["q"][:n], d["k_cache"], d["weights"][:n], d["seq_lens"][:n], d["block_table"][:n],
                       num_pages=d["num_pages"], nthreads=threads)
    oracle.topk(lg, d["seq_lens"][:n], d["block_table"][:n])
    t_or = time.perf_counter() - t0
    sample = (f"first {n} of {inp.rows} rows of config{args.config} per step, torch CPU formulation "
              f"(torch.get_num_threads()={tth} of {threads} host CPUs)")
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 -> f32 GEMM (torch CPU), f32 top-k", "data": "synthetic (seeded)",
        "config": {"workload": f"config{args.config}: {W.CONFIGS[args.config]}", "rows_sampled": n, "seed": seed},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": tth, "kind": "port", "sample": sample,
                         "c_oracle": {"value": round(alg / t_or / 1e9, 4), "unit": "GB/s", "cores": threads,
                                      "sample": f"the same {n} rows, exact fp64 C oracle, {t_or:.2f} s"}},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def bench_writer(args, world, rank, local):
    """The index-K cache writer (dsai_write_k via write_index_k): n new bf16
    keys quantised to e4m3 and scattered to shuffled physical slots of a pool
    1.1x their size.  Algorithmic bytes per call: n x (256 B of bf16 keys +
    4 B of slot id + 132 B of e4m3 row and scale).  Three rotating input
    sets keep L2 from holding a previous call's data."""
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import write_index_k
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = args.tokens
    pages = (n * 11 // 10 + 63) // 64
    g = torch.Generator(device="cpu").manual_seed(7)
    sets = []
    for _ in range(N_SETS):
        k = torch.randn((n, 128), generator=g).to(torch.bfloat16).to(dev)
        ids = torch.randperm(pages * 64, generator=g)[:n].to(torch.int32).to(dev)
        pool = torch.zeros((pages, 64, 1, 132), dtype=torch.uint8, device=dev)
        sets.append((k, ids, pool))
    alg = n * (256 + 4 + 132)
    for i in range(args.warmup):
        write_index_k(*sets[i % N_SETS])
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        write_index_k(*sets[i % N_SETS])
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    gbs = alg / (ms / 1e3) / 1e9
    peak, peak_src = measured_hbm_peak()
    line = {
        "metric": "index-K cache writer GB/s (bf16 keys -> e4m3 pages + fp32 scales)", "value": round(gbs, 1),
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "us_per_call": round(ms * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 -> e4m3 (fp32 scale)",
        "data": "synthetic (seeded N(0,1) keys, shuffled slots)",
        "config": {"workload": f"write_k: {n} new tokens into a {pages}-page pool",
                   "l2": f"{N_SETS} rotating input sets of {(n * 392 + pages * 8448) / 1e6:.0f} MB"},
        "roofline": {"kernel": "write_k_kernel", "bound": "hbm", "achieved": round(gbs, 1), "peak": peak,
                     "peak_source": peak_src, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "algorithmic_bytes_per_launch": alg, "traffic": None},
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        from oracle import oracle as O
        k, ids, pool = sets[0]
        m = min(n, 16384)
        kc = k[:m].float().cpu().numpy()
        idc = ids[:m].cpu().numpy()
        cache = np.zeros(pages * 8448, np.uint8)
        t0 = time.perf_counter()
        O.write_k(kc, idc, cache, pages)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(m * 392 / dt / 1e9, 4), "unit": "GB/s", "cores": 1,
                                "kind": "port", "sample": f"first {m} of {n} tokens, C oracle writer, {dt:.3f} s"}
    return line


def bench_graph(args, world, rank, local):
    """Small-batch latency: the drop-in kernel(...) called eagerly against
    the same call captured once (IndexerGraph) and replayed, both timed over
    K back-to-back calls with CUDA events.  Workload: benchmark config 0
    (B=2, seq_lens {1500, 4096}, 64 pages per row), where per-call host work
    dominates."""
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import IndexerGraph
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = W.config_inputs(0, device=dev)
    out = g.out()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps * 1e3

    eager_us = timed(lambda: kernel(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out))
    graph = IndexerGraph(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out)
    clocks = ClockSampler(dev)
    clocks.start()
    graph_us = timed(graph.replay)
    clk = clocks.stop()
    return {
        "metric": "us per indexer call, config 0 (B=2), CUDA-graph replay", "value": round(graph_us, 2),
        "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(graph_us / 1e3, 5), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (scores), u32 keys (select)",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": f"config0: {W.CONFIGS[0]}", "rows": g.rows, "max_pages": g.max_pages},
        "eager_us_per_call": round(eager_us, 2),
        "gpu_launches": 2 * args.steps,
        "clocks": clk,
    }


def bench_attn(args, world, rank, local):
    """Sparse MLA attention over top-2048 slots (the indexer's consumer):
    --tokens-attn decode tokens, each over 2048 random slots of its own
    4096-slot (64-page) range of a bf16 ckv/kpe pool (295 MB at 64 tokens,
    larger than L2), two rotating index sets.  value = algorithmic bytes
    (2048 x 1152 B of gathered rows + q, indices, output, lse per token) per
    second over K back-to-back calls."""
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import sparse_attention
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T = args.tokens_attn
    pages = 64 * T
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    qn = torch.randn((T, 16, 512), generator=g, device=dev).to(torch.bfloat16)
    qp = torch.randn((T, 16, 64), generator=g, device=dev).to(torch.bfloat16)
    ckv = torch.randn((pages, 64, 512), generator=g, device=dev).to(torch.bfloat16)
    kpe = torch.randn((pages, 64, 64), generator=g, device=dev).to(torch.bfloat16)
    base = (torch.arange(T, device=dev, dtype=torch.int32) * 4096)[:, None]
    idx_sets = [(torch.argsort(torch.rand((T, 4096), generator=g, device=dev), dim=1)[:, :2048].to(torch.int32) + base)
                .contiguous() for _ in range(2)]
    out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, 16), dtype=torch.float32, device=dev)
    scale = 1.0 / math.sqrt(192.0)
    alg = T * (2048 * (1024 + 128) + 16 * 576 * 2 + 2048 * 4 + 16 * 512 * 2 + 16 * 4)
    flops = T * 16 * 2048 * (576 + 512) * 2

    def step(i):
        sparse_attention(qn, qp, ckv, kpe, idx_sets[i % 2], scale, out, lse)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    e0.record()
    for i in range(args.steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    us = e0.elapsed_time(e1) / args.steps * 1e3
    peak, peak_src = measured_hbm_peak()
    gbs = alg / (us / 1e6) / 1e9
    line = {
        "metric": f"sparse MLA attention GB/s (T={T} decode tokens x 2048 slots, h16 ckv512 kpe64)",
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(us / 1e3, 5), "us_per_call": round(us, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 x bf16 -> f32 (tcgen05), bf16 out",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": f"attn: {T} tokens, 2048 of 4096 own slots each, {pages}-page bf16 pool",
                   "l2": f"pool {(ckv.numel() + kpe.numel()) * 2 / 1e6:.0f} MB (> 126 MB L2), 2 rotating index sets"},
        "roofline": {"kernel": "attn_kernel (+ attn_combine_kernel)", "bound": "hbm", "achieved": round(gbs, 1),
                     "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "algorithmic_bytes_per_launch": alg,
                     "traffic": None,
                     "traffic_last_profiled": 152_770_560 + 4_194_048 if T == 64 else None,
                     "traffic_source": "ncu capture of an earlier build of attn_kernel (T=64), not of this run",
                     "tensor": {"achieved": round(flops / (us / 1e6) / 1e12, 1), "unit": "TFLOP/s",
                                "algorithmic_flops_per_launch": flops}},
        "gpu_launches": 2 * args.steps,
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        from oracle import oracle  # CPU baseline leg only
        n = 4
        t0 = time.perf_counter()
        oracle.sparse_attention(qn[:n].float().cpu().numpy(), qp[:n].float().cpu().numpy(),
                                ckv.float().cpu().numpy(), kpe.float().cpu().numpy(),
                                idx_sets[0][:n].cpu().numpy(), scale)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(alg / T * n / dt / 1e9, 4), "unit": "GB/s", "cores": os.cpu_count() or 1,
                                "kind": "port", "sample": f"{n} of {T} tokens (numpy fp64 oracle), {dt:.2f} s"}
    return line


def bench_prefill(args, world, rank, local):
    """A prefill chunk: `--chunk` causal query rows of one sequence whose
    last row sees `--last-len` tokens, all over the sequence's block table.
    Timed in groups of 4 rows (rows_per_seq=4: each K tile staged once per
    group) and row by row, each call bracketed by CUDA events, with L2
    flushed (a 256 MB write) before every call since the chunk's K pages
    (~8.6 MB for 64K tokens) would otherwise stay in L2."""
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = W.prefill_inputs(args.chunk, args.last_len, device=dev)
    out = g.out()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    token_rows = int(g.seq_lens.to(torch.int64).sum().item())
    alg = g.algorithmic_bytes()  # K once per chunk would be the floor; counted per group of 4 here

    def timed(rps):
        for _ in range(args.warmup):
            run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, rows_per_seq=rps)
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(args.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, rows_per_seq=rps)
            e1.record()
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        return total / args.steps * 1e3

    clocks = ClockSampler(dev)
    clocks.start()
    us4 = timed(4)
    clk = clocks.stop()
    us1 = timed(1)
    return {
        "metric": f"us per prefill-chunk indexer call ({args.chunk} causal rows, last row {args.last_len} tokens)",
        "value": round(us4, 2), "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(us4 / 1e3, 5), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> f32 (scores), u32 keys (select)", "data": "synthetic (seeded, generated on device)",
        "config": {"workload": g.name, "rows": g.rows, "rows_per_seq": 4, "max_pages": g.max_pages,
                   "l2": "256 MB write before every timed call"},
        "token_rows_per_s": round(token_rows / (us4 / 1e6), 1),
        "algorithmic_bytes": alg,
        "row_by_row_us": round(us1, 2),
        "gpu_launches": 2 * args.steps,
        "clocks": clk,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4])
    ap.add_argument("--rows-per-seq", type=int, default=0,
                    help="override the config's rows per sequence (1 scores config 4 row by row)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of torch CPU work for cpu_baseline")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the strong_config2 / split_config3 / configs keys of the default line")
    ap.add_argument("--extra-steps", type=int, default=100, help="timed calls of each extra config")
    ap.add_argument("--strong-steps", type=int, default=100, help="timed calls of strong_config2")
    ap.add_argument("--ref-step-budget", type=float, default=2.0, help="seconds per reference-arm step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-kernel", action="store_true",
                    help="skip timing the reference's own CUDA kernel (reference_kernel key)")
    ap.add_argument("--chunk", type=int, default=256, help="--op prefill: query rows of the chunk")
    ap.add_argument("--last-len", type=int, default=65536, help="--op prefill: tokens the last row sees")
    ap.add_argument("--tokens-attn", type=int, default=64, help="--op attn: decode tokens per call")
    ap.add_argument("--op", default="indexer", choices=["indexer", "write_k", "graph", "prefill", "attn"],
                    help="write_k: the index-K cache writer; graph: small-batch latency, eager vs CUDA graph")
    ap.add_argument("--tokens", type=int, default=131072, help="new tokens per write_k call")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    try:
        if args.op == "write_k":
            line = bench_writer(args, world, rank, local) if rank == 0 else None
        elif args.op == "graph":
            line = bench_graph(args, world, rank, local) if rank == 0 else None
        elif args.op == "prefill":
            line = bench_prefill(args, world, rank, local) if rank == 0 else None
        elif args.op == "attn":
            line = bench_attn(args, world, rank, local) if rank == 0 else None
        elif args.impl == "reference":
            line = bench_reference(args, world, rank)
        elif args.config == 3:
            line = bench_split(args, world, rank, local)
        else:
            line = bench_ours(args, world, rank, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
