#!/usr/bin/env python3
"""Throughput of the sm_100a sampling path on the headline workload.

One step = one batched TokenSampler.SampleNext over a [256, 128256] fp32 logits
batch (Zipf-ranked logits, 1024-id histories, repetition 1.15, T 0.7, top-k 50,
top-p 0.9), i.e. the C ABI call ncb_sample_rows_device on device-resident inputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N>1 runs under torch.distributed (one process per GPU, NCCL for the barrier and
the max-over-ranks timing only): every rank samples its own batch (rows shard
across GPUs with no data-path exchange), so scaling is weak.
--impl reference times the reference's CPU sampler on the host: the C# code
cannot run here (no .NET runtime), so its C restatement (oracle/) stands in.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/sec at B×V=256×128256 fp32; achieved HBM GB/s vs B200 peak"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0
NBUF = 4  # input copies rotated across steps: 4 x 132 MB > 126 MB L2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload():
    from neuraval_b200 import workloads
    return workloads.zipf_ranked()


def config_of(wl, extra=None):
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    c = {"workload": wl["name"], "B": B, "V": V, "history_per_row": H,
         "top_k": wl["params"]["top_k"], "top_p": wl["params"]["top_p"],
         "temperature": wl["params"]["temperature"],
         "repetition_penalty": wl["params"]["repetition_penalty"],
         "uniforms": "one seeded u in [0,1) per row",
         "l2": f"inputs larger than L2: {NBUF} copies of the batch rotated across steps"}
    if extra:
        c.update(extra)
    return c


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """DRAM bytes (read + write) per launch of the top-k kernel, from the committed
    ncu summary of this workload (its `dram_bytes_per_launch:` line)."""
    path = os.path.join(ROOT, "profiles", "topk_ldg_kernel_zipf_ranked_256x128256.md")
    try:
        with open(path) as fh:
            for line in fh:
                m = re.match(r"\s*-?\s*`?dram_bytes_per_launch`?:\s*([0-9]+)", line)
                if m:
                    return int(m.group(1))
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons, self.ok = [], 0, False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.005)

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
        except Exception:
            pass

    def __enter__(self):
        if self.ok:
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()
            self._sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def cpu_baseline(wl, seconds):
    """The oracle (C restatement of the C# sampler) on all host cores over a
    bounded sample of the same workload; returns (rows/s, threads, sample desc, 1-thread rows/s)."""
    from oracle import pyoracle
    pyoracle.build()
    threads = os.cpu_count() or 1
    p = pyoracle.make_params(**wl["params"])
    offs = np.asarray(wl["hist_offsets"], np.int64)
    B = wl["logits"].shape[0]
    # single thread on 16 rows
    sub = 16
    t0 = time.perf_counter()
    pyoracle.sample_rows(wl["logits"][:sub], wl["hist_ids"][: offs[sub]], offs[: sub + 1],
                         wl["uniforms"][:sub], p, exp_mode=pyoracle.EXP_GLIBC, threads=1)
    one = sub / (time.perf_counter() - t0)
    rows = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds and rows < 2000 * B:
        pyoracle.sample_rows(wl["logits"], wl["hist_ids"], offs, wl["uniforms"], p,
                             exp_mode=pyoracle.EXP_GLIBC, threads=threads)
        rows += B
    dt = time.perf_counter() - t0
    return rows / dt, threads, f"{rows} rows ({rows // B} full batches of {B}) in {dt:.1f} s", one


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    wl = workload()
    from oracle import pyoracle
    pyoracle.build()
    threads = os.cpu_count() or 1
    p = pyoracle.make_params(**wl["params"])
    offs = np.asarray(wl["hist_offsets"], np.int64)
    B = wl["logits"].shape[0]
    rows_per_step = min(B, 8 * threads)  # bounded sample per step
    lg = wl["logits"][:rows_per_step]
    h = wl["hist_ids"][: offs[rows_per_step]]
    o = offs[: rows_per_step + 1]
    u = wl["uniforms"][:rows_per_step]
    for _ in range(args.warmup):
        pyoracle.sample_rows(lg, h, o, u, p, exp_mode=pyoracle.EXP_GLIBC, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pyoracle.sample_rows(lg, h, o, u, p, exp_mode=pyoracle.EXP_GLIBC, threads=threads)
    dt = time.perf_counter() - t0
    value = rows_per_step * args.steps / dt
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic", "config": config_of(wl, {"rows_per_step": rows_per_step}),
           "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": f"{rows_per_step} rows of the batch per step, {args.steps} steps; "
                                      "C restatement of TokenSampler.SampleFiltered (libm expf); "
                                      "the C# original needs a .NET runtime, absent here"},
           "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    from neuraval_b200 import native, workloads
    from neuraval_b200.sampler import CudaTokenSampler

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    wl = workload()
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    params = native.make_params(**wl["params"])
    sampler = CudaTokenSampler(device=local, max_rows=B, max_vocab=V, max_history=H)

    bufs = []
    for i in range(NBUF):
        lg = torch.from_numpy(wl["logits"]).to(dev)
        if i:
            lg = lg.roll(i, dims=0)  # distinct copies, same workload
        bufs.append(lg.contiguous())
    hist = torch.from_numpy(wl["hist_ids"]).to(dev)
    offs = torch.from_numpy(wl["hist_offsets"]).to(dev)
    u = torch.from_numpy(wl["uniforms"]).to(dev)
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    flags = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i, stream):
        sampler.sample_rows_device(bufs[i % NBUF], hist, offs, u, params, tokens, flags,
                                   None, stream)

    cur = torch.cuda.current_stream(dev)
    for i in range(max(3, args.warmup)):
        step(i, cur)
    torch.cuda.synchronize()

    # eager launches (each call goes through ctypes): reported for reference
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for i in range(args.steps):
        step(i, cur)
    e1.record(cur)
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1)

    # timed region: the K steps captured once in a CUDA graph and replayed, so the
    # device timeline holds only the sampling kernels (no host launch gaps)
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(cur)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for i in range(args.steps):
                step(i, torch.cuda.current_stream(dev))
    torch.cuda.synchronize()
    graph.replay()  # one untimed replay
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    with clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(cur)
        graph.replay()
        t_end.record(cur)
        torch.cuda.synchronize()
    total_ms = t_start.elapsed_time(t_end)
    per_launch_ms = total_ms / args.steps
    if world > 1:
        t = torch.tensor([total_ms, per_launch_ms, eager_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms, per_launch_ms, eager_ms = float(t[0]), float(t[1]), float(t[2])
    value = world * B * args.steps / (total_ms / 1e3)
    del graph

    # end to end through the host-array entry point (pinned host buffers)
    e2e = None
    if args.e2e_steps > 0:
        h_logits = torch.from_numpy(wl["logits"]).pin_memory().numpy()
        h_hist = torch.from_numpy(wl["hist_ids"]).pin_memory().numpy()
        h_offs = torch.from_numpy(wl["hist_offsets"]).pin_memory().numpy()
        h_u = torch.from_numpy(wl["uniforms"]).pin_memory().numpy()
        for _ in range(2):
            sampler.sample_rows(h_logits, h_hist, h_offs, h_u, params)
        if world > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            sampler.sample_rows(h_logits, h_hist, h_offs, h_u, params)
        e2e_s = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_s = float(t[0])
        e2e = {"value": world * B * args.e2e_steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": int(h_logits.nbytes + h_hist.nbytes + h_offs.nbytes +
                                         h_u.nbytes),
               "d2h_bytes_per_step": int(B * 4 * 2),
               "api": "ncb_sample_rows (host arrays; copies in, samples, synchronises, "
                      "copies out)"}

    if rank == 0:
        peak, peak_kind = measured_peak()
        bytes_per_launch = B * workloads.bytes_per_row(V, H)
        achieved = bytes_per_launch / (per_launch_ms / 1e3) / 1e9
        out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
               "dtype": "fp32", "data": "synthetic (seeded generator, no dataset)",
               "config": config_of(wl, {"parallelism": f"rows sharded, {world} GPU(s), no exchange"}),
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "peak_source": peak_kind,
                            "traffic": profiled_traffic(),
                            "kernel": "topk_ldg_kernel (+ its fix-up launch, timed together)",
                            "algorithmic_bytes_per_launch": bytes_per_launch},
               "e2e": e2e,
               "gpu_launches": 2 * args.steps,
               "eager_value": world * B * args.steps / (eager_ms / 1e3),
               "timing": "CUDA events around one replay of a CUDA graph holding the K steps",
               "clocks": clocks.summary()}
        if world == 1 and args.cpu_seconds > 0:
            v, cores, sample, one = cpu_baseline(wl, args.cpu_seconds)
            out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                   "sample": sample, "single_thread_value": one}
        print(json.dumps(out), flush=True)
    sampler.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
