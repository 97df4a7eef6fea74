#!/usr/bin/env python3
"""Throughput of the sm_100a sampling path on the headline workload.

One step = one batched TokenSampler.SampleNext over a [256, 128256] fp32 logits
batch (Zipf-ranked logits, 1024-id histories, repetition 1.15, T 0.7, top-k 50,
top-p 0.9), i.e. the C ABI call ncb_sample_rows_device on device-resident inputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload zipf_ranked|vocab_sharded|softmax_rows] [--exchange nccl|peer]

N>1 runs under torch.distributed (one process per GPU, NCCL for the barrier and
the max-over-ranks timing only): every rank samples its own batch (rows shard
across GPUs with no data-path exchange), so scaling is weak.
--impl reference times the reference's CPU sampler on the host: the C# code
cannot run here (no .NET runtime), so its C restatement (oracle/) stands in.
Other workloads: vocab_sharded (the 128 x 262144 batch with its vocabulary split
over the GPUs, strong scaling) and softmax_rows (the row softmax of the 256 x
128256 batch; its reference arm is the reference's own CUDA kernel).
"""
from __future__ import annotations

import argparse
import contextlib
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
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--exchange", default="nccl", choices=["nccl", "peer"],
                    help="vocab_sharded: records exchanged by an NCCL all-gather, or through "
                         "peer memory by the shard kernel itself")
    ap.add_argument("--workload", default="zipf_ranked",
                    choices=["zipf_ranked", "peaked_head", "zipf_history_nucleus",
                             "high_entropy_nucleus", "vocab_sharded", "softmax_rows"],
                    help="zipf_ranked: the headline (rows shard over GPUs); vocab_sharded: "
                         "128 x 262144, vocabulary split over GPUs; softmax_rows: row softmax "
                         "of the 256 x 128256 logits batch")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload(rank=0, name="zipf_ranked"):
    """The batch of a sampling workload (the headline by default); rank r > 0 of
    a multi-GPU run gets its own rows (same generator, another seed)."""
    from neuraval_b200 import workloads
    gen = workloads.WORKLOADS[name]
    return gen() if rank == 0 else gen(seed=1000 * rank + 7)


def config_of(wl, extra=None):
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    c = {"workload": wl["name"], "B": B, "V": V, "history_per_row": H,
         **{k: v for k, v in wl["params"].items()},
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
    # single thread on up to 16 rows
    sub = min(16, B)
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


def kernels_of(params, V):
    """The kernels one sampling call launches for these parameters (the
    dispatch of ncb_sample_rows_device): a name for the timed pair and the
    number of launches per step."""
    k = params.get("top_k", 0) or 0
    if params.get("greedy"):
        return "greedy_kernel", 1
    if 0 < k < V and k <= 64:
        return "topk_ldg_kernel (+ its fix-up launch, timed together)", 2
    if 0 < k < V and k <= 1024:
        return "topk_kernel (+ its fix-up launch, timed together)", 2
    return "nucleus_kernel (+ its full-sort fix-up launch, timed together)", 2


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    if args.workload == "softmax_rows":
        return run_softmax_reference(args)
    wl = workload(0, args.workload)
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

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    try:
        if args.workload == "vocab_sharded":
            out = run_vocab_sharded(args, rank, world, dev)
        elif args.workload == "softmax_rows":
            out = run_softmax(args, rank, world, dev)
        else:
            out = run_rows(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
    return 0


def run_rows(args, rank, world, dev):
    """The headline: every rank samples its own 256-row batch (rows shard with
    no exchange), timed as one replay of a CUDA graph holding the K steps."""
    import torch
    from neuraval_b200 import native, sharding, workloads
    from neuraval_b200.sampler import CudaTokenSampler

    wl = workload(rank, args.workload)
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    params = native.make_params(**wl["params"])
    sampler = CudaTokenSampler(device=dev.index, max_rows=B, max_vocab=V, max_history=H)
    nbuf = max(NBUF, -(-2 * L2_BYTES // max(1, B * V * 4)))  # rotated copies span 2 x L2

    bufs = []
    for i in range(nbuf):
        lg = torch.from_numpy(wl["logits"]).to(dev)
        if i:
            lg = lg.roll(i, dims=0) if B > 1 else lg.roll(i * 97, dims=1)  # distinct copies
        bufs.append(lg.contiguous())
    hist = torch.from_numpy(wl["hist_ids"]).to(dev)
    offs = torch.from_numpy(wl["hist_offsets"]).to(dev)
    u = torch.from_numpy(wl["uniforms"]).to(dev)
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    flags = torch.empty(B, dtype=torch.int32, device=dev)

    def step(i, stream):
        sampler.sample_rows_device(bufs[i % nbuf], hist, offs, u, params, tokens, flags,
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
    clocks = ClockSampler(dev.index)
    with clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(cur)
        graph.replay()
        t_end.record(cur)
        torch.cuda.synchronize()
    total_ms, eager_ms = sharding.max_over_ranks([t_start.elapsed_time(t_end), eager_ms], dev)
    per_launch_ms = total_ms / args.steps
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
        (e2e_s,) = sharding.max_over_ranks([time.perf_counter() - t0], dev)
        e2e = {"value": world * B * args.e2e_steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": int(h_logits.nbytes + h_hist.nbytes + h_offs.nbytes +
                                         h_u.nbytes),
               "d2h_bytes_per_step": int(B * 4 * 2),
               "api": "ncb_sample_rows (host arrays; copies in, samples, synchronises, "
                      "copies out)"}

    out = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        bytes_per_launch = B * workloads.bytes_per_row(V, H)
        achieved = bytes_per_launch / (per_launch_ms / 1e3) / 1e9
        kernel, launches = kernels_of(wl["params"], V)
        out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
               "dtype": "fp32", "data": "synthetic (seeded generator, no dataset)",
               "config": config_of(wl, {"parallelism": f"rows sharded, {world} GPU(s) x {B} rows"
                                                       ", no exchange",
                                        "l2": f"inputs larger than L2: {nbuf} copies of the "
                                              "batch rotated across steps"}),
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "peak_source": peak_kind,
                            "traffic": profiled_traffic() if wl["name"].startswith("zipf_ranked")
                            else None,
                            "kernel": kernel,
                            "algorithmic_bytes_per_launch": bytes_per_launch},
               "e2e": e2e,
               "gpu_launches": launches * args.steps,
               "eager_value": world * B * args.steps / (eager_ms / 1e3),
               "timing": "CUDA events around one replay of a CUDA graph holding the K steps; "
                         "max over ranks",
               "clocks": clocks.summary()}
        if world == 1 and args.cpu_seconds > 0:
            v, cores, sample, one = cpu_baseline(wl, args.cpu_seconds)
            out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                   "sample": sample, "single_thread_value": one}
    sampler.close()
    return out


def run_vocab_sharded(args, rank, world, dev):
    """The 128 x 262144 batch (top-k 64) with its vocabulary split over the ranks:
    per step, the shard candidate kernel, one NCCL all-gather of the records and
    the merge kernel on every rank. Total work is fixed (strong scaling). The
    K steps are captured in one CUDA graph (the all-gather included) and
    replayed; each part is also timed alone the same way."""
    import torch
    from neuraval_b200 import native, sharding, workloads
    from neuraval_b200.sampler import CudaTokenSampler

    wl = workloads.vocab_sharded()
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    params = native.make_params(**wl["params"])
    lo, hi = sharding.vocab_range(V, world, rank)
    width = hi - lo
    sampler = CudaTokenSampler(device=dev.index, max_rows=B, max_vocab=max(width, 1),
                               max_history=H)
    shard = torch.from_numpy(np.ascontiguousarray(wl["logits"][:, lo:hi]))
    # rotated copies of the shard: a copy is read again only after twice the L2
    # capacity has streamed through
    nbuf = min(32, max(2, -(-2 * L2_BYTES // max(1, B * width * 4))))
    bufs = [shard.to(dev).roll(i, dims=0).contiguous() for i in range(nbuf)]
    hist = torch.from_numpy(wl["hist_ids"]).to(dev)
    offs = torch.from_numpy(wl["hist_offsets"]).to(dev)
    u = torch.from_numpy(wl["uniforms"]).to(dev)
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    flags = torch.empty(B, dtype=torch.int32, device=dev)
    words = sampler.shard_record_bytes // 4
    local = torch.zeros((B, words), dtype=torch.int32, device=dev)
    gathered = torch.zeros((world, B, words), dtype=torch.int32, device=dev)
    peer = sharding.PeerVocabShardedSampler(sampler, V) if args.exchange == "peer" else None

    def candidates(i):
        sampler.shard_candidates_device(bufs[i % nbuf], V, lo, hist, offs, params, local,
                                        torch.cuda.current_stream(dev))

    def exchange(i):
        if world > 1:
            torch.distributed.all_gather_into_tensor(gathered, local)
        else:
            gathered[0].copy_(local)

    def merge(i):
        if peer is not None:
            sampler.shard_merge_peer_device(B, V, u, params, tokens, flags,
                                            torch.cuda.current_stream(dev))
        else:
            sampler.shard_merge_device(gathered, world, B, V, u, params, tokens, flags,
                                       torch.cuda.current_stream(dev))

    def full(i):
        if peer is not None:
            peer.sample(bufs[i % nbuf], hist, offs, u, params, tokens, flags,
                        torch.cuda.current_stream(dev))
        else:
            candidates(i)
            exchange(i)
            merge(i)

    cur = torch.cuda.current_stream(dev)
    for i in range(max(3, args.warmup)):
        full(i)
    torch.cuda.synchronize()

    def timed(fn, clocks=None):
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(cur)
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                for i in range(args.steps):
                    fn(i)
        torch.cuda.synchronize()
        graph.replay()  # one untimed replay
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (clocks if clocks is not None else contextlib.nullcontext()):
            t0.record(cur)
            graph.replay()
            t1.record(cur)
            torch.cuda.synchronize()
        del graph  # graphs holding NCCL calls go before the process group
        return t0.elapsed_time(t1)

    clocks = ClockSampler(dev.index)
    total_ms = timed(full, clocks)
    if peer is not None:
        # a merge alone re-reads the last call's records (its flags are already set)
        parts = [timed(candidates), 0.0, timed(merge)]
        parts[1] = max(0.0, total_ms - parts[0] - parts[2])
    else:
        parts = [timed(candidates), timed(exchange), timed(merge)]
    total_ms, *parts = sharding.max_over_ranks([total_ms] + parts, dev)
    # the sampled tokens equal the single-GPU sampler's on the whole rows
    ok = True
    full(0)  # every rank: the step holds a collective
    torch.cuda.synchronize()
    if rank == 0:
        ref_s = CudaTokenSampler(device=dev.index, max_rows=B, max_vocab=V, max_history=H)
        full_logits = torch.from_numpy(wl["logits"]).to(dev)
        rt = torch.empty_like(tokens)
        rf = torch.empty_like(flags)
        ref_s.sample_rows_device(full_logits, hist, offs, u, params, rt, rf)
        torch.cuda.synchronize()
        ok = bool(torch.equal(rt, tokens) and torch.equal(rf, flags))
        ref_s.close()
        del full_logits
    out = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        per_gpu_bytes = B * (4 * width + 4 * H + 8)
        per_step_s = total_ms / args.steps / 1e3
        out = {"metric": "sampled rows/sec, vocabulary split over GPUs", "value":
               B * args.steps / (total_ms / 1e3), "unit": UNIT, "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
               "dtype": "fp32", "data": "synthetic (seeded generator, no dataset)",
               "config": config_of(wl, {"parallelism": f"vocabulary sharded over {world} GPU(s);"
                                                       f" {args.exchange} record exchange",
                                        "l2": f"{nbuf} rotated copies of each shard",
                                        "shard_columns": width,
                                        "record_bytes_per_rank": B * sampler.shard_record_bytes}),
               "parts_us_per_step": {"candidates": parts[0] / args.steps * 1e3,
                                     "exchange": parts[1] / args.steps * 1e3,
                                     "merge": parts[2] / args.steps * 1e3},
               "exchange": ("records stored into every GPU's exchange area over NVLink by the "
                            "library (epoch flags and acks)" if peer is not None else
                            "NCCL all-gather of the records"),
               "tokens_match_single_gpu": ok,
               "roofline": {"bound": "hbm", "achieved": per_gpu_bytes / per_step_s / 1e9,
                            "peak": peak, "unit": "GB/s",
                            "frac": per_gpu_bytes / per_step_s / 1e9 / peak,
                            "peak_source": peak_kind, "traffic": None,
                            "kernel": "shard candidate kernel + all-gather + merge, per step",
                            "algorithmic_bytes_per_launch": per_gpu_bytes},
               "e2e": None,
               "gpu_launches": (3 if peer is not None else 2) * args.steps,
               "timing": "CUDA events around one replay of a CUDA graph holding the K steps "
                         "(all-gather included); max over ranks",
               "clocks": clocks.summary()}
    sampler.close()
    return out


SOFTMAX_METRIC = "softmax rows/sec at B×V=256×128256 fp32"


def _softmax_inputs(dev):
    import torch
    from neuraval_b200 import workloads
    wl = workloads.zipf_ranked(H=1)
    x = torch.from_numpy(wl["logits"]).to(dev)
    bufs = [x] + [x.roll(i, dims=0).contiguous() for i in range(1, NBUF)]
    return wl, bufs, torch.empty_like(x)


def run_softmax(args, rank, world, dev):
    """F-row: ncb_softmax_rows_device on the 256 x 128256 batch; each rank its own
    copy (weak scaling), K launches in one CUDA graph."""
    import ctypes
    import torch
    from neuraval_b200 import native, sharding
    lib = native.load()
    wl, bufs, out = _softmax_inputs(dev)
    B, V = wl["logits"].shape

    def step(i):
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        rc = lib.ncb_softmax_rows_device(ctypes.c_void_p(bufs[i % NBUF].data_ptr()),
                                         ctypes.c_void_p(out.data_ptr()), B, V, st)
        assert rc == 0, rc

    cur = torch.cuda.current_stream(dev)
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(cur)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for i in range(args.steps):
                step(i)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = ClockSampler(dev.index)
    with clocks:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(cur)
        graph.replay()
        t1.record(cur)
        torch.cuda.synchronize()
    (total_ms,) = sharding.max_over_ranks([t0.elapsed_time(t1)], dev)
    del graph
    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    per_launch_s = total_ms / args.steps / 1e3
    alg = B * V * 8  # read the row once, write it once
    return {"metric": SOFTMAX_METRIC, "value": world * B * args.steps / (total_ms / 1e3),
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded generator, no dataset)",
            "config": {"workload": "softmax_rows_256x128256", "B": B, "V": V,
                       "l2": f"inputs larger than L2: {NBUF} copies rotated across steps",
                       "parallelism": f"each of {world} GPU(s) its own batch"},
            "roofline": {"bound": "hbm", "achieved": alg / per_launch_s / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": alg / per_launch_s / 1e9 / peak,
                         "peak_source": peak_kind, "traffic": None,
                         "kernel": "softmax_rows_kernel",
                         "algorithmic_bytes_per_launch": alg,
                         "design_bytes_per_launch": B * V * 16},
            "e2e": None, "gpu_launches": args.steps,
            "timing": "CUDA events around one replay of a CUDA graph holding the K launches",
            "clocks": clocks.summary()}


def run_softmax_reference(args):
    """The reference's own kernel (ncb_cuda_softmax_rows_device from its
    navcuda.cu, compiled for sm_100a into oracle/_ref) on the same batch; it
    launches on the legacy default stream, so it is timed eagerly."""
    import ctypes
    import torch
    from oracle import refcuda
    if not refcuda.available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libnavcuda.so not built (needs the reference source)"}))
        return 0
    lib = refcuda.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    assert lib.ncb_cuda_init(0) == 1
    wl, bufs, out = _softmax_inputs(dev)
    B, V = wl["logits"].shape
    step = lambda i: lib.ncb_cuda_softmax_rows_device(ctypes.c_void_p(bufs[i % NBUF].data_ptr()),
                                                      ctypes.c_void_p(out.data_ptr()), B, V)
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    value = B * args.steps / (ms / 1e3)
    print(json.dumps({"impl": "reference", "metric": SOFTMAX_METRIC, "value": value, "unit": UNIT,
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": ms / args.steps, "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
                      "data": "synthetic", "config": {"workload": "softmax_rows_256x128256"},
                      "cpu_baseline": {"value": value, "unit": UNIT, "cores": 0,
                                       "kind": "reference",
                                       "sample": "the reference's CUDA kernel, every launch on "
                                                 "the GPU (its own implementation of this op)"},
                      "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
