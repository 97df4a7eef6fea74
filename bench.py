#!/usr/bin/env python3
"""Throughput of the sm_100a sampling path on the headline workload.

One step = one batched TokenSampler.SampleNext over a [256, 128256] fp32 logits
batch (Zipf-ranked logits, 1024-id histories, repetition 1.15, T 0.7, top-k 50,
top-p 0.9): the C ABI call ncb_sample_rows_device on device-resident inputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload zipf_ranked|peaked_head|zipf_history_nucleus|
                              high_entropy_nucleus|vocab_sharded|softmax_rows]
                  [--exchange nccl|peer]

N>1 runs under torch.distributed, one process per GPU. The fixed 256-row batch
is split over the GPUs by rows (sharding.row_range); each step every GPU
samples its rows and one NCCL all-gather gives every GPU all 256 token ids and
flags (strong scaling). Extra keys on the same line: every rank sampling its
own 256-row batch with no exchange (weak replicas), the 128 x 262144 batch with
its vocabulary split over the GPUs, the 1024 x 151936 nucleus batch split by
rows, one-row latency through the host-array call, the host-to-device copy
alone, and the parity of the sampled batch against the oracle.
--impl reference times the reference's CPU sampler on the host: the C# code
cannot run here (no .NET runtime), so its C restatement (oracle/) stands in,
on the whole batch with every host thread.
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
    ap.add_argument("--extras", type=int, default=1,
                    help="headline only: 0 skips the extra measurements (replicas, "
                         "vocabulary shards, nucleus batch, one-row latency)")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="rows split over GPUs: every GPU's tokens and flags gathered to every "
                         "GPU through peer memory by the library, or by an NCCL all-gather")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="vocab_sharded: records exchanged by an NCCL all-gather, or through "
                         "peer memory by the shard kernel itself")
    ap.add_argument("--workload", default="zipf_ranked",
                    choices=["zipf_ranked", "peaked_head", "zipf_history_nucleus",
                             "high_entropy_nucleus", "vocab_sharded", "softmax_rows"],
                    help="zipf_ranked: the headline (rows split over GPUs); vocab_sharded: "
                         "128 x 262144, vocabulary split over GPUs; softmax_rows: row softmax "
                         "of the 256 x 128256 logits batch; the others: their batch split "
                         "over the GPUs by rows")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def workload(rank=0, name="zipf_ranked"):
    """The batch of a sampling workload (the headline by default); rank r > 0
    gets its own rows (same generator, another seed) -- the weak replicas."""
    from neuraval_b200 import workloads
    gen = workloads.WORKLOADS[name]
    return gen() if rank == 0 else gen(seed=1000 * rank + 7)


def nbuf_for(rows, V, least=NBUF):
    """Rotated input copies per GPU so that a copy is read again only after
    twice the L2 capacity has streamed through."""
    return max(least, -(-2 * L2_BYTES // max(1, rows * V * 4)))


GATHER_KERNEL = {"peer": " and row_gather_kernel (tokens stored into every GPU), per step",
                 "nccl": " and the NCCL all-gather of the tokens, per step"}


def rows_config(wl, world, gather="peer"):
    """The `config` of a rows-split line; identical in both arms of the bench."""
    from neuraval_b200 import sharding
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    lo, hi = sharding.row_range(B, world, 0)
    nb = nbuf_for(hi - lo, V)
    how = ("stored into every GPU over NVLink by the library" if gather == "peer" else
           "all-gathered over NCCL")
    par = (f"{B} rows split over {world} GPUs (contiguous row ranges), token ids and flags "
           f"{how} every step" if world > 1 else f"{B} rows on 1 GPU")
    return {"workload": wl["name"], "B": B, "V": V, "history_per_row": H,
            **{k: v for k, v in wl["params"].items()},
            "uniforms": "one seeded u in [0,1) per row",
            "parallelism": par,
            "l2": (f"inputs larger than L2: each GPU rotates {nb} copies of its rows across "
                   "steps (twice the L2 capacity between reuses); the CPU arm reads the whole "
                   "batch, larger than its caches")}


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """DRAM bytes (read + write) per step of the top-k kernels, from the committed
    ncu summary of this workload (its `dram_bytes_per_launch:` line)."""
    path = os.path.join(ROOT, "profiles", "topk_chunk_kernels_zipf_ranked_256x128256.md")
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
            time.sleep(0.001)

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


# ---- the oracle: timed CPU baseline and the parity checker (rank 0 only) ------

def cpu_baseline(wl, seconds):
    """The oracle (C restatement of the C# sampler) on all host cores over a
    bounded sample of the same workload; returns (rows/s, threads, sample desc,
    1-thread rows/s)."""
    from oracle import pyoracle
    pyoracle.build()
    threads = host_threads()
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


def parity_of(wl, tokens, flags):
    """Tokens and flags of the sampled batch against the oracle: bit for bit with
    the correctly rounded exp the kernels use, and against libm expf (the
    reference's MathF.Exp), where rows may differ only when a boundary or tie
    flag is set; the flagged rows are counted."""
    from neuraval_b200 import native
    from oracle import pyoracle
    pyoracle.build()
    p = pyoracle.make_params(**wl["params"])
    offs = np.asarray(wl["hist_offsets"], np.int64)
    th = host_threads()
    cmp = ~native.FLAG_EXP_SLOW & 0xFFFFFFFF
    ct, cf, _ = pyoracle.sample_rows(wl["logits"], wl["hist_ids"], offs, wl["uniforms"], p,
                                     exp_mode=pyoracle.EXP_CR, threads=th)
    lt, lf, _ = pyoracle.sample_rows(wl["logits"], wl["hist_ids"], offs, wl["uniforms"], p,
                                     exp_mode=pyoracle.EXP_GLIBC, threads=th)
    tokens = np.asarray(tokens, np.int32)
    flags = np.asarray(flags, np.uint32)
    both = flags | lf
    exempt = (both & native.PARITY_EXEMPT) != 0
    differ = tokens != lt
    return {"rows": int(tokens.size),
            "exact_cr_rows_differ": int(((tokens != ct) | ((flags & cmp) != (cf & cmp))).sum()),
            "flagged_boundary": int(((both & (native.FLAG_DRAW_BOUNDARY |
                                              native.FLAG_CUTOFF_BOUNDARY)) != 0).sum()),
            "flagged_tie": int(((both & native.FLAG_TIE_AT_DRAW) != 0).sum()),
            "differ_unflagged": int((differ & ~exempt).sum()),
            "differ_flagged": int((differ & exempt).sum()),
            "nonfinite_or_overflow": int(((flags & (native.FLAG_NONFINITE |
                                                    native.FLAG_TIES_OVERFLOW)) != 0).sum()),
            "checker": "oracle/ (C restatement of TokenSampler.cs:54-135): exact with the "
                       "correctly rounded exp; libm expf for the flag-exempt comparison"}


def kernels_of(params, V):
    """The kernels one sampling call launches for these parameters (the
    dispatch of ncb_sample_rows_device): a name for the timed pair and the
    number of launches per step."""
    k = params.get("top_k", 0) or 0
    if params.get("greedy"):
        return "greedy_kernel", 1
    lowering = (params.get("repetition_penalty", 1.0) >= 1.0 and
                params.get("frequency_penalty", 0.0) >= 0.0 and
                params.get("presence_penalty", 0.0) >= 0.0)
    if 0 < k < V and k <= 64 and lowering and V >= 8192 and 683 * k <= V and V <= 262144:
        return ("topk_chunk_kernel (stream) + topk_chunk_finish_kernel (+ the fix-up launch), "
                "timed together"), 3
    if 0 < k < V and k <= 64:
        return "topk_ldg_kernel (+ its fix-up launch, timed together)", 2
    if 0 < k < V and k <= 1024:
        return "topk_kernel (+ its fix-up launch, timed together)", 2
    return "nucleus_kernel (+ its full-sort fix-up launch, timed together)", 2


def run_reference(args, rank, world):
    """The reference arm: the oracle port of TokenSampler on the host's cores,
    the whole batch every step, rank 0 only."""
    if rank != 0:
        return 0
    if args.workload == "softmax_rows":
        return run_softmax_reference(args)
    name = "zipf_ranked" if args.workload == "zipf_ranked" else args.workload
    wl = workload(0, name)
    from oracle import pyoracle
    pyoracle.build()
    threads = host_threads()
    p = pyoracle.make_params(**wl["params"])
    offs = np.asarray(wl["hist_offsets"], np.int64)
    B = wl["logits"].shape[0]
    lg, h, u = wl["logits"], wl["hist_ids"], wl["uniforms"]
    for _ in range(args.warmup):
        pyoracle.sample_rows(lg, h, offs, u, p, exp_mode=pyoracle.EXP_GLIBC, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pyoracle.sample_rows(lg, h, offs, u, p, exp_mode=pyoracle.EXP_GLIBC, threads=threads)
    dt = time.perf_counter() - t0
    value = B * args.steps / dt
    metric = METRIC if name == "zipf_ranked" else f"sampled rows/sec, {wl['name']}"
    cfg = (rows_config(wl, world, args.gather) if name != "vocab_sharded" else
           {"workload": wl["name"], "B": B, "V": wl["logits"].shape[1]})
    out = {"impl": "reference", "metric": metric, "value": value, "unit": UNIT, "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
           "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
           "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic (seeded generator, no dataset)", "config": cfg,
           "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": f"the whole {B}-row batch every step, {args.steps} steps, "
                                      f"{threads} threads; C restatement of "
                                      "TokenSampler.SampleFiltered (libm expf); the C# "
                                      "original needs a .NET runtime, absent here"},
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
        elif args.workload == "zipf_ranked":
            out = run_headline(args, rank, world, dev)
        else:
            out = run_rows_line(args, rank, world, dev, args.workload)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
    return 0


# ---- rows split over the GPUs ---------------------------------------------------

def start_gate(dev, world):
    """Queues work on the current stream ahead of a start event, without a host
    synchronisation after it: an all-reduce of one word over the ranks (every
    rank's timed region then starts within the all-reduce's own skew, not the
    hosts') and a spin of about 50 microseconds, long enough for the host to
    queue the timed launches behind the start event before it fires."""
    import torch
    if world > 1:
        torch.distributed.all_reduce(torch.zeros(1, device=dev))
    torch.cuda._sleep(100_000)


def time_graph(fn, steps, dev, world, clocks=None):
    """`fn(i)` for i < steps captured once in a CUDA graph, one untimed replay,
    then one replay between CUDA events on the current stream (ms). The clock
    sampler's thread starts before the ranks line up, so that starting it
    delays no rank's launches."""
    import torch
    cur = torch.cuda.current_stream(dev)
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(cur)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for i in range(steps):
                fn(i)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with (clocks if clocks is not None else contextlib.nullcontext()):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        start_gate(dev, world)
        t0.record(cur)
        graph.replay()
        t1.record(cur)
        torch.cuda.synchronize()
    del graph  # graphs holding NCCL calls go before the process group
    return t0.elapsed_time(t1)


class RowSplit:
    """One GPU's share of a row-split batch: its rows on the device (rotated
    copies), its sampler, and the all-gather of every GPU's tokens and flags."""

    def __init__(self, wl, rank, world, dev, least_buffers=NBUF, gather="peer"):
        import torch
        from neuraval_b200 import native, sharding
        from neuraval_b200.sampler import CudaTokenSampler
        self.wl, self.world, self.dev = wl, world, dev
        B, V = wl["logits"].shape
        self.B, self.V = B, V
        self.H = int(wl["hist_offsets"][-1] // B)
        lo, hi = sharding.row_range(B, world, rank)
        self.lo, self.rows = lo, hi - lo
        offs = np.asarray(wl["hist_offsets"], np.int64)
        self.params = native.make_params(**wl["params"])
        self.sampler = CudaTokenSampler(device=dev.index, max_rows=max(1, self.rows),
                                        max_vocab=V, max_history=max(1, self.H))
        mine = wl["logits"][lo:hi]
        self.nbuf = nbuf_for(max(1, self.rows), V, least_buffers)
        base = torch.from_numpy(np.ascontiguousarray(mine)).to(dev)
        self.bufs = [base] + [
            (base.roll(i, dims=0) if self.rows > 1 else base.roll(i * 97, dims=1)).contiguous()
            for i in range(1, self.nbuf)]
        h = wl["hist_ids"][offs[lo]: offs[hi]]
        self.hist = torch.from_numpy(np.ascontiguousarray(h if h.size else np.zeros(1, np.int32),
                                                          dtype=np.int32)).to(dev)
        self.offs = torch.from_numpy((offs[lo: hi + 1] - offs[lo]).astype(np.int32)).to(dev)
        self.u = torch.from_numpy(np.ascontiguousarray(wl["uniforms"][lo:hi])).to(dev)
        # world > 1: the library's row-split sampler (its rows, then every GPU's
        # tokens and flags gathered to every GPU: peer stores or an NCCL all-gather)
        self.split = None
        if world > 1:
            cls = sharding.PeerRowShardedSampler if gather == "peer" else sharding.RowShardedSampler
            self.split = cls(self.sampler, B)
        self.local = torch.zeros((2, max(1, self.rows)), dtype=torch.int32, device=dev)

    def step(self, i):
        import torch
        if self.split is not None:
            self.split.sample(self.bufs[i % self.nbuf], self.hist, self.offs, self.u,
                              self.params)
        else:
            self.sampler.sample_rows_device(self.bufs[i % self.nbuf], self.hist, self.offs,
                                            self.u, self.params, self.local[0], self.local[1],
                                            None, torch.cuda.current_stream(self.dev))

    def tokens_flags(self):
        """Every row's token and flags of the last step, in batch order (host)."""
        if self.split is not None:
            tok, fl = self.split.tokens_flags()
        else:
            tok, fl = self.local[0], self.local[1]
        return tok.cpu().numpy(), fl.cpu().numpy().astype(np.uint32)

    def close(self):
        self.sampler.close()


def run_split(wl, args, rank, world, dev, steps, clocks=None, least_buffers=NBUF, gather=None):
    """Times `steps` steps of the row-split batch (graph replay, max over ranks),
    then samples the unrotated batch once more for the parity check.
    Returns (ms for the steps, eager ms, tokens, flags, RowSplit)."""
    import torch
    from neuraval_b200 import sharding
    rs = RowSplit(wl, rank, world, dev, least_buffers, gather or args.gather)
    for i in range(max(3, args.warmup)):
        rs.step(i)
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start_gate(dev, world)
    e0.record(cur)
    for i in range(steps):
        rs.step(i)
    e1.record(cur)
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1)
    total_ms = time_graph(rs.step, steps, dev, world, clocks)
    total_ms, eager_ms = sharding.max_over_ranks([total_ms, eager_ms], dev)
    rs.step(0)  # the batch itself (copy 0), every rank: the step holds a collective
    torch.cuda.synchronize()
    tok, fl = rs.tokens_flags()
    return total_ms, eager_ms, tok, fl, rs


def run_headline(args, rank, world, dev):
    """The headline line: the fixed 256 x 128256 batch split over the GPUs by
    rows, plus the extra measurements."""
    import torch
    from neuraval_b200 import sharding, workloads
    wl = workload(0, "zipf_ranked")
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    clocks = ClockSampler(dev.index)
    total_ms, eager_ms, tok, fl, rs = run_split(wl, args, rank, world, dev, args.steps, clocks)
    nbuf = rs.nbuf
    rows_here = rs.rows
    per_step_ms = total_ms / args.steps
    value = B * args.steps / (total_ms / 1e3)

    out = None
    extras = {}
    if args.e2e_steps > 0:
        extras["e2e"] = e2e_rows(rs, args, world, dev)
    rs.close()
    del rs
    torch.cuda.empty_cache()
    if args.extras:
        extras["replicas"] = weak_replicas(args, rank, world, dev)
        torch.cuda.empty_cache()
        if world > 1:
            other = "nccl" if args.gather == "peer" else "peer"
            o_ms, _, o_tok, o_fl, o_rs = run_split(wl, args, rank, world, dev, args.steps,
                                                  gather=other)
            o_rs.close()
            del o_rs
            torch.cuda.empty_cache()
            if rank == 0:
                extras[f"{other}_gather"] = {
                    "value": B * args.steps / (o_ms / 1e3), "unit": UNIT,
                    "ms_per_step": o_ms / args.steps,
                    "kernel": kernels_of(wl["params"], V)[0] + GATHER_KERNEL[other],
                    "parity": parity_of(wl, o_tok, o_fl)}
        extras["vocab_sharded"] = vocab_sharded_summary(args, rank, world, dev)
        torch.cuda.empty_cache()
        extras["high_entropy_nucleus"] = nucleus_split_summary(args, rank, world, dev)
        torch.cuda.empty_cache()
        if world > 1:
            torch.distributed.barrier()
        if rank == 0:
            extras["e2e_b1"] = e2e_one_row(dev)
        if world > 1:
            torch.distributed.barrier()

    if rank == 0:
        peak, peak_kind = measured_peak()
        rows_max = sharding.row_range(B, world, 0)[1]  # the largest share
        bytes_per_launch = rows_max * workloads.bytes_per_row(V, H)
        achieved = bytes_per_launch / (per_step_ms / 1e3) / 1e9
        kernel, launches = kernels_of(wl["params"], V)
        out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step_ms,
               "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
               "vs_baseline": None, "dtype": "fp32",
               "data": "synthetic (seeded generator, no dataset)",
               "config": rows_config(wl, world, args.gather),
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "peak_source": peak_kind,
                            "traffic": profiled_traffic() if world == 1 else None,
                            "kernel": kernel + (GATHER_KERNEL[args.gather] if world > 1 else ""),
                            "algorithmic_bytes_per_launch": bytes_per_launch,
                            "per_gpu_rows": rows_max},
               "gpu_launches": (launches + (1 if world > 1 and args.gather == "peer" else 0))
                               * args.steps,
               "eager_value": B * args.steps / (eager_ms / 1e3),
               "timing": "CUDA events around one replay of a CUDA graph holding the K steps "
                         "(the token all-gather included); max over ranks",
               "clocks": clocks.summary(),
               "parity": parity_of(wl, tok, fl)}
        out["e2e"] = extras.pop("e2e", None)
        out.update(extras)
        if world == 1 and args.cpu_seconds > 0:
            v, cores, sample, one = cpu_baseline(wl, args.cpu_seconds)
            out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                   "sample": sample, "single_thread_value": one}
    return out


def e2e_rows(rs, args, world, dev):
    """End to end through the host-array call ncb_sample_rows: every step copies
    this GPU's rows in from pinned host memory, samples, synchronises and copies
    the tokens and flags out. Also the host-to-device copy of the same bytes
    alone, for comparison."""
    import torch
    from neuraval_b200 import sharding
    wl, lo, rows = rs.wl, rs.lo, rs.rows
    offs = np.asarray(wl["hist_offsets"], np.int64)
    h_logits = torch.from_numpy(np.ascontiguousarray(wl["logits"][lo: lo + rows])).pin_memory()
    h_hist = torch.from_numpy(np.ascontiguousarray(
        wl["hist_ids"][offs[lo]: offs[lo + rows]])).pin_memory()
    h_offs = torch.from_numpy((offs[lo: lo + rows + 1] - offs[lo]).astype(np.int32)).pin_memory()
    h_u = torch.from_numpy(np.ascontiguousarray(wl["uniforms"][lo: lo + rows])).pin_memory()
    hl, hh, ho, hu = (t.numpy() for t in (h_logits, h_hist, h_offs, h_u))
    from neuraval_b200.sampler import CudaTokenSampler
    # a handle of its own, as a caller of the host-array API would hold
    sampler = CudaTokenSampler(device=dev.index, max_rows=max(1, rows), max_vocab=rs.V,
                               max_history=max(1, rs.H))
    # the host-to-device copy alone (pinned, one copy per step), timed step by
    # step alternately with the call so that both see the same link (the PCIe
    # bandwidth of a shared host drifts between runs)
    d = torch.empty(h_logits.shape, dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(dev)

    def h2d():
        with torch.cuda.stream(s):
            d.copy_(h_logits, non_blocking=True)
            s.synchronize()

    for _ in range(3):
        sampler.sample_rows(hl, hh, ho, hu, rs.params)
        h2d()
    if world > 1:
        torch.distributed.barrier()
    e2e_s = h2d_s = 0.0
    for _ in range(args.e2e_steps):
        t0 = time.perf_counter()
        sampler.sample_rows(hl, hh, ho, hu, rs.params)
        t1 = time.perf_counter()
        h2d()
        t2 = time.perf_counter()
        e2e_s += t1 - t0
        h2d_s += t2 - t1
    sampler.close()
    e2e_s, h2d_s = sharding.max_over_ranks([e2e_s, h2d_s], dev)
    B = rs.B
    return {"value": B * args.e2e_steps / e2e_s, "unit": UNIT,
            "h2d_bytes_per_step": int(hl.nbytes + hh.nbytes + ho.nbytes + hu.nbytes),
            "d2h_bytes_per_step": int(rows * 4 * 2),
            "api": "ncb_sample_rows (host arrays; copies in, samples, synchronises, copies out); "
                   "each GPU its own rows, max over ranks",
            "ms_per_step": e2e_s / args.e2e_steps * 1e3,
            "h2d_only_ms_per_step": h2d_s / args.e2e_steps * 1e3,
            "h2d_only_gbs": hl.nbytes / (h2d_s / args.e2e_steps) / 1e9}


def e2e_one_row(dev):
    """The drop-in where the reference calls it: one 1 x 32000 row per call
    (TextGenerator.cs:93) through ncb_sample_rows with host arrays, against the
    oracle port on one thread (the reference's model: one call, one thread)."""
    import torch
    from neuraval_b200 import native, workloads
    from neuraval_b200.sampler import CudaTokenSampler
    from oracle import pyoracle
    wl = workloads.peaked_head(B=1)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()
    lg, hi, of, u = (pin(wl["logits"]), pin(wl["hist_ids"]), pin(wl["hist_offsets"]),
                     pin(wl["uniforms"]))
    p = native.make_params(**wl["params"])
    n = 300
    with CudaTokenSampler(device=dev.index, max_rows=1, max_vocab=32000, max_history=64) as s:
        for _ in range(20):
            s.sample_rows(lg, hi, of, u, p)
        t0 = time.perf_counter()
        for _ in range(n):
            tok, _, _ = s.sample_rows(lg, hi, of, u, p)
        gpu_us = (time.perf_counter() - t0) / n * 1e6
    pyoracle.build()
    op = pyoracle.make_params(**wl["params"])
    offs = np.asarray(wl["hist_offsets"], np.int64)
    for _ in range(5):
        pyoracle.sample_rows(wl["logits"], wl["hist_ids"], offs, wl["uniforms"], op,
                             exp_mode=pyoracle.EXP_GLIBC, threads=1)
    t0 = time.perf_counter()
    for _ in range(n):
        ot, _, _ = pyoracle.sample_rows(wl["logits"], wl["hist_ids"], offs, wl["uniforms"], op,
                                        exp_mode=pyoracle.EXP_GLIBC, threads=1)
    cpu_us = (time.perf_counter() - t0) / n * 1e6
    return {"workload": wl["name"], "us_per_call": gpu_us, "cpu_single_thread_us_per_row": cpu_us,
            "same_token": bool(tok[0] == ot[0]),
            "api": "ncb_sample_rows, host arrays (pinned), 1 row: copy in, sample, synchronise, "
                   "copy out"}


def weak_replicas(args, rank, world, dev):
    """Every rank samples its own 256-row batch (same generator, its own seed):
    no exchange; whole-job rows/s (weak scaling)."""
    import torch
    wl = workload(rank, "zipf_ranked")
    # one "world" of one: each rank alone, no gather
    total_ms, _, _, _, rs = run_split(wl, args, 0, 1, dev, args.steps)
    from neuraval_b200 import sharding
    (total_ms,) = sharding.max_over_ranks([total_ms], dev)
    rs.close()
    B = wl["logits"].shape[0]
    return {"value": world * B * args.steps / (total_ms / 1e3), "unit": UNIT,
            "ms_per_step": total_ms / args.steps, "scaling": "weak",
            "parallelism": f"{world} GPU(s), each its own {B}-row batch, no exchange"}


def nucleus_split_summary(args, rank, world, dev):
    """The 1024 x 151936 high-entropy nucleus batch (no top-k) split by rows."""
    from neuraval_b200 import workloads
    wl = workloads.high_entropy_nucleus()
    steps = max(3, min(args.steps, 40))
    total_ms, _, tok, fl, rs = run_split(wl, args, rank, world, dev, steps, least_buffers=2)
    rs.close()
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    out = None
    if rank == 0:
        from neuraval_b200 import sharding
        peak, _ = measured_peak()
        rows_max = sharding.row_range(B, world, 0)[1]
        ach = rows_max * workloads.bytes_per_row(V, H) / (total_ms / steps / 1e3) / 1e9
        out = {"value": B * steps / (total_ms / 1e3), "unit": UNIT, "steps": steps,
               "ms_per_step": total_ms / steps, "hbm_frac": ach / peak,
               "kernel": kernels_of(wl["params"], V)[0],
               "config": rows_config(wl, world, args.gather), "parity": parity_of(wl, tok, fl)}
    return out


def run_rows_line(args, rank, world, dev, name):
    """A secondary workload as its own line, split over the GPUs by rows."""
    from neuraval_b200 import sharding, workloads
    wl = workload(0, name)
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    clocks = ClockSampler(dev.index)
    total_ms, eager_ms, tok, fl, rs = run_split(wl, args, rank, world, dev, args.steps, clocks)
    rs.close()
    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    rows_max = sharding.row_range(B, world, 0)[1]
    per_step_ms = total_ms / args.steps
    bytes_per_launch = rows_max * workloads.bytes_per_row(V, H)
    achieved = bytes_per_launch / (per_step_ms / 1e3) / 1e9
    kernel, launches = kernels_of(wl["params"], V)
    out = {"metric": f"sampled rows/sec, {wl['name']}", "value": B * args.steps / (total_ms / 1e3),
           "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": per_step_ms, "higher_is_better": True,
           "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic (seeded generator, no dataset)",
           "config": rows_config(wl, world, args.gather),
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                        "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                        "kernel": kernel, "algorithmic_bytes_per_launch": bytes_per_launch},
           "e2e": None, "gpu_launches": launches * args.steps,
           "eager_value": B * args.steps / (eager_ms / 1e3),
           "timing": "CUDA events around one replay of a CUDA graph holding the K steps; "
                     "max over ranks",
           "clocks": clocks.summary(), "parity": parity_of(wl, tok, fl)}
    if world == 1 and args.cpu_seconds > 0:
        v, cores, sample, one = cpu_baseline(wl, args.cpu_seconds)
        out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                               "sample": sample, "single_thread_value": one}
    return out


# ---- vocabulary split over the GPUs ----------------------------------------------

def vocab_sharded_measure(args, rank, world, dev, clocks=None, exchange=None):
    """The 128 x 262144 batch (top-k 64) with its vocabulary split over the ranks:
    per step, the shard candidate kernel, one NCCL all-gather of the records and
    the merge kernel on every rank. Total work is fixed (strong scaling). The
    K steps are captured in one CUDA graph (the all-gather included) and
    replayed; each part is also timed alone the same way. Returns a dict of
    the measured numbers (rank 0) and the tokens' check against one GPU."""
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
    exchange = exchange or args.exchange
    peer = sharding.PeerVocabShardedSampler(sampler, V) if exchange == "peer" else None

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

    for i in range(max(3, args.warmup)):
        full(i)
    torch.cuda.synchronize()
    total_ms = time_graph(full, args.steps, dev, world, clocks)
    if peer is not None:
        # a merge needs the words its call's pushes store, so it is not timed
        # alone: the shard kernel is, and the exchange and merge are the rest
        parts = [time_graph(candidates, args.steps, dev, world), 0.0, 0.0]
        parts[2] = max(0.0, total_ms - parts[0])
    else:
        parts = [time_graph(f, args.steps, dev, world) for f in (candidates, exchange, merge)]
    total_ms, *parts = sharding.max_over_ranks([total_ms] + parts, dev)
    full(0)  # every rank: the step holds a collective
    torch.cuda.synchronize()
    res = None
    if rank == 0:
        # the sampled tokens equal the single-GPU sampler's on the whole rows
        ref_s = CudaTokenSampler(device=dev.index, max_rows=B, max_vocab=V, max_history=H)
        full_logits = torch.from_numpy(wl["logits"]).to(dev)
        rt = torch.empty_like(tokens)
        rf = torch.empty_like(flags)
        ref_s.sample_rows_device(full_logits, hist, offs, u, params, rt, rf)
        torch.cuda.synchronize()
        ok = bool(torch.equal(rt, tokens) and torch.equal(rf, flags))
        ref_s.close()
        del full_logits
        res = dict(wl=wl, B=B, V=V, H=H, width=width, nbuf=nbuf, total_ms=total_ms, parts=parts,
                   ok=ok, record_bytes=sampler.shard_record_bytes,
                   tokens=tokens.cpu().numpy(), flags=flags.cpu().numpy().astype(np.uint32))
    sampler.close()
    return res


def vocab_sharded_summary(args, rank, world, dev):
    r = vocab_sharded_measure(args, rank, world, dev)
    other = None
    if world > 1:
        import torch
        torch.cuda.empty_cache()
        o = vocab_sharded_measure(args, rank, world, dev,
                                  exchange="nccl" if args.exchange == "peer" else "peer")
        if rank == 0:
            other = {"ms_per_step": o["total_ms"] / args.steps,
                     "parts_us_per_step": {"candidates": o["parts"][0] / args.steps * 1e3,
                                           "exchange": o["parts"][1] / args.steps * 1e3,
                                           "merge": o["parts"][2] / args.steps * 1e3},
                     "tokens_match_single_gpu": o["ok"]}
    if rank != 0:
        return None
    s = args.steps
    out = {"value": r["B"] * s / (r["total_ms"] / 1e3), "unit": UNIT,
            "ms_per_step": r["total_ms"] / s, "n_gpus": world, "shard_columns": r["width"],
            "parts_us_per_step": {"candidates": r["parts"][0] / s * 1e3,
                                  "exchange": r["parts"][1] / s * 1e3,
                                  "merge": r["parts"][2] / s * 1e3},
            "exchange": "NCCL all-gather of the records" if args.exchange == "nccl" else
                        "records stored into every GPU's exchange area over NVLink by the "
                        "shard kernel as epoch-tagged words; 'merge' is the step minus the "
                        "shard kernel timed alone (exchange included)",
            "tokens_match_single_gpu": r["ok"],
            "parity": parity_of(r["wl"], r["tokens"], r["flags"]),
            "config": {"workload": r["wl"]["name"], "B": r["B"], "V": r["V"],
                       "parallelism": f"vocabulary split over {world} GPU(s)"}}
    if other is not None:
        out["nccl_exchange" if args.exchange == "peer" else "peer_exchange"] = other
    return out


def run_vocab_sharded(args, rank, world, dev):
    clocks = ClockSampler(dev.index)
    r = vocab_sharded_measure(args, rank, world, dev, clocks)
    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    B, H, width = r["B"], r["H"], r["width"]
    per_gpu_bytes = B * (4 * width + 4 * H + 8)
    per_step_s = r["total_ms"] / args.steps / 1e3
    parts = r["parts"]
    return {"metric": "sampled rows/sec, vocabulary split over GPUs", "value":
            B * args.steps / (r["total_ms"] / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["total_ms"] / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic (seeded generator, no dataset)",
            "config": {"workload": r["wl"]["name"], "B": B, "V": r["V"], "history_per_row": H,
                       **r["wl"]["params"],
                       "parallelism": f"vocabulary sharded over {world} GPU(s); "
                                      f"{args.exchange} record exchange",
                       "l2": f"{r['nbuf']} rotated copies of each shard",
                       "shard_columns": width,
                       "record_bytes_per_rank": B * r["record_bytes"]},
            "parts_us_per_step": {"candidates": parts[0] / args.steps * 1e3,
                                  "exchange": parts[1] / args.steps * 1e3,
                                  "merge": parts[2] / args.steps * 1e3},
            "exchange": ("records stored into every GPU's exchange area over NVLink by the "
                         "shard kernel as epoch-tagged words, waited for by the merge; 'merge' "
                         "is the step minus the shard kernel timed alone"
                         if args.exchange == "peer" else "NCCL all-gather of the records"),
            "tokens_match_single_gpu": r["ok"],
            "parity": parity_of(r["wl"], r["tokens"], r["flags"]),
            "roofline": {"bound": "hbm", "achieved": per_gpu_bytes / per_step_s / 1e9,
                         "peak": peak, "unit": "GB/s",
                         "frac": per_gpu_bytes / per_step_s / 1e9 / peak,
                         "peak_source": peak_kind, "traffic": None,
                         "kernel": "shard candidate kernel + all-gather + merge, per step",
                         "algorithmic_bytes_per_launch": per_gpu_bytes},
            "e2e": None,
            "gpu_launches": 2 * args.steps,  # the shard kernel and the merge
            "timing": "CUDA events around one replay of a CUDA graph holding the K steps "
                      "(all-gather included); max over ranks",
            "clocks": clocks.summary()}


# ---- row softmax ------------------------------------------------------------------

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

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    total_ms = time_graph(step, args.steps, dev, world, clocks)
    (total_ms,) = sharding.max_over_ranks([total_ms], dev)
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
