"""Host side of multi-GPU sampling, on CPU: the row and vocabulary splits, and
the vocabulary-shard decomposition run as two gloo ranks.

The decomposition test restates the per-shard record and the merge in numpy
(the record layout of ncb_vocab_shard_candidates_device: 4 header words, 128
values, 128 ids) and checks, over a real all-gather between two processes,
that the merged candidate set equals the candidate set of the whole rows
(TokenSampler.cs:73-93: every value >= the K-th largest, with multiplicity).
"""
import os
import socket

import numpy as np
import pytest

from neuraval_b200 import sharding, workloads

CAP, HDR = 128, 4
OVF_AT_KTH = 0x1000


@pytest.mark.parametrize("rows,world", [(0, 1), (1, 1), (7, 2), (256, 3), (5, 8), (1024, 8)])
def test_row_range_partitions(rows, world):
    got = [sharding.row_range(rows, world, r) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == rows
    for (a, b), (c, d) in zip(got, got[1:]):
        assert b == c
    sizes = [b - a for a, b in got]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("vocab,world", [(1, 1), (10, 2), (32000, 3), (128256, 8), (262144, 8),
                                         (151936, 7), (5, 4)])
def test_vocab_range_partitions(vocab, world):
    got = [sharding.vocab_range(vocab, world, r) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == vocab
    for (a, b), (c, d) in zip(got, got[1:]):
        assert b == c
    for a, b in got:
        assert b == a or a % 4 == 0  # every non-empty shard starts 16-byte aligned
    assert all(b >= a for a, b in got)


def test_ranges_reject_bad_arguments():
    with pytest.raises(ValueError):
        sharding.row_range(4, 0, 0)
    with pytest.raises(ValueError):
        sharding.vocab_range(0, 2, 0)
    with pytest.raises(ValueError):
        sharding.vocab_range(10, 2, 2)


def _values(logits, hist, params):
    """AdjustLogit then x (1/T), fp32, one row (TokenSampler.cs:68-71, :137-143)."""
    f32 = np.float32
    v = logits.astype(np.float32).copy()
    V = v.size
    h = hist[(hist >= 0) & (hist < V)]
    pen = f32(params.get("repetition_penalty", 1.0))
    if pen != f32(1.0) and h.size:
        m = np.zeros(V, bool)
        m[h] = True
        v = np.where(m, np.where(v > 0, v / pen, v * pen), v).astype(np.float32)
    freq = f32(params.get("frequency_penalty", 0.0))
    pres = f32(params.get("presence_penalty", 0.0))
    if (freq != 0 or pres != 0) and h.size:
        c = np.bincount(h, minlength=V).astype(np.float32)
        hit = c > 0
        v = np.where(hit, (v - c * freq).astype(np.float32), v).astype(np.float32)
        v = np.where(hit, (v - pres).astype(np.float32), v).astype(np.float32)
    scale = f32(1.0) / f32(params["temperature"])
    return (v * scale).astype(np.float32)


def _record(vals, ids, K):
    rec = np.zeros(HDR + 2 * CAP, np.int32)
    if vals.size == 0:
        return rec
    kth = np.sort(vals)[::-1][K - 1] if vals.size >= K else np.float32(-np.inf)
    above = np.nonzero(vals > kth)[0]
    ties = np.nonzero(vals == kth)[0]
    keep = np.concatenate([above, ties])[:CAP]
    rec[0] = keep.size
    rec[1] = OVF_AT_KTH if above.size + ties.size > CAP else 0
    rec[2] = np.float32(kth).view(np.int32)
    rec[3] = above.size + ties.size
    rec[HDR:HDR + keep.size] = vals[keep].view(np.int32)
    rec[HDR + CAP:HDR + CAP + keep.size] = ids[keep]
    return rec


def _merge(recs, K):
    """recs [shards, REC] of one row -> (sorted candidate ids, overflow flag)."""
    v, i = [], []
    for r in recs:
        n = int(r[0])
        v.append(r[HDR:HDR + n].view(np.float32))
        i.append(r[HDR + CAP:HDR + CAP + n])
    v, i = np.concatenate(v), np.concatenate(i)
    theta = np.sort(v)[::-1][K - 1]
    cut = any((int(r[1]) & OVF_AT_KTH) and r[2:3].view(np.float32)[0] == theta for r in recs)
    return np.sort(i[v >= theta]), cut


def _full_candidates(vals, K):
    theta = np.sort(vals)[::-1][K - 1]
    return np.sort(np.nonzero(vals >= theta)[0]).astype(np.int32)


def _rank_main(rank, world, port, name):
    case = CASES[name]
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = case["make"]()
        B, V = wl["logits"].shape
        K = min(wl["params"]["top_k"], V)
        lo, hi = sharding.vocab_range(V, world, rank)
        offs = wl["hist_offsets"]
        recs = np.zeros((B, HDR + 2 * CAP), np.int32)
        full = []
        for b in range(B):
            vals = _values(wl["logits"][b], wl["hist_ids"][offs[b]:offs[b + 1]], wl["params"])
            full.append(vals)
            recs[b] = _record(vals[lo:hi], np.arange(lo, hi, dtype=np.int32), K)
        gathered = sharding.gather_records(torch.from_numpy(recs)).numpy()
        assert gathered.shape == (world, B, HDR + 2 * CAP)
        assert np.array_equal(gathered[rank], recs)  # rank order = column order
        n_cut = 0
        for b in range(B):
            ids, cut = _merge(gathered[:, b], K)
            if cut:  # flagged rows: only where the shards' records had to cut ties
                assert case.get("expect_cut"), b
                assert _full_candidates(full[b], K).size > CAP - K + 1, b
                n_cut += 1
                continue
            assert np.array_equal(ids, _full_candidates(full[b], K)), b
        assert (n_cut > 0) == bool(case.get("expect_cut"))
        # the slowest rank's time is what a multi-GPU step reports
        mx = sharding.max_over_ranks([float(rank), 10.0 - rank])
        assert mx == [float(world - 1), 10.0]
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tied_rows():
    # a quantised batch: many values equal to the K-th largest
    rng = np.random.default_rng(7)
    wl = workloads.zipf_ranked(B=4, V=3000, H=16, seed=9, top_k=40)
    wl["logits"] = np.round(wl["logits"] * 2.0).astype(np.float32) / np.float32(2.0)
    wl["logits"][0, :] = 1.0  # every value tied: the shards cut ties at the global K-th
    wl["logits"][1, rng.choice(3000, 60, replace=False)] = 50.0  # 60 ties above the rest
    return wl


def _zipf_rows():
    return workloads.zipf_ranked(B=6, V=5003, H=40, seed=11)


def _count_rows():
    return dict(workloads.zipf_history_nucleus(B=5, V=4000, H=64, seed=12),
                params=dict(temperature=0.9, top_k=64, top_p=0.9, frequency_penalty=0.4,
                            presence_penalty=0.2))


CASES = {
    "zipf_ranked": dict(make=_zipf_rows),
    "counts": dict(make=_count_rows),
    "ties": dict(make=_tied_rows, expect_cut=True),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_vocab_shard_decomposition_two_gloo_ranks(case):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port(), case), nprocs=2,
                       start_method="spawn", join=True)
