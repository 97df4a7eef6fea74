"""Vocabulary-shard kernels on one GPU: G shards emulated on one device (each
column range reduced to its records, records stacked in column order, merged)
must give the same tokens and flags as the single-GPU entry point on the whole
rows, and the oracle's tokens. The exchange itself (an all-gather) is covered
by the gloo tests and the multi-GPU bench."""
import ctypes

import numpy as np
import pytest

from neuraval_b200 import native, sharding, workloads
from tests.gpu_util import assert_exact, run_gpu, run_oracle, to_dev

pytestmark = pytest.mark.gpu


def run_sharded(s, wl, G, params=None, contiguous=False):
    import torch
    logits, hist, offs, u = to_dev(wl)
    B, V = wl["logits"].shape
    p = params if params is not None else native.make_params(**wl["params"])
    recs = torch.zeros((G, B, s.shard_record_bytes // 4), dtype=torch.int32, device="cuda")
    for g in range(G):
        lo, hi = sharding.vocab_range(V, G, g)
        if hi > lo:
            shard = logits[:, lo:hi]
            if contiguous:
                shard = shard.contiguous()
            s.shard_candidates_device(shard, V, lo, hist, offs, p, recs[g])
    tokens = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    flags = torch.zeros(B, dtype=torch.int32, device="cuda")
    s.shard_merge_device(recs, G, B, V, u, p, tokens, flags)
    torch.cuda.synchronize()
    return tokens.cpu().numpy(), flags.cpu().numpy().astype(np.uint32)


def assert_same_as_single(s, wl, G, contiguous=False, allow_cut=False):
    st, sf = run_sharded(s, wl, G, contiguous=contiguous)
    rt, rf, _ = run_gpu(s, wl)
    cut = (sf & native.FLAG_TIES_OVERFLOW) != 0
    if not allow_cut:
        assert not cut.any(), np.nonzero(cut)[0]
    ok = ~cut
    bad = np.nonzero(ok & ((st != rt) | (sf != rf)))[0]
    assert bad.size == 0, (G, bad[:8], st[bad[:8]], rt[bad[:8]], sf[bad[:8]], rf[bad[:8]])
    assert np.all(st[cut] == -1)
    return st, sf, cut


@pytest.mark.parametrize("G", [1, 2, 3, 4, 8])
def test_zipf_ranked_shards(gpu_sampler, oracle, G):
    wl = workloads.zipf_ranked(B=16, V=50000, H=256, seed=21)
    st, sf, _ = assert_same_as_single(gpu_sampler, wl, G, contiguous=(G == 3))
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    assert_exact(st, sf, ot, of, f"zipf_ranked G={G}")


@pytest.mark.parametrize("G", [2, 4, 8])
def test_vocab_sharded_workload(gpu_sampler, oracle, G):
    """The whole 128 x 262144 batch through the shard and merge kernels."""
    from tests.gpu_util import parity_report
    wl = workloads.vocab_sharded()
    st, sf, _ = assert_same_as_single(gpu_sampler, wl, G)
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    assert_exact(st, sf, ot, of, f"vocab_sharded G={G}")
    lt, lf, _ = run_oracle(oracle, wl, oracle.EXP_GLIBC)
    rep = parity_report(st, sf, lt, lf)
    assert rep["differ_unflagged"] == 0, rep


def test_counts_and_raising_penalty(gpu_sampler, oracle):
    wl = workloads.zipf_history_nucleus(B=12, V=32000, H=300, seed=23)
    wl["params"] = dict(temperature=0.9, top_k=64, top_p=0.9, frequency_penalty=0.4,
                        presence_penalty=0.2)
    assert_same_as_single(gpu_sampler, wl, 4)
    wl2 = workloads.zipf_ranked(B=10, V=40000, H=128, seed=24, repetition_penalty=0.8)
    st, sf, _ = assert_same_as_single(gpu_sampler, wl2, 3)
    ot, of, _ = run_oracle(oracle, wl2, oracle.EXP_CR)
    assert_exact(st, sf, ot, of, "penalty < 1")


def test_greedy_shards_with_nan(gpu_sampler):
    wl = workloads.peaked_head(B=10, V=30000, seed=25, greedy=True)
    wl["logits"][1, 0] = np.nan      # NaN at global id 0: token 0
    wl["logits"][2, 17000] = np.nan  # NaN elsewhere never wins
    wl["logits"][3, :] = 0.5         # all equal: first id
    for G in (2, 3, 5):
        st, sf, _ = assert_same_as_single(gpu_sampler, wl, G)
        assert st[1] == 0 and st[3] == 0


def test_nonfinite_and_small_vocab(gpu_sampler):
    wl = workloads.zipf_ranked(B=6, V=20000, H=32, seed=26)
    wl["logits"][2, 12345] = np.nan
    wl["logits"][4, 3] = np.inf
    st, sf, _ = assert_same_as_single(gpu_sampler, wl, 4)
    assert st[2] == -1 and sf[2] & native.FLAG_NONFINITE
    assert st[4] == -1 and sf[4] & native.FLAG_NONFINITE
    small = workloads.zipf_ranked(B=3, V=10, H=4, seed=27, top_k=5)
    assert_same_as_single(gpu_sampler, small, 4)  # shards of 4, 4, 2 and 0 columns


def test_masked_columns(gpu_sampler, oracle):
    wl = workloads.zipf_ranked(B=5, V=24000, H=32, seed=30, top_k=50)
    wl["logits"][:, 18000:] = -np.inf                           # a masked shard
    wl["logits"][1, :] = -np.inf                                # nothing finite
    wl["logits"][2, :] = -np.inf
    wl["logits"][2, [5, 900, 7000, 12000, 23999 - 8000]] = [1.0, 2.0, 0.5, 3.0, -1.0]  # < K finite
    st, sf, _ = assert_same_as_single(gpu_sampler, wl, 4)
    assert st[1] == -1 and sf[1] & native.FLAG_NONFINITE
    assert st[2] in (5, 900, 7000, 12000, 15999)
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    keep = np.array([0, 2, 3, 4])
    assert_exact(st[keep], sf[keep], ot[keep], of[keep], "masked columns")


def test_ties_beyond_the_record(gpu_sampler):
    wl = workloads.zipf_ranked(B=4, V=30000, H=16, seed=28, top_k=40)
    wl["logits"][0, :] = 1.0                                            # ties everywhere
    wl["logits"][1, np.random.default_rng(1).choice(30000, 60, replace=False)] = 50.0
    st, sf, cut = assert_same_as_single(gpu_sampler, wl, 2, allow_cut=True)
    assert cut[0] and sf[0] == native.FLAG_TIES_OVERFLOW
    assert not cut[1:].any()


def test_history_beyond_capacity(navlib):
    from neuraval_b200.sampler import CudaTokenSampler
    wl = workloads.zipf_history_nucleus(B=3, V=8000, H=200, seed=29)
    wl["params"] = dict(temperature=1.0, top_k=20, frequency_penalty=0.3)
    with CudaTokenSampler(0, max_rows=8, max_vocab=8192, max_history=64) as s:
        st, sf = run_sharded(s, wl, 2)
        rt, rf, _ = run_gpu(s, wl)
    assert np.array_equal(st, rt) and np.array_equal(sf, rf)
    assert np.all(st == -1) and np.all(sf & native.FLAG_BAD_HISTORY)


def test_shard_capacity_and_argument_errors(gpu_sampler):
    import torch
    lib = native.load()
    x = torch.zeros((2, 64), dtype=torch.float32, device="cuda")
    offs = torch.zeros(3, dtype=torch.int32, device="cuda")
    recs = torch.zeros((17, 2, gpu_sampler.shard_record_bytes // 4), dtype=torch.int32,
                       device="cuda")
    u = torch.zeros(2, dtype=torch.float32, device="cuda")
    tok = torch.zeros(2, dtype=torch.int32, device="cuda")
    h = gpu_sampler._h
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    big = native.make_params(top_k=65)
    ok = native.make_params(top_k=8)
    assert lib.ncb_vocab_shard_candidates_device(h, P(x), 2, 100, 0, 64, 64, None, P(offs),
                                                 ctypes.byref(big), P(recs), None) == \
        native.NCB_ERROR_CAPACITY
    assert lib.ncb_vocab_shard_candidates_device(h, P(x), 2, 100, 60, 124, 64, None, P(offs),
                                                 ctypes.byref(ok), P(recs), None) == \
        native.NCB_ERROR_INVALID_ARGUMENT
    assert lib.ncb_vocab_shard_merge_device(h, P(recs), 17, 2, 100, P(u), ctypes.byref(ok),
                                            P(tok), None, None) == native.NCB_ERROR_CAPACITY
    assert lib.ncb_vocab_shard_record_bytes() == 1040


@pytest.mark.parametrize("G", [2, 4])
def test_peer_exchange_emulated_on_one_gpu(navlib, G):
    """The peer-memory exchange with every shard's area on one GPU: all shards
    push, then all merge, for three calls in a row (epochs, flags and acks)."""
    import torch
    from neuraval_b200.sampler import CudaTokenSampler
    B, V = 12, 30000
    samplers = [CudaTokenSampler(0, max_rows=16, max_vocab=V, max_history=512) for _ in range(G)]
    ref = CudaTokenSampler(0, max_rows=16, max_vocab=V, max_history=512)
    try:
        handles = b"".join(s.peer_setup(G, g) for g, s in enumerate(samplers))
        for s in samplers:
            s.peer_connect(handles)
        for call in range(3):
            wl = workloads.zipf_ranked(B=B, V=V, H=64, seed=40 + call)
            if call == 2:
                wl = workloads.peaked_head(B=B, V=V, seed=43, greedy=True)
            logits, hist, offs, u = to_dev(wl)
            p = native.make_params(**wl["params"])
            for g, s in enumerate(samplers):
                lo, hi = sharding.vocab_range(V, G, g)
                s.shard_push_peer_device(logits[:, lo:hi], V, lo, hist, offs, p)
            outs = []
            for s in samplers:
                tok = torch.full((B,), -7, dtype=torch.int32, device="cuda")
                fl = torch.zeros(B, dtype=torch.int32, device="cuda")
                s.shard_merge_peer_device(B, V, u, p, tok, fl)
                outs.append((tok, fl))
            rt, rf, _ = run_gpu(ref, wl)
            torch.cuda.synchronize()
            for tok, fl in outs:
                assert np.array_equal(tok.cpu().numpy(), rt), (G, call)
                assert np.array_equal(fl.cpu().numpy().astype(np.uint32), rf), (G, call)
    finally:
        for s in samplers + [ref]:
            s.close()


def _peer_rank_main(rank, world, port):
    import os
    import datetime
    import torch
    import torch.distributed as dist
    from neuraval_b200.sampler import CudaTokenSampler
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        B, V = 16, 65536
        s = CudaTokenSampler(rank, max_rows=B, max_vocab=V, max_history=256)
        s2 = CudaTokenSampler(rank, max_rows=B, max_vocab=V, max_history=256)
        peer = sharding.PeerVocabShardedSampler(s, V)
        nccl = sharding.VocabShardedSampler(s2, V)
        for call in range(4):
            wl = workloads.zipf_ranked(B=B, V=V, H=128, seed=60 + call)
            logits, hist, offs, u = to_dev(wl)
            shard = logits[:, peer.col_begin:peer.col_end].contiguous()
            p = native.make_params(**wl["params"])
            t1 = torch.empty(B, dtype=torch.int32, device="cuda")
            f1 = torch.zeros(B, dtype=torch.int32, device="cuda")
            t2 = torch.empty_like(t1)
            f2 = torch.zeros_like(f1)
            peer.sample(shard, hist, offs, u, p, t1, f1)
            nccl.sample(shard, hist, offs, u, p, t2, f2)
            torch.cuda.synchronize()
            assert torch.equal(t1, t2) and torch.equal(f1, f2), (rank, call)
            if rank == 0:
                with CudaTokenSampler(0, max_rows=B, max_vocab=V, max_history=256) as one:
                    rt, rf, _ = run_gpu(one, wl)
                assert np.array_equal(t1.cpu().numpy(), rt), call
        torch.cuda.synchronize()
        dist.barrier()
        s.close()
        s2.close()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_two_gpus():
    import socket
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    mp.start_processes(_peer_rank_main, args=(2, port), nprocs=2, start_method="spawn", join=True)


def test_peer_connect_rejects_mismatched_layouts(navlib):
    """A GPU writes into a peer's area at offsets computed from its own layout,
    so connect refuses handles set up for another shard count, row count or
    exchange (no kernel runs here)."""
    from neuraval_b200.sampler import CudaTokenSampler
    mk = lambda rows: CudaTokenSampler(0, max_rows=rows, max_vocab=4096, max_history=64)
    ss = [mk(16), mk(32), mk(16), mk(16), mk(8), mk(8), mk(8), mk(8)]
    try:
        a, b, c = ss[0].peer_setup(2, 0), ss[1].peer_setup(2, 1), ss[2].peer_setup(2, 1)
        with pytest.raises(native.NcbError):
            ss[0].peer_connect(a + b)          # max_rows 16 against 32
        ss[0].peer_connect(a + c)              # the same layout connects
        d = ss[3].peer_setup(3, 0)
        with pytest.raises(native.NcbError):
            ss[3].peer_connect(d + c + c)      # set up for 3 shards, peers for 2
        r0, r1 = ss[4].row_gather_setup(2, 0, 100), ss[5].row_gather_setup(2, 1, 101)
        with pytest.raises(native.NcbError):
            ss[4].row_gather_connect(r0 + r1)  # rows_total 100 against 101
        with pytest.raises(native.NcbError):
            ss[4].row_gather_connect(r0 + c)   # a vocabulary-shard handle
        r2 = ss[6].row_gather_setup(2, 1, 100)
        ss[4].row_gather_connect(r0 + r2)
        assert len(r0) == native.load().ncb_peer_handle_bytes()
    finally:
        for s in ss:
            s.close()
