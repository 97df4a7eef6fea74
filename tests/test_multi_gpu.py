"""Sampling over two real GPUs, one process per GPU, NCCL over NVLink: the
headline batch split by rows (each GPU samples its rows; the tokens and flags
gathered by one NCCL all-gather, or stored into every GPU over NVLink by the
library's row_gather_kernel) and the 128 x 262144 batch split by vocabulary (shard
records all-gathered, merged on every GPU). Every rank gets all rows' tokens;
rank 0 checks them against the oracle bit for bit (correctly rounded exp) and
against libm expf (rows may differ only where a boundary or tie flag is set).
Skipped with fewer than two GPUs; the vocabulary-shard kernels themselves are
also covered on one GPU with emulated shards."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _check(wl, tok, fl):
    from oracle import pyoracle
    from tests.gpu_util import assert_exact, parity_report, run_oracle
    pyoracle.build()
    ot, of, _ = run_oracle(pyoracle, wl, pyoracle.EXP_CR)
    assert_exact(tok, fl, ot, of, wl["name"])
    lt, lf, _ = run_oracle(pyoracle, wl, pyoracle.EXP_GLIBC)
    rep = parity_report(tok, fl, lt, lf)
    assert rep["differ_unflagged"] == 0, rep


def _rows_peer(rank, world, dev):
    """The row split with the library's peer-memory gather: three calls, the
    uniforms changed between them, so a copy left from an earlier call (the
    gather alternates between two copies) would show."""
    import torch
    from neuraval_b200 import native, sharding, workloads
    from neuraval_b200.sampler import CudaTokenSampler
    wl = workloads.zipf_ranked()
    B, V = wl["logits"].shape
    H = int(wl["hist_offsets"][-1] // B)
    lo, hi = sharding.row_range(B, world, rank)
    offs = np.asarray(wl["hist_offsets"], np.int64)
    variants = [wl, dict(wl, uniforms=np.ascontiguousarray(np.roll(wl["uniforms"], 37)),
                         name=wl["name"] + " (uniforms rolled)"), wl]
    with CudaTokenSampler(rank, max_rows=hi - lo, max_vocab=V, max_history=H) as s:
        rs = sharding.PeerRowShardedSampler(s, B)
        logits = torch.from_numpy(np.ascontiguousarray(wl["logits"][lo:hi])).to(dev)
        hist = torch.from_numpy(np.ascontiguousarray(wl["hist_ids"][offs[lo]:offs[hi]])).to(dev)
        ho = torch.from_numpy((offs[lo:hi + 1] - offs[lo]).astype(np.int32)).to(dev)
        p = native.make_params(**wl["params"])
        for v in variants:
            u = torch.from_numpy(np.ascontiguousarray(v["uniforms"][lo:hi])).to(dev)
            rs.sample(logits, hist, ho, u, p)
            tok, fl = rs.tokens_flags()
            torch.cuda.synchronize()
            tok = tok.cpu().numpy()
            fl = fl.cpu().numpy().astype(np.uint32)
            assert not np.any(fl & native.FLAG_PEER_TIMEOUT), rank
            if rank == 0:
                _check(v, tok, fl)
        torch.cuda.synchronize()


def _rank_main(rank, world, port, case):
    import torch
    import torch.distributed as dist
    from neuraval_b200 import native, sharding, workloads
    from neuraval_b200.sampler import CudaTokenSampler
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        if case == "rows_peer":
            _rows_peer(rank, world, dev)
        elif case == "rows":
            wl = workloads.zipf_ranked()
            B, V = wl["logits"].shape
            H = int(wl["hist_offsets"][-1] // B)
            lo, hi = sharding.row_range(B, world, rank)
            offs = np.asarray(wl["hist_offsets"], np.int64)
            with CudaTokenSampler(rank, max_rows=hi - lo, max_vocab=V, max_history=H) as s:
                rs = sharding.RowShardedSampler(s, B)
                logits = torch.from_numpy(np.ascontiguousarray(wl["logits"][lo:hi])).to(dev)
                hist = torch.from_numpy(np.ascontiguousarray(wl["hist_ids"][offs[lo]:offs[hi]])).to(dev)
                ho = torch.from_numpy((offs[lo:hi + 1] - offs[lo]).astype(np.int32)).to(dev)
                u = torch.from_numpy(np.ascontiguousarray(wl["uniforms"][lo:hi])).to(dev)
                p = native.make_params(**wl["params"])
                for _ in range(2):  # twice: the gather buffers are reused
                    rs.sample(logits, hist, ho, u, p)
                    tok, fl = rs.tokens_flags()
                    torch.cuda.synchronize()
                    tok = tok.cpu().numpy()
                    fl = fl.cpu().numpy().astype(np.uint32)
                    if rank == 0:
                        _check(wl, tok, fl)
                torch.cuda.synchronize()
        else:
            wl = workloads.vocab_sharded()
            B, V = wl["logits"].shape
            H = int(wl["hist_offsets"][-1] // B)
            lo, hi = sharding.vocab_range(V, world, rank)
            with CudaTokenSampler(rank, max_rows=B, max_vocab=hi - lo, max_history=H) as s:
                vs = sharding.VocabShardedSampler(s, V)
                shard = torch.from_numpy(np.ascontiguousarray(wl["logits"][:, lo:hi])).to(dev)
                hist = torch.from_numpy(wl["hist_ids"]).to(dev)
                ho = torch.from_numpy(wl["hist_offsets"]).to(dev)
                u = torch.from_numpy(wl["uniforms"]).to(dev)
                p = native.make_params(**wl["params"])
                tok = torch.full((B,), -7, dtype=torch.int32, device=dev)
                fl = torch.zeros(B, dtype=torch.int32, device=dev)
                vs.sample(shard, hist, ho, u, p, tok, fl)
                torch.cuda.synchronize()
                t, f = tok.cpu().numpy(), fl.cpu().numpy().astype(np.uint32)
                all_t = [torch.empty_like(tok) for _ in range(world)]
                dist.all_gather(all_t, tok)  # every rank merged the same tokens
                for x in all_t:
                    assert torch.equal(x, tok), rank
                if rank == 0:
                    _check(wl, t, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["rows", "rows_peer", "vocab"])
def test_two_gpus_nccl(case):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank_main, args=(2, _port(), case), nprocs=2, start_method="spawn",
                       join=True)
