"""GPU parity of the sampling kernels against the CPU oracle, through the C ABI.

Bar: with the correctly rounded exp the kernels must agree with the oracle bit
for bit (tokens, flags, probabilities); against the reference's own arithmetic
(libm expf, what MathF.Exp calls) tokens must agree on every row without a
boundary/tie flag, and probabilities within 1e-5 relative.
"""
import json
import os

import numpy as np
import pytest

from neuraval_b200 import native, workloads
from tests.gpu_util import assert_exact, parity_report, run_gpu, run_oracle

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))


def full_check(gpu_sampler, oracle, wl, probs=True, label=""):
    gt, gf, gp = run_gpu(gpu_sampler, wl, want_probs=probs)
    ot, of, op = run_oracle(oracle, wl, oracle.EXP_CR, want_probs=probs)
    assert_exact(gt, gf, ot, of, label)
    if probs:
        bad = np.argwhere(gp != op)
        assert bad.size == 0, (label, len(bad), [(int(r), int(c), float(gp[r, c]), float(op[r, c]))
                                                 for r, c in bad[:6]])
    rt, rf, rp = run_oracle(oracle, wl, oracle.EXP_GLIBC, want_probs=probs)
    rep = parity_report(gt, gf, rt, rf)
    assert rep["differ_unflagged"] == 0, (label, rep)
    if probs:
        np.testing.assert_allclose(gp, rp, rtol=1e-5, atol=0)
    return rep


@pytest.mark.parametrize("case", KATS["sampler"], ids=lambda c: c["name"])
def test_reference_kats_through_host_api(gpu_sampler, case):
    p = native.make_params(**case["params"])
    n = len(case["uniforms"])
    logits = np.tile(np.asarray(case["logits"], dtype=np.float32), (n, 1))
    H = len(case["history"])
    hist = np.tile(np.asarray(case["history"], dtype=np.int32), n)
    offs = (np.arange(n + 1) * H).astype(np.int32)
    toks, flags, _ = gpu_sampler.sample_rows(logits, hist, offs,
                                             np.asarray(case["uniforms"], np.float32), p)
    assert (toks == case["expect"]).all(), (case["src"], toks)


def test_peaked_head_single_row(gpu_sampler, oracle):
    wl = workloads.peaked_head()
    full_check(gpu_sampler, oracle, wl, label="peaked_head")
    wl = workloads.peaked_head(greedy=True)
    full_check(gpu_sampler, oracle, wl, probs=False, label="peaked_head greedy")


@pytest.mark.parametrize("greedy", [False, True])
def test_peaked_head_many_rows(gpu_sampler, oracle, greedy):
    wl = workloads.peaked_head(B=96, seed=21, greedy=greedy)
    full_check(gpu_sampler, oracle, wl, probs=not greedy, label="peaked_head x96")


def test_zipf_ranked_full_size(gpu_sampler, oracle):
    wl = workloads.zipf_ranked()
    rep = full_check(gpu_sampler, oracle, wl, probs=True, label="zipf_ranked 256x128256")
    print("zipf_ranked parity", rep)


@pytest.mark.parametrize("name", ["zipf_ranked", "high_entropy_nucleus"])
def test_host_arrays_sliced_copies(gpu_sampler, oracle, name):
    """ncb_sample_rows with host arrays: batches of 16 MiB and more go in
    slices (each sliced call samples its rows while the next slice copies);
    the tokens, flags and probabilities equal the oracle's for the whole
    batch."""
    wl = getattr(workloads, name)()
    if name == "high_entropy_nucleus":
        sel = slice(0, 96)  # 96 x 151936 rows: 58 MB, six slices
        offs = np.asarray(wl["hist_offsets"], np.int64)
        wl = dict(wl, logits=np.ascontiguousarray(wl["logits"][sel]),
                  hist_ids=np.ascontiguousarray(wl["hist_ids"][offs[0]:offs[96]]),
                  hist_offsets=offs[:97].copy(), uniforms=np.ascontiguousarray(wl["uniforms"][sel]))
    p = native.make_params(**wl["params"])
    want_probs = name == "zipf_ranked"
    gt, gf, gp = gpu_sampler.sample_rows(wl["logits"], wl["hist_ids"],
                                         np.asarray(wl["hist_offsets"], np.int32), wl["uniforms"],
                                         p, want_probs=want_probs)
    ot, of, op = run_oracle(oracle, wl, oracle.EXP_CR, want_probs=want_probs)
    assert_exact(gt, gf.astype(np.uint32), ot, of, name + " host arrays")
    if want_probs:
        assert np.array_equal(gp, op)


@pytest.mark.parametrize("mantissa_bits", [7, 3])
def test_quantised_logits_with_ties(gpu_sampler, oracle, mantissa_bits):
    # logits of a bf16 model (7 mantissa bits) and coarser: many exactly equal
    # values around the K-th, across the kernel's warps and at the draw
    wl = workloads.zipf_ranked(B=64, V=50000, H=256, seed=31)
    lg = wl["logits"].astype(np.float32)
    m, e = np.frexp(lg)
    q = np.float32(2.0 ** (mantissa_bits + 1))
    wl["logits"] = np.ldexp(np.round(m * q) / q, e).astype(np.float32)
    rep = full_check(gpu_sampler, oracle, wl, probs=True, label=f"quantised {mantissa_bits}")
    print("quantised parity", mantissa_bits, rep)


def test_zipf_history_nucleus_full_size(gpu_sampler, oracle):
    wl = workloads.zipf_history_nucleus()
    rep = full_check(gpu_sampler, oracle, wl, probs=True, label="zipf_history_nucleus 32x32000")
    print("zipf_history_nucleus parity", rep)


def test_high_entropy_nucleus_rows(gpu_sampler, oracle):
    wl = workloads.high_entropy_nucleus(B=48)
    rep = full_check(gpu_sampler, oracle, wl, probs=True, label="high_entropy_nucleus 48 rows")
    print("high_entropy_nucleus parity", rep)


def test_high_entropy_nucleus_full_batch(gpu_sampler, oracle):
    """All 1024 rows of the 1024 x 151936 nucleus batch: every one of a row's
    151936 weights enters the sequential sum that decides its token."""
    wl = workloads.high_entropy_nucleus()
    rep = full_check(gpu_sampler, oracle, wl, probs=False, label="high_entropy_nucleus 1024 rows")
    print("high_entropy_nucleus full batch parity", rep)


def test_vocab_sharded_workload_single_gpu(gpu_sampler, oracle):
    wl = workloads.vocab_sharded(B=32)
    full_check(gpu_sampler, oracle, wl, probs=False, label="vocab_sharded 32x262144")


@pytest.mark.parametrize("splits", ["1", "3", "7", "16"])
def test_column_splits_merge(navlib, oracle, monkeypatch, splits):
    from neuraval_b200.sampler import CudaTokenSampler
    monkeypatch.setenv("NAVSAMPLER_SPLITS", splits)  # read when the handle is created
    with CudaTokenSampler(0, max_rows=32, max_vocab=50000, max_history=512) as s:
        wl = workloads.zipf_ranked(B=24, V=50000, H=300, seed=9)
        full_check(s, oracle, wl, label=f"splits={splits}")
        wl = workloads.peaked_head(B=24, V=50000, seed=5, greedy=True)
        full_check(s, oracle, wl, probs=False, label=f"greedy splits={splits}")


def _edge_rows(V, rng):
    rows = [rng.standard_normal(V).astype(np.float32) * 2,
            np.round(rng.standard_normal(V)).astype(np.float32),      # heavy ties
            np.zeros(V, np.float32),                                  # all equal
            np.where(rng.random(V) < 0.5, -np.inf, rng.standard_normal(V)).astype(np.float32),
            np.full(V, -np.inf, np.float32),                          # no finite max
            rng.standard_normal(V).astype(np.float32)]
    r = rng.standard_normal(V).astype(np.float32)
    r[V // 2] = np.nan
    rows.append(r)
    r = rng.standard_normal(V).astype(np.float32)
    r[V - 1] = np.inf
    rows.append(r)
    r = rng.standard_normal(V).astype(np.float32)
    r[0] = -0.0
    r[1:2] = 0.0
    r[2:] = -1
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("V", [1, 3, 5, 1001, 8195, 40003])
@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("mode", ["topk", "full", "greedy", "bigk"])
def test_edge_cases(gpu_sampler, oracle, V, offset, mode):
    rng = np.random.default_rng(V * 7 + offset)
    logits = _edge_rows(V, rng)
    B = logits.shape[0]
    Hs = rng.integers(0, 40, B)
    Hs[0] = 0
    hist = np.concatenate([rng.integers(-5, V + 5, h) for h in Hs]).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(Hs)]).astype(np.int32)
    params = dict(temperature=0.9, top_p=0.8, repetition_penalty=1.3, frequency_penalty=0.25,
                  presence_penalty=0.1)
    if mode == "topk":
        params["top_k"] = max(1, min(50, V - 1))
    elif mode == "full":
        params["top_k"] = native.INT_MAX
    elif mode == "bigk":
        params["top_k"] = max(1, min(1500, V - 1))
        params["top_p"] = 1.0
    else:
        params["greedy"] = True
    wl = dict(logits=logits, hist_ids=hist, hist_offsets=offs,
              uniforms=rng.random(B).astype(np.float32), params=params)
    gt, gf, gp = run_gpu(gpu_sampler, wl, want_probs=(mode != "greedy"), offset=offset)
    ot, of, op = run_oracle(oracle, wl, oracle.EXP_CR, want_probs=(mode != "greedy"))
    assert_exact(gt, gf, ot, of, f"edge V={V} off={offset} {mode}")
    if mode != "greedy":
        ok = gt >= 0
        assert np.array_equal(gp[ok], op[ok]), f"probs V={V} {mode}"


def test_empty_batch_is_a_noop(gpu_sampler):
    import torch
    z = torch.zeros((0, 10), dtype=torch.float32, device="cuda")
    offs = torch.zeros(1, dtype=torch.int32, device="cuda")
    t = torch.zeros(0, dtype=torch.int32, device="cuda")
    gpu_sampler.sample_rows_device(z, None, offs, t, native.make_params(top_k=5), t)


def test_capacity_and_argument_errors(gpu_sampler):
    import torch
    p = native.make_params(top_k=5)
    big = torch.zeros((1, 300000), dtype=torch.float32, device="cuda")
    offs = torch.zeros(2, dtype=torch.int32, device="cuda")
    u = torch.zeros(1, dtype=torch.float32, device="cuda")
    t = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(native.NcbError) as e:
        gpu_sampler.sample_rows_device(big, None, offs, u, p, t)
    assert e.value.status == native.NCB_ERROR_CAPACITY
    with pytest.raises(native.NcbError) as e:
        gpu_sampler.sample_rows_device(big[:, :10], None, offs, u,
                                       native.make_params(temperature=0.0), t)
    assert e.value.status == native.NCB_ERROR_INVALID_ARGUMENT


def test_history_beyond_capacity_is_flagged(navlib):
    import torch
    from neuraval_b200.sampler import CudaTokenSampler
    with CudaTokenSampler(0, max_rows=2, max_vocab=1000, max_history=8) as s:
        rng = np.random.default_rng(1)
        wl = dict(logits=rng.standard_normal((2, 1000)).astype(np.float32),
                  hist_ids=np.concatenate([np.arange(20), np.arange(3)]).astype(np.int32),
                  hist_offsets=np.array([0, 20, 23], np.int32),
                  uniforms=np.array([0.5, 0.5], np.float32),
                  params=dict(temperature=1.0, top_k=10, frequency_penalty=0.5))
        gt, gf, _ = run_gpu(s, wl)
        assert gt[0] == -1 and gf[0] & native.FLAG_BAD_HISTORY
        assert gt[1] >= 0 and not gf[1] & native.FLAG_BAD_HISTORY
