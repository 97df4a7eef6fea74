"""Parity of the bucketed full-vocabulary kernel (top-k >= V, or above the top-k
kernels' limit, with no probability output) with the oracle, bit for bit, and
that the kernel settles the rows itself: the hand-over to the full-sort kernel
stays at zero on ordinary rows."""
from __future__ import annotations

import numpy as np
import pytest

from tests.gpu_util import assert_exact, run_gpu, run_oracle
from neuraval_b200 import native, workloads
from neuraval_b200.sampler import fast_exp_max_steps

pytestmark = pytest.mark.gpu

FAST_EXP_STEPS = 21  # the bound the kernel's rounding decisions rely on (x in [-17, 0])


def check(sampler, oracle, wl, label, max_full_sort=0):
    before = sampler.full_sort_rows()
    gt, gf, _ = run_gpu(sampler, wl)
    redone = sampler.full_sort_rows() - before
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    assert_exact(gt, gf, ot, of, label)
    assert redone <= max_full_sort, f"{label}: {redone} rows redone by the full-sort kernel"
    return redone


def _rows(B, V, rng, sigma, H, hist_lo=0):
    logits = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(sigma))
    Hs = np.full(B, H)
    hist = rng.integers(hist_lo, V, int(Hs.sum())).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(Hs)]).astype(np.int32)
    return logits, hist, offs


def test_fast_exp_bound_over_the_kernels_domain(navlib):
    assert fast_exp_max_steps(-17.0, 0.0) <= FAST_EXP_STEPS


def test_zipf_history_nucleus_full_batch(gpu_sampler, oracle):
    check(gpu_sampler, oracle, workloads.zipf_history_nucleus(), "zipf_history_nucleus 32x32000")


def test_high_entropy_nucleus_rows(gpu_sampler, oracle):
    check(gpu_sampler, oracle, workloads.high_entropy_nucleus(B=64, seed=11),
          "high_entropy_nucleus 64x151936")


DISTRIBUTIONS = [
    (32000, 0.05, 1.0, 0.9),     # nearly flat: every value relevant, dense buckets
    (32000, 6.0, 0.6, 0.95),     # very peaked: few relevant values
    (50257, 2.0, 1.3, 0.8),
    (50257, 1.0, 0.9, 1.0),      # no top-p: the draw over every candidate
    (151936, 0.3, 1.0, 0.99),
    (151936, 3.0, 0.8, 0.5),
    (262144, 1.5, 1.1, 0.97),
]


def _distribution(V, sigma, temperature, top_p):
    rng = np.random.default_rng(V + int(sigma * 100))
    logits, hist, offs = _rows(24, V, rng, sigma, 128)
    params = dict(temperature=temperature, top_p=top_p, top_k=native.INT_MAX,
                  repetition_penalty=1.2, presence_penalty=0.1)
    return dict(logits=logits, hist_ids=hist, hist_offsets=offs,
                uniforms=rng.random(24).astype(np.float32), params=params)


@pytest.mark.parametrize("V,sigma,temperature,top_p", DISTRIBUTIONS)
def test_distributions(gpu_sampler, oracle, V, sigma, temperature, top_p):
    check(gpu_sampler, oracle, _distribution(V, sigma, temperature, top_p),
          f"V={V} sigma={sigma} T={temperature} p={top_p}")


def _tiled(wl, copies):
    """The batch repeated `copies` times (rows, histories and uniforms)."""
    B = wl["logits"].shape[0]
    offs = np.asarray(wl["hist_offsets"])
    lens = np.tile(np.diff(offs), copies)
    return dict(logits=np.tile(wl["logits"], (copies, 1)),
                hist_ids=np.tile(np.asarray(wl["hist_ids"])[:offs[B]], copies),
                hist_offsets=np.concatenate([[0], np.cumsum(lens)]).astype(np.int32),
                uniforms=np.tile(wl["uniforms"], copies), params=wl["params"])


@pytest.mark.parametrize("case", [f"dist{i}" for i in range(len(DISTRIBUTIONS))] +
                         ["high_entropy", "zipf_history", "top_k_1500"])
def test_batch_shapes_agree(gpu_sampler, case):
    """A batch of at most one row per SM runs one 1024-thread CTA per SM, a
    larger one two 512-thread CTAs per SM with fewer, wider buckets (where two
    fit an SM's shared memory): the same rows give the same tokens and flags
    either way (the small batch is checked against the oracle by the tests
    above)."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if case.startswith("dist"):
        wl = _distribution(*DISTRIBUTIONS[int(case[4:])])
    elif case == "high_entropy":
        wl = workloads.high_entropy_nucleus(B=64, seed=11)
    elif case == "zipf_history":
        wl = workloads.zipf_history_nucleus()
    else:
        rng = np.random.default_rng(1500)
        logits, hist, offs = _rows(24, 128256, rng, 1.0, 256)
        wl = dict(logits=logits, hist_ids=hist, hist_offsets=offs,
                  uniforms=rng.random(24).astype(np.float32),
                  params=dict(temperature=0.8, top_p=0.9, top_k=1500, repetition_penalty=1.1))
    B = wl["logits"].shape[0]
    assert B <= sms
    copies = sms // B + 1
    before = gpu_sampler.full_sort_rows()
    st, sf, _ = run_gpu(gpu_sampler, wl)
    bt, bf, _ = run_gpu(gpu_sampler, _tiled(wl, copies))
    assert gpu_sampler.full_sort_rows() == before, case
    assert len(bt) == B * copies > sms
    np.testing.assert_array_equal(bt, np.tile(st, copies), err_msg=case)
    np.testing.assert_array_equal(bf, np.tile(sf, copies), err_msg=case)


@pytest.mark.parametrize("top_k,top_p", [(1500, 0.9), (2000, 1.0), (40000, 0.95)])
def test_large_top_k_cut(gpu_sampler, oracle, top_k, top_p):
    rng = np.random.default_rng(top_k)
    logits, hist, offs = _rows(24, 128256, rng, 1.0, 256)
    params = dict(temperature=0.8, top_p=top_p, top_k=top_k, repetition_penalty=1.1)
    wl = dict(logits=logits, hist_ids=hist, hist_offsets=offs,
              uniforms=rng.random(24).astype(np.float32), params=params)
    check(gpu_sampler, oracle, wl, f"top_k={top_k} top_p={top_p}")


@pytest.mark.parametrize("mantissa_bits", [10, 7, 3])
def test_quantised_logits(gpu_sampler, oracle, mantissa_bits):
    # bf16-like logits: many exactly equal values, exact halves on the grid
    wl = workloads.high_entropy_nucleus(B=16, seed=40 + mantissa_bits)
    m, e = np.frexp(wl["logits"] * np.float32(4.0))
    q = np.float32(2.0 ** (mantissa_bits + 1))
    wl["logits"] = np.ldexp(np.round(m * q) / q, e).astype(np.float32)
    # three mantissa bits leave buckets of tens of thousands of equal values,
    # which go to the full-sort kernel
    check(gpu_sampler, oracle, wl, f"quantised {mantissa_bits}",
          max_full_sort=16 if mantissa_bits <= 3 else 0)


def test_degenerate_rows(gpu_sampler, oracle):
    V = 40003
    rng = np.random.default_rng(5)
    rows = [np.zeros(V, np.float32),                                  # all equal
            np.where(rng.random(V) < 0.5, 1.0, 0.0).astype(np.float32),  # two values
            np.full(V, -30.0, np.float32),                            # one value far above
            rng.standard_normal(V).astype(np.float32) * np.float32(40.0)]  # very wide
    rows[2][123] = 5.0
    logits = np.stack(rows)
    B = logits.shape[0]
    offs = np.zeros(B + 1, np.int32)
    params = dict(temperature=1.0, top_p=0.7, top_k=native.INT_MAX)
    wl = dict(logits=logits, hist_ids=np.zeros(0, np.int32), hist_offsets=offs,
              uniforms=np.array([0.3, 0.999, 0.5, 0.1], np.float32), params=params)
    check(gpu_sampler, oracle, wl, "degenerate rows", max_full_sort=2)


@pytest.mark.parametrize("V", [1, 3, 5, 1001, 8195])
@pytest.mark.parametrize("offset", [0, 1])
def test_small_and_unaligned_rows(gpu_sampler, oracle, V, offset):
    rng = np.random.default_rng(V * 3 + offset)
    B = 8
    logits = rng.standard_normal((B, V)).astype(np.float32) * np.float32(2.0)
    Hs = rng.integers(0, 20, B)
    hist = np.concatenate([rng.integers(-3, V + 3, h) for h in Hs]).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(Hs)]).astype(np.int32)
    params = dict(temperature=0.9, top_p=0.8, top_k=native.INT_MAX, repetition_penalty=1.3,
                  frequency_penalty=0.25, presence_penalty=0.1)
    wl = dict(logits=logits, hist_ids=hist, hist_offsets=offs,
              uniforms=rng.random(B).astype(np.float32), params=params)
    gt, gf, _ = run_gpu(gpu_sampler, wl, offset=offset)
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    assert_exact(gt, gf, ot, of, f"V={V} offset={offset}")


def test_nonfinite_rows_are_flagged(gpu_sampler, oracle):
    rng = np.random.default_rng(9)
    logits = rng.standard_normal((3, 5000)).astype(np.float32)
    logits[0, 17] = np.nan
    logits[1, 4000] = np.inf
    logits[2, :] = -np.inf
    wl = dict(logits=logits, hist_ids=np.zeros(0, np.int32), hist_offsets=np.zeros(4, np.int32),
              uniforms=np.array([0.5, 0.5, 0.5], np.float32),
              params=dict(temperature=1.0, top_p=0.9, top_k=native.INT_MAX))
    check(gpu_sampler, oracle, wl, "non-finite rows")


@pytest.mark.parametrize("seed", range(12))
def test_randomized_sweep(gpu_sampler, oracle, seed):
    # random row shapes, value distributions (normal, heavy-tailed, quantised,
    # Zipf-ranked), temperatures, top-p, large top-k and all three penalties
    rng = np.random.default_rng(1000 + seed)
    B = 16
    V = int(rng.choice([1000, 4099, 32000, 50257, 128256, 151936]))
    kind = seed % 4
    if kind == 0:
        logits = rng.standard_normal((B, V)).astype(np.float32) * np.float32(rng.uniform(0.05, 8.0))
    elif kind == 1:
        logits = rng.standard_t(2.5, (B, V)).astype(np.float32) * np.float32(rng.uniform(0.3, 3.0))
    elif kind == 2:
        lg = rng.standard_normal((B, V)).astype(np.float32) * np.float32(2.0)
        m, e = np.frexp(lg)
        q = np.float32(2.0 ** int(rng.integers(5, 11)))
        logits = np.ldexp(np.round(m * q) / q, e).astype(np.float32)
    else:
        wl = workloads.zipf_ranked(B=B, V=V, H=64, seed=seed)
        logits = wl["logits"]
    H = int(rng.integers(0, 600))
    hist = rng.integers(0, V, B * H).astype(np.int32)
    offs = (np.arange(B + 1) * H).astype(np.int32)
    top_k = native.INT_MAX if rng.random() < 0.7 else int(rng.integers(1100, max(1101, V)))
    params = dict(temperature=float(rng.uniform(0.3, 2.0)), top_p=float(rng.choice([rng.uniform(0.05, 0.999), 1.0])),
                  top_k=top_k, repetition_penalty=float(rng.uniform(0.8, 1.6)),
                  frequency_penalty=float(rng.choice([0.0, rng.uniform(-0.2, 0.8)])),
                  presence_penalty=float(rng.choice([0.0, rng.uniform(-0.2, 0.8)])))
    wl = dict(logits=np.ascontiguousarray(logits), hist_ids=hist, hist_offsets=offs,
              uniforms=rng.random(B).astype(np.float32), params=params)
    check(gpu_sampler, oracle, wl, f"sweep seed={seed} V={V} kind={kind} {params}", max_full_sort=2)
